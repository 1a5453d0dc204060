#!/usr/bin/env python
"""bench.py -- the HE-LRM embedding PCMM on B200.

One step = one batch of 64 encrypted Criteo-shaped queries through the
embedding layer, the reference's hot path (examples/criteo/dlrm.py:226-229
-> orion/nn/linear.py:99-140): the BSGS diagonal linear transform of the
26-table block-diagonal 416 x 4224 matrix (512 diagonals; `--bsgs-ratio`,
default 8: bs 64, 8 giant groups) on ciphertexts at LogN 16 with 24 limbs
+ 4 special primes (dnum 4), then the rescale and the 6 hybrid-fold
rotations.  Inputs are seeded synthetic data with the reference's shapes
(the Criteo dataset is not available), weights N(0, 0.05), queries
Zipf(1.05).  On one GPU the line also carries the config-3 primitive
microbenchmark, a compact config-4 forward (the whole bootstrapped HE-LRM
network), the CPU baseline and a level-4 secondary.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    python bench.py --mode tables        # the 26 tables sharded over the ranks
    python bench.py --mode helrm         # config 4: the end-to-end forward

Under torchrun each rank runs its own batch (query-batch data parallelism,
keys and diagonals replicated, no data-path collective): weak scaling.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "HE-LRM encrypted inferences/sec; embedding PCMM ms; key-switch HBM GB/s"
UNIT = "inferences/s"
HBM_FALLBACK_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--mode", default="dp", choices=["dp", "tables", "helrm"],
                    help="dp: each rank its own batch (weak scaling); tables: the 26 tables split across the "
                         "ranks, one batch, partial ciphertexts summed by one NCCL reduce (strong scaling); "
                         "helrm: BASELINE config 4, the whole bootstrapped HE-LRM forward, each rank its own batch")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--level", type=int, default=23, help="PCMM input level (23 = all 24 limbs)")
    ap.add_argument("--bsgs-ratio", type=float, default=8.0,
                    help="the embedding layer's bsgs_ratio (orion/nn/linear.py:149; bs = ceil(sqrt(512 * ratio)))")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cfg3", action="store_true", help="skip the config-3 primitive microbenchmark")
    ap.add_argument("--no-cfg4", action="store_true",
                    help="skip the compact config-4 forward (one warm-up, one timed step) of the default line")
    ap.add_argument("--cpu-threads", type=int, default=0, help="oracle threads (0 = all host cores)")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: same 512-diagonal PCMM on 8 q limbs + 2 special primes (dnum 4, "
                         "so four digits as in the headline), so an ncu capture keeps a few GB on the device")
    args = ap.parse_args()
    if args.small:
        args.level = min(args.level, 7)
    return args


# --------------------------------------------------------------------------- distributed plumbing
class Dist:
    """One process per GPU (torchrun env vars).  NCCL on GPU hosts; gloo when
    no GPU is visible or HELRM_DIST_BACKEND=gloo (the CPU tests of this
    plumbing).  The only collectives are a barrier around the timed region
    and the max of the per-rank times: ciphertext batches are independent,
    so the data path has no exchange."""

    def __init__(self, backend: str | None = None, timeout_s: float = 120.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        self.backend = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            backend = backend or os.environ.get("HELRM_DIST_BACKEND") or \
                ("nccl" if torch.cuda.is_available() else "gloo")
            timeout = datetime.timedelta(seconds=timeout_s)
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(backend, timeout=timeout)
            self.pg = dist
            self.backend = backend

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        """max over ranks of a per-rank device time"""
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device="cuda" if self.backend == "nccl" else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


def whole_job_rate(world: int, batch: int, steps: int, t_max_s: float) -> float:
    """inferences/s of the whole job: every rank ran `steps` steps of `batch`
    ciphertexts (one query each); the job took the slowest rank's time"""
    return world * batch * steps / t_max_s


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            sel = str(device_index)
        self.sel = sel

    def start(self):
        """Start sampling and wait for the first sample: nvidia-smi's start-up
        (NVML initialisation) stalls the GPU's work submission for tens of
        milliseconds and must not fall inside the timed region."""
        self.first = ""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.sel, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        import select
        if select.select([self.proc.stdout], [], [], 10.0)[0]:
            self.first = self.proc.stdout.readline()

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        # the first sample (read in start()) precedes the timed region
        rows = [r.split(", ") for r in out.strip().splitlines() if r.strip()]
        sm = [float(r[0]) for r in rows if len(r) >= 8 and r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if len(r) >= 8 and r[1].replace(".", "").isdigit()]
        pw = [float(r[2]) for r in rows if len(r) >= 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 8 for i in range(4) if r[4 + i].strip() == "Active"})
        loaded = [s for s in sm if s > 0.5 * (max(mx) if mx else 0)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(rows), "reasons": reasons}


# --------------------------------------------------------------------------- workload
def build_workload(batch: int, seed: int):
    from helrm_b200 import workload as W
    V = W.cfg2_vocab()
    M = W.block_diag_matrix(V, 64, 16, 0.05, seed=0)
    d, rot = W.diagonalize(M, 32768, "hybrid")
    diags = d[(0, 0)]
    ks = sorted(diags)
    q = W.zipf_queries(V, batch, seed=seed)
    xs = [W.selector(qq, V) for qq in q]
    return M, ks, diags, rot, xs


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def ncu_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            t = json.load(f)
        return t.get(kernel)
    except Exception:
        return None


# --------------------------------------------------------------------------- CPU baseline (oracle)
def oracle_for_cfg2():
    from oracle import oracle as om
    from helrm_b200.params import CFG2, CFG2_DNUM
    main, aux = om.scheme_primes(CFG2.logq, CFG2.logp, CFG2.logn)
    return om, om.Oracle(CFG2.logn, main, aux, CFG2_DNUM)


def cpu_operands_own(o, om, ks, diags, rot, x, level, threads, ratio, seed=4242):
    """Keys, extended-basis diagonals and one ciphertext for the oracle,
    made on the CPU from its own seed (the reference arm has no GPU)."""
    from concurrent.futures import ThreadPoolExecutor
    from helrm_b200 import workload as W
    from helrm_b200.params import CFG2
    plan = W.bsgs_plan(ks, ratio, o.N // 2)
    nq = level + 1
    scale = float(1 << CFG2.logscale)
    # one task per diagonal / key, each single-threaded inside the oracle
    # (ctypes releases the GIL, so the pool runs them in parallel)
    om.set_threads(1)
    sk = o.secret_ntt(o.sample_secret(seed, CFG2.h))
    gal = sorted({o.galois(dd) for dd in plan["rotation_keys"]} |
                 {o.galois((o.N // 2) >> i) for i in range(1, rot + 1)})
    with ThreadPoolExecutor(max_workers=threads) as ex:
        pts = list(ex.map(lambda k: o.encode(W.preroll(diags[k], k // plan["stride"], plan["stride"]), nq, scale,
                                             ext=True), ks))
        keys = dict(zip(gal, ex.map(lambda g: o.rotation_key(sk, seed, g), gal)))
    v = np.zeros(o.N // 2)
    v[:len(x)] = x
    ct = o.encrypt(sk, o.encode(v, nq, scale), 7)
    return ct, pts, plan["stride"], keys


def cpu_pcmm_times(o, om, ct, ks, pts, stride, keys, rot, threads, reps=1):
    """The same PCMM step (LT + rescale + fold) for one ciphertext on the
    oracle with `threads` host threads: (per-rep seconds, last output)."""
    om.set_threads(threads)
    times, out = [], None
    for _ in range(reps):
        t1 = time.time()
        out = o.pcmm(ct, ks, pts, stride, keys, rot)
        times.append(time.time() - t1)
    om.set_threads(1)
    return times, out


# --------------------------------------------------------------------------- reference arm
def run_reference(args, dist):
    """The reference's CPU implementation of the path cannot be built here
    (Lattigo is Go, absent with its module cache; Cheddar is not vendored),
    so the arm times the oracle port on all host cores: one ciphertext of
    the same PCMM per step."""
    if dist.rank != 0:
        return
    threads = args.cpu_threads or os.cpu_count() or 1
    M, ks, diags, rot, xs = build_workload(1, seed=100)
    om, o = oracle_for_cfg2()
    t0 = time.time()
    ct, pts, stride, keys = cpu_operands_own(o, om, ks, diags, rot, xs[0], args.level, threads, args.bsgs_ratio)
    setup = time.time() - t0
    times_all, _ = cpu_pcmm_times(o, om, ct, ks, pts, stride, keys, rot, threads, reps=args.warmup + args.steps)
    times = times_all[args.warmup:]
    ms = 1000.0 * sum(times) / len(times)
    value = 1000.0 / ms
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": cfg_dict(args, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "1 ciphertext of the cfg2 PCMM per step (LT + rescale + 6 fold rotations), "
                                   f"oracle port on {threads} threads; Lattigo (Go) is not buildable here"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": setup,
    }
    print(json.dumps(line), flush=True)


def bs_of(ratio):
    """baby steps of the 512-diagonal transform (cheddar bindings.py:160-175 rule)"""
    return max(1, math.ceil(math.sqrt(512 * ratio)))


def cfg_dict(args, batch):
    d = {"workload": "cfg2: 26-table block-diagonal embedding PCMM (BASELINE configs[1])",
         "logN": 16, "slots": 32768, "q_limbs": 24, "q_bits": 36, "special_primes": 4, "p_bits": 60,
         "dnum": 4, "pcmm_level": args.level, "matrix": "416x4224 block-diagonal", "diagonals": 512,
         "bsgs_ratio": args.bsgs_ratio, "bs": bs_of(args.bsgs_ratio), "giant_groups": -(-512 // bs_of(args.bsgs_ratio)),
         "fold_rotations": 6, "batch_ciphertexts": batch,
         "queries_per_ciphertext": 1, "parallelism": f"dp{args.gpus} (query batch)",
         "l2": "inputs larger than L2 (1.5 GiB ciphertexts, 7 GiB diagonals, 5.7 GiB keys per step)"}
    if getattr(args, "small", False):
        d.update({"workload": "profiling case (NOT the headline): cfg2 PCMM on 8 q limbs + 2 special primes",
                  "q_limbs": 8, "special_primes": 2, "dnum": 4})
    return d


# --------------------------------------------------------------------------- B200 arm
REL_TOL = 2.0 ** -15   # north_star: decrypted embedding slots within 2^-15 relative


def read_profile(capi, _capi, steps):
    """per-kernel-class statistics of the library's CUDA-event profiler"""
    K = 16
    pms, pby, pwk = (ctypes.c_double * K)(), (ctypes.c_double * K)(), (ctypes.c_double * K)()
    pl = (ctypes.c_uint64 * K)()
    ncls = ctypes.c_int(0)
    _capi.check(capi.helrm_ProfileRead(pms, pby, pwk, pl, K, ctypes.byref(ncls)))
    buf = ctypes.create_string_buffer(64)
    raw = {}
    for i in range(ncls.value):
        capi.helrm_KernelClassName(i, buf, 64)
        if pl[i]:
            raw[buf.value.decode()] = (pms[i], pby[i], pwk[i], pl[i])
    kern = {}
    for nm, (ms_, by, wk, n) in raw.items():
        kern[nm] = {"ms_per_step": ms_ / steps, "launches_per_step": n / steps, "share": None,
                    "GBps": by / (ms_ * 1e6) if ms_ else None, "Gops": wk / (ms_ * 1e6) if ms_ else None}
    tot = sum(v["ms_per_step"] for v in kern.values()) or 1.0
    for v in kern.values():
        v["share"] = v["ms_per_step"] / tot
    return kern, raw


def run_b200(args, dist):
    import torch

    from helrm_b200 import B200Library, CKKSConfig, _capi
    from helrm_b200.params import CFG2, CFG2_DNUM

    dev = dist.local
    torch.cuda.set_device(dev)
    if args.small:
        cfg, dnum = CKKSConfig(logn=16, logq=[36] * 8, logp=[60] * 2, logscale=36, h=192), 4
    else:
        cfg, dnum = CFG2, CFG2_DNUM
    lib = B200Library(dnum=dnum, seed=1000 + dist.rank, device=dev)
    lib.setup_bindings(cfg)
    lib.GenerateSecretKey()
    M, ks, diags, rot, xs = build_workload(args.batch, seed=100 + dist.rank)
    info = lib.scheme_info()
    slots, N = info["slots"], info["N"]
    data = np.concatenate([diags[k].astype(np.float64) for k in ks])
    lt = lib.GenerateLinearTransform(ks, data, args.level, args.bsgs_ratio, "none")
    for k in lib.GetLinearTransformRotationKeys(lt):
        lib.GenerateLinearTransformRotationKey(k)
    for i in range(1, rot + 1):
        lib.AddRotationKey(slots >> i)
    scale = float(1 << CFG2.logscale)

    def encrypt_batch(level):
        out = []
        for x in xs:
            v = np.zeros(slots)
            v[:len(x)] = x
            pt = lib.Encode(list(v), level, scale)
            out.append(lib.Encrypt(pt))
            lib.DeletePlaintext(pt)
        return out

    cts = encrypt_batch(args.level)
    capi = _capi.load()

    def step(ids, t=lt):
        outs = lib.EvaluateLinearTransformBatch(t, ids)
        lib.RescaleBatch(outs)
        lib.HybridFoldBatch(outs, rot)
        return outs

    # correctness spot check outside the timed region: first ciphertext,
    # decrypted embedding slots against the cleartext product (relative
    # to the largest magnitude), residues kept for the CPU leg's comparison
    o = step(cts[:1])[0]
    gpu_out0 = lib.GetCiphertextData(o)
    got = np.array(lib.Decode(lib.Decrypt(o)))[:416]
    ref = M.astype(np.float64) @ xs[0]
    max_err = float(np.abs(got - ref).max())
    rel_err = max_err / float(np.abs(ref).max())
    correct = bool(rel_err <= REL_TOL)
    lib.DeleteCiphertext(o)

    def timed_steps(nsteps, ids, t=lt, profile=False):
        """nsteps steps on the library stream between CUDA events; returns
        (device ms, launches of this library in the region)"""
        lib.Synchronize()
        torch.cuda.synchronize()
        if profile:
            _capi.check(capi.helrm_ProfileEnable(1))
        n0 = ctypes.c_uint64(0)
        _capi.check(capi.helrm_GetLaunchCount(ctypes.byref(n0)))
        _capi.check(capi.helrm_TimerStart())
        for _ in range(nsteps):
            for oo in step(ids, t):
                lib.DeleteCiphertext(oo)
        ms = ctypes.c_double(0)
        _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
        n1 = ctypes.c_uint64(0)
        _capi.check(capi.helrm_GetLaunchCount(ctypes.byref(n1)))
        return ms.value, int(n1.value - n0.value)

    for _ in range(args.warmup):
        for oo in step(cts):
            lib.DeleteCiphertext(oo)
    lib.Synchronize()
    torch.cuda.synchronize()

    # ---- device-resident timed region (per-kernel profiling off)
    clocks = ClockSampler(dev)
    dist.barrier()
    torch.cuda.synchronize()
    lib.Synchronize()
    clocks.start()
    ms_dev, launches = timed_steps(args.steps, cts)
    clk = clocks.stop()
    torch.cuda.synchronize()
    dist.barrier()
    t_dev = dist.max(ms_dev / 1000.0)
    value = whole_job_rate(dist.world, args.batch, args.steps, t_dev)
    ms_step = 1000.0 * t_dev / args.steps

    # ---- a second pass over the same steps with per-kernel CUDA events on
    # the library stream: the kernel breakdown and the roofline's kernel
    # duration (the events add a little time, so this pass is not the headline)
    prof_steps = max(1, min(args.steps, 5))
    _capi.check(capi.helrm_ProfilerRange(1))
    ms_prof, _ = timed_steps(prof_steps, cts, profile=True)
    kern, raw = read_profile(capi, _capi, prof_steps)
    _capi.check(capi.helrm_ProfileEnable(0))
    _capi.check(capi.helrm_ProfilerRange(0))
    dom = max(kern, key=lambda k: kern[k]["ms_per_step"])
    dms, dby, _, dl = raw[dom]
    hbm, src = peaks()
    achieved = dby / (dms * 1e6)
    roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured"
                else "fallback 6.65 TB/s", "bytes_per_launch": dby / dl, "avg_launch_ms": dms / dl,
                "traffic": ncu_traffic(dom), "profiled_steps": prof_steps,
                "profiled_ms_per_step": ms_prof / prof_steps}
    keymult = kern.get("keymult", {}).get("GBps")

    # ---- secondary line (NOT the headline): the same PCMM with the selector
    # at level 4, where the reference's HE-LRM compiler places the embedding
    # input (examples/criteo/table2.py:212, examples/criteo/network.py:209-211)
    low = None
    if not args.small and args.level > 4 and dist.world == 1:
        # at 5 limbs the giant steps are cheap: the reference's default ratio
        # 2 (bs 32) is the faster split there
        lt4 = lib.GenerateLinearTransform(ks, data, 4, 2.0, "none")
        for k in lib.GetLinearTransformRotationKeys(lt4):
            lib.GenerateLinearTransformRotationKey(k)
        cts4 = encrypt_batch(4)
        for _ in range(args.warmup):
            for oo in step(cts4, lt4):
                lib.DeleteCiphertext(oo)
        ms4, _ = timed_steps(args.steps, cts4, lt4)
        low = {"note": "not the headline: selector at level 4 (5 q limbs), the reference's placement",
               "pcmm_level": 4, "bsgs_ratio": 2.0, "bs": bs_of(2.0), "ms_per_step": ms4 / args.steps,
               "value": args.batch * args.steps / (ms4 / 1000.0), "unit": UNIT}
        for c in cts4:
            lib.DeleteCiphertext(c)
        lib.DeleteLinearTransform(lt4)

    # ---- end to end through the C ABI with host buffers
    e2e = None
    if not args.no_e2e:
        nq_in, nq_out = args.level + 1, args.level
        words_in, words_out = 2 * nq_in * N, 2 * nq_out * N
        hin = torch.empty((args.batch, words_in), dtype=torch.int64, pin_memory=True)
        hout = torch.empty((args.batch, words_out), dtype=torch.int64, pin_memory=True)
        for i, c in enumerate(cts):
            hin[i].copy_(torch.from_numpy(lib.GetCiphertextData(c).reshape(-1).view(np.int64)))

        # pinned host buffers; uploads and read-backs go through the library's
        # transfer streams, so step i+1's upload and step i's read-back overlap
        # the arithmetic (every copy is still inside the timed region: the
        # timer stops after the last read-back has landed in host memory)
        in_ptrs = (ctypes.c_void_p * args.batch)(*[hin[i].data_ptr() for i in range(args.batch)])
        out_ptrs = (ctypes.c_void_p * args.batch)(*[hout[i].data_ptr() for i in range(args.batch)])

        def e2e_step():
            ids = (ctypes.c_int * args.batch)()
            _capi.check(capi.helrm_UploadCiphertextsAsync(in_ptrs, args.batch, args.level, 2, scale, ids))
            outs = step(list(ids))
            oa = (ctypes.c_int * len(outs))(*outs)
            _capi.check(capi.helrm_DownloadCiphertextsAsync(oa, len(outs), out_ptrs, words_out))
            for x in list(ids) + outs:
                lib.DeleteCiphertext(x)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        _capi.check(capi.helrm_TransferSync())
        dist.barrier()
        lib.Synchronize()
        hout.zero_()
        _capi.check(capi.helrm_TimerStart())
        for _ in range(args.steps):
            e2e_step()
        _capi.check(capi.helrm_TransferSync())
        ms2 = ctypes.c_double(0)
        _capi.check(capi.helrm_TimerStop(ctypes.byref(ms2)))
        # the read-back holds the last step's results: the first one must be
        # the spot-checked ciphertext's output, residue for residue
        back0 = hout[0].numpy().view(np.uint64).reshape(gpu_out0.shape)
        e2e_match = bool(np.array_equal(back0, gpu_out0))
        t_e2e = dist.max(ms2.value / 1000.0)
        e2e = {"value": whole_job_rate(dist.world, args.batch, args.steps, t_e2e), "unit": UNIT,
               "h2d_bytes_per_step": args.batch * words_in * 8, "d2h_bytes_per_step": args.batch * words_out * 8,
               "ms_per_step": 1000.0 * t_e2e / args.steps, "readback_matches_device_output": e2e_match}
        correct = correct and e2e_match

    # ---- CPU baseline: the oracle on the same ciphertext, diagonals and
    # switching keys as the GPU run (fetched from the library), at all host
    # cores and at one thread; its output residues must equal the GPU's
    cpu = None
    residues_match = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline and not args.small:
        threads = args.cpu_threads or os.cpu_count() or 1
        try:
            from helrm_b200 import workload as W
            om, o = oracle_for_cfg2()
            t0 = time.time()
            plan = W.bsgs_plan(ks, args.bsgs_ratio, slots)
            gal = sorted({o.galois(d) for d in plan["rotation_keys"]} |
                         {o.galois(slots >> i) for i in range(1, rot + 1)})
            keys = {g: lib.GetKeyData(g) for g in gal}
            pts = [lib.GetLinearTransformPlaintext(lt, k) for k in ks]
            ct0 = lib.GetCiphertextData(cts[0])
            setup = time.time() - t0
            tall, out_all = cpu_pcmm_times(o, om, ct0, ks, pts, plan["stride"], keys, rot, threads)
            residues_match = bool(np.array_equal(out_all, gpu_out0))
            t1, out_1 = cpu_pcmm_times(o, om, ct0, ks, pts, plan["stride"], keys, rot, 1)
            residues_match = residues_match and bool(np.array_equal(out_1, gpu_out0))
            cpu = {"value": 1.0 / tall[0], "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"1 ciphertext of the same PCMM (LT + rescale + {rot} fold rotations) on the oracle "
                             f"port with the GPU run's ciphertext, diagonals and keys: {tall[0]:.2f} s on "
                             f"{threads} threads, {t1[0]:.2f} s on 1 thread (operand fetch {setup:.1f} s untimed)",
                   "nproc": os.cpu_count(), "single_thread": {"value": 1.0 / t1[0], "unit": UNIT, "cores": 1,
                                                              "seconds": t1[0]},
                   "residues_match": residues_match,
                   "lattigo": go_probe()}
            del keys, pts
            correct = correct and residues_match
        except Exception as ex:  # the baseline must not sink the GPU line
            cpu = {"value": None, "unit": UNIT, "cores": threads, "kind": "port", "sample": f"failed: {ex}"}

    lib.DeleteScheme()

    # ---- config 3 (primitive microbenchmark), its own scheme; the
    # key-switch figure is the whole hoisted key switch (ModUp + KeyMult +
    # ModDown, NTTs included) over 32 rotations at batch 16
    cfg3 = None
    keyswitch = None
    if dist.world == 1 and not args.small and not args.no_cfg3:
        from helrm_b200 import microbench
        cfg3 = microbench.run(batches=(1, 16, 128), reps=3, device=dev)
        cfg3.append(microbench.run_table_matmul(device=dev))
        for r in cfg3:
            if r["op"] == "hoisted_keyswitch_R32" and r["batch"] == 16:
                keyswitch = {"GBps": r["GBps"], "frac_hbm": r["frac_hbm"], "batch": 16, "rotations": 32,
                             "ms": r["ms"], "what": "whole hoisted key switch (ModUp + KeyMult + ModDown, NTTs "
                                                    "included), algorithmic bytes: each operand read or written once"}

    # ---- config 4 (the whole HE-LRM forward), compact: three warm-up steps
    # (the first one checked against the cleartext), one timed step
    # (bench.py --mode helrm for the full line with the kernel breakdown
    # and e2e)
    cfg4 = None
    if dist.world == 1 and not args.small and not args.no_cfg4:
        try:
            cfg4 = helrm_measure(dist, args.batch, 1, 3, profile=False, e2e=False)
            cfg4["config"] = helrm_config(args)
            cfg4["note"] = ("config 4 end to end: HE-LRM inferences/s (the headline value above is the config-2 "
                            "embedding PCMM, one query per ciphertext)")
            correct = correct and cfg4["correct"]
        except Exception as ex:  # the PCMM line must not be lost with it
            cfg4 = {"value": None, "error": f"{type(ex).__name__}: {ex}"}

    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64", "data": "synthetic (seeded Criteo-shaped queries; dataset absent)",
            "config": cfg_dict(args, args.batch),
            "pcmm_ms_per_batch": ms_step, "keyswitch_GBps": keyswitch["GBps"] if keyswitch else None,
            "keyswitch": keyswitch, "keymult_GBps": keymult,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clk, "kernels": kern,
            "max_abs_err_embedding": max_err, "rel_err_embedding": rel_err, "rel_tol": REL_TOL,
            "residues_match": residues_match, "correct": correct, "level4_secondary": low, "cfg3": cfg3,
            "cfg4_helrm_forward": cfg4,
        }
        print(json.dumps(line), flush=True)
    if not correct:
        raise SystemExit("bench: results out of tolerance or residues differ from the oracle")


def run_b200_tables(args, dist):
    """Table-sharded embedding layer (helrm_b200/sharding.py): every rank
    holds the same keys and the same encrypted batch and evaluates only its
    contiguous group of tables (block height 64 at 8 ranks); the partial
    packed ciphertexts are summed as 64-bit residues by one NCCL reduce to
    rank 0, which imports the sum with every limb reduced modulo its prime.
    One step = one batch through the whole layer; the job's rate is the
    batch over the slowest rank's device time (strong scaling)."""
    import torch

    from helrm_b200 import B200Library, sharding as S
    from helrm_b200.params import CFG2, CFG2_DNUM

    dev = dist.local
    torch.cuda.set_device(dev)
    lib = B200Library(dnum=CFG2_DNUM, seed=1000, device=dev)  # one key set, shared by every rank
    lib.setup_bindings(CFG2)
    lib.GenerateSecretKey()
    M, ks, diags, rot, xs = build_workload(args.batch, seed=100)
    tables = S.table_shards(26, dist.world)[dist.rank]
    se = S.ShardedEmbedding(lib, M, tables, args.level)
    info = lib.scheme_info()
    slots, N = info["slots"], info["N"]
    scale = float(1 << CFG2.logscale)
    cts = []
    for x in xs:
        v = np.zeros(slots)
        v[:len(x)] = x
        pt = lib.Encode(list(v), args.level, scale)
        cts.append(lib.Encrypt(pt))
        lib.DeletePlaintext(pt)
    nq_out = args.level - 1
    words = 2 * nq_out * N
    part = torch.zeros((args.batch, words), dtype=torch.int64, device="cuda")
    tdist = dist.pg

    def step(keep=False):
        outs = se.evaluate(cts)
        out_scale = lib.GetCiphertextScale(outs[0])
        lib.CiphertextsToDevice(outs, part.data_ptr(), words)
        for o in outs:
            lib.DeleteCiphertext(o)
        S.exchange_sum(part, tdist, dst=0)
        merged = None
        if dist.rank == 0:
            torch.cuda.current_stream().synchronize()
            merged = lib.NewCiphertextsFromDeviceSum(part.data_ptr(), args.batch, args.level - 2, 2, out_scale)
            if not keep:
                for m in merged:
                    lib.DeleteCiphertext(m)
        lib.Synchronize()
        return merged

    merged = step(keep=True)
    correct, rel_err = True, None
    if dist.rank == 0:
        got = np.array(lib.Decode(lib.Decrypt(merged[0])))[:416]
        ref = M.astype(np.float64) @ xs[0]
        rel_err = float(np.abs(got - ref).max() / np.abs(ref).max())
        correct = rel_err <= REL_TOL
        for m in merged:
            lib.DeleteCiphertext(m)
    for _ in range(args.warmup):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    lib.Synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev)
    clocks.start()
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    e1.synchronize()
    clk = clocks.stop()
    dist.barrier()
    t = dist.max(e0.elapsed_time(e1) / 1000.0)
    value = args.batch * args.steps / t
    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * t / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u64",
            "data": "synthetic (seeded Criteo-shaped queries; dataset absent)",
            "config": dict(cfg_dict(args, args.batch), parallelism=f"tables{dist.world} (26 tables over "
                           f"{dist.world} ranks, one NCCL reduce of the packed partial ciphertexts)",
                           shard_tables=[len(r) for r in S.table_shards(26, dist.world)],
                           shard_block_height=se.bh, shard_diagonals=len(se.ks), shard_fold_rotations=se.rot,
                           shard_bsgs_ratio=se.ratio),
            "mode": "tables", "rel_err_embedding": rel_err, "correct": correct, "clocks": clk,
            "exchange_bytes_per_rank": args.batch * words * 8, "e2e": None,
        }
        print(json.dumps(line), flush=True)
    se.close()
    lib.DeleteScheme()
    if not correct:
        raise SystemExit("bench: sharded embedding out of tolerance")


LOGIT_TOL = 1e-3   # north_star: decrypted logits within 1e-3


def helrm_measure(dist, batch: int, steps: int, warmup: int, profile: bool = True, e2e: bool = True) -> dict:
    """the end-to-end HE-LRM forward (bottom MLP, the
    26-table embedding, top MLP, Orion's composite ReLUs and five
    bootstraps per query) over a batch of ciphertexts, one query each.
    A step is the forward of the batch with its inputs resident (the first
    warm-up step is checked against the cleartext forward); e2e adds the
    encoding and encryption of the host inputs and the decryption and
    decoding of the logits to host memory.  Returns the measurements (the
    rank's own; times are maxima over ranks)."""
    import torch

    from helrm_b200 import B200Library, _capi
    from helrm_b200 import helrm as H
    from helrm_b200 import workload as W
    from helrm_b200.params import CFG4, CFG4_DNUM

    dev = dist.local
    torch.cuda.set_device(dev)
    lib = B200Library(dnum=CFG4_DNUM, seed=2000 + dist.rank, device=dev)
    lib.setup_bindings(CFG4)
    lib.GenerateSecretKey()
    lib.GenerateRelinearizationKey()
    t0 = time.time()
    net = H.HELRM(lib, seed=0)
    setup_s = time.time() - t0
    dense = H.dense_inputs(batch, 100 + dist.rank)
    sel = net.selectors(W.zipf_queries(net.vocab, batch, seed=200 + dist.rank))
    d_cts, s_cts = net.encrypt(dense, sel)
    capi = _capi.load()

    def run(nsteps):
        for _ in range(nsteps):
            for o in net.forward(d_cts, s_cts):
                lib.DeleteCiphertext(o)

    outs = net.forward(d_cts, s_cts)
    got = net.decrypt(outs)
    for o in outs:
        lib.DeleteCiphertext(o)
    want = net.cleartext(dense, sel)
    exact = net.cleartext(dense, sel, poly=False)
    err_poly = float(np.abs(got - want).max())
    run(max(0, warmup - 1))
    lib.Synchronize()
    torch.cuda.synchronize()

    clocks = ClockSampler(dev)
    dist.barrier()
    torch.cuda.synchronize()
    lib.Synchronize()
    clocks.start()
    n0 = ctypes.c_uint64(0)
    _capi.check(capi.helrm_GetLaunchCount(ctypes.byref(n0)))
    _capi.check(capi.helrm_TimerStart())
    run(steps)
    ms = ctypes.c_double(0)
    _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
    n1 = ctypes.c_uint64(0)
    _capi.check(capi.helrm_GetLaunchCount(ctypes.byref(n1)))
    clk = clocks.stop()
    torch.cuda.synchronize()
    dist.barrier()
    t_dev = dist.max(ms.value / 1000.0)
    res = {"value": whole_job_rate(dist.world, batch, steps, t_dev), "unit": UNIT,
           "ms_per_step": 1000.0 * t_dev / steps, "steps": steps, "warmup": warmup, "batch_ciphertexts": batch,
           "gpu_launches": int(n1.value - n0.value), "clocks": clk,
           "max_abs_err_logits_vs_polynomial_cleartext": err_poly,
           "max_abs_err_logits_vs_relu_cleartext": float(np.abs(got - exact).max()),
           "composite_relu_approximation_error": float(np.abs(want - exact).max()),
           "logit_tol": LOGIT_TOL, "correct": err_poly <= LOGIT_TOL, "setup_s": setup_s, "plan": net.info()}

    if profile:  # one more step with the per-kernel profiler: breakdown and roofline
        _capi.check(capi.helrm_ProfilerRange(1))
        _capi.check(capi.helrm_ProfileEnable(1))
        lib.Synchronize()
        _capi.check(capi.helrm_TimerStart())
        run(1)
        ms_prof = ctypes.c_double(0)
        _capi.check(capi.helrm_TimerStop(ctypes.byref(ms_prof)))
        kern, raw = read_profile(capi, _capi, 1)
        _capi.check(capi.helrm_ProfileEnable(0))
        _capi.check(capi.helrm_ProfilerRange(0))
        dom = max(kern, key=lambda k: kern[k]["ms_per_step"])
        dms, dby, _, dl = raw[dom]
        hbm, src = peaks()
        achieved = dby / (dms * 1e6)
        res["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                           "frac": achieved / hbm,
                           "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured"
                           else "fallback 6.65 TB/s", "bytes_per_launch": dby / dl, "avg_launch_ms": dms / dl,
                           "traffic": None, "profiled_ms_per_step": ms_prof.value}
        res["kernels"] = kern

    if e2e:  # host inputs -> encode + encrypt -> forward -> decrypt + decode -> host logits
        def e2e_step():
            dc, sc = net.encrypt(dense, sel)
            outs = net.forward(dc, sc)
            net.decrypt(outs)
            for x in dc + sc + outs:
                lib.DeleteCiphertext(x)

        e2e_step()
        dist.barrier()
        lib.Synchronize()
        _capi.check(capi.helrm_TimerStart())
        for _ in range(steps):
            e2e_step()
        ms2 = ctypes.c_double(0)
        _capi.check(capi.helrm_TimerStop(ctypes.byref(ms2)))
        t_e2e = dist.max(ms2.value / 1000.0)
        slots = lib.scheme_info()["slots"]
        res["e2e"] = {"value": whole_job_rate(dist.world, batch, steps, t_e2e), "unit": UNIT,
                      "h2d_bytes_per_step": int(dense.size * 8 + sel.size * 8),
                      "d2h_bytes_per_step": int(batch * 2 * slots * 8),
                      "ms_per_step": 1000.0 * t_e2e / steps,
                      "what": "EncodeBatch of the host features and selectors, Encrypt, the forward, Decrypt, "
                              "Decode (decoded on the device; the slot values, re and im, are read back)"}
    res["memory"] = {"peak_device_mb": lib.GetPeakDeviceMemoryMB(), "key_mb": lib.GetKeyMemoryMB()}
    net.close()
    lib.DeleteScheme()
    return res


def helrm_config(args) -> dict:
    from helrm_b200 import helrm as H
    from helrm_b200.params import CFG4_DNUM
    return {"workload": "cfg4: end-to-end HE-LRM forward (BASELINE configs[3])", "logN": 16,
            "q_limbs_usable": 24, "q_bits": "50 + 23 x 36", "boot_primes": "11 x 60", "special_primes": "6 x 60",
            "dnum": CFG4_DNUM, "h": 192, "batch_ciphertexts": args.batch, "queries_per_ciphertext": 1,
            "bottom": list(H.BOTTOM), "top": [432] + list(H.TOP_HIDDEN) + [1], "relu": list(H.SIGN_DEGREES),
            "bsgs": "32 baby steps per transform (64 above 512 diagonals)",
            "parallelism": f"dp{args.gpus} (query batch)",
            "l2": "inputs larger than L2 (tens of GB of diagonals and keys per step)"}


def run_b200_helrm(args, dist):
    """bench.py --mode helrm: the config-4 line."""
    r = helrm_measure(dist, args.batch, args.steps, args.warmup, profile=True, e2e=not args.no_e2e)
    if dist.rank == 0:
        cfg = helrm_config(args)
        cfg["plan"] = r.pop("plan")
        line = {
            "metric": METRIC, "value": r.pop("value"), "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r.pop("ms_per_step"), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64",
            "data": "synthetic (seeded Criteo-shaped dense features and Zipf queries; random-init weights)",
            "config": cfg, "roofline": r.pop("roofline"),
            "cpu_baseline": {"value": None, "unit": UNIT, "cores": 0, "kind": "port",
                             "sample": "not run: one bootstrapped LogN-16 forward on the oracle port takes hours; "
                                       "the config-2 line carries the CPU baseline of the embedding product"},
            "e2e": r.pop("e2e", None), "gpu_launches": r.pop("gpu_launches"), "clocks": r.pop("clocks"),
        }
        line.update(r)
        print(json.dumps(line), flush=True)
    if not r["correct"]:
        raise SystemExit("bench: logits out of tolerance")


def go_probe() -> str:
    """Whether the reference's Lattigo CPU path could be built on this host:
    a Go toolchain and the lattigo/v6 module in the module cache."""
    import shutil
    go = shutil.which("go")
    if not go:
        return "unavailable on this box: no go toolchain on PATH"
    try:
        ver = subprocess.run([go, "version"], capture_output=True, text=True, timeout=20).stdout.strip()
        modc = subprocess.run([go, "env", "GOMODCACHE"], capture_output=True, text=True, timeout=20).stdout.strip()
    except Exception as ex:
        return f"go present, probe failed: {ex}"
    have = os.path.isdir(os.path.join(modc, "github.com", "baahl-nyu")) if modc else False
    return f"{ver}; lattigo module cache {'present' if have else 'absent'}"


class _Solo:
    """rank 0 of the reference arm: no process group (the other ranks exit
    at once, so nothing waits on rank 0's minutes of CPU work)"""
    world, rank, local = 1, 0, 0


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args, _Solo())
        return
    dist = Dist()
    try:
        if args.mode == "tables":
            run_b200_tables(args, dist)
        elif args.mode == "helrm":
            run_b200_helrm(args, dist)
        else:
            run_b200(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
