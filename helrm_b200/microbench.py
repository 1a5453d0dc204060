"""Config-3 primitive microbenchmark.

LogN 16, 24 q limbs (36-bit) + 4 special primes (60-bit), dnum 4:
forward/inverse NTT, automorphism, plaintext-ciphertext MAC over 32 pairs,
rescale, and the hoisted key switch for 32 rotations (one ModUp shared by
all of them), on batches of 1, 16 and 128 ciphertexts of seeded uniform
residues.  Every primitive runs through its kernel-level C-ABI entry point
on device buffers; times are CUDA events on the stream the kernels run on,
after warm-up, with inputs larger than L2.

    python -m helrm_b200.microbench [--batches 1,16,128] [--reps 5] [--ops ntt,ks]

Prints one JSON line per (primitive, batch): milliseconds per launch,
algorithmic GB/s (each operand read or written once per ciphertext) and
its fraction of the measured HBM copy bandwidth.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def run(batches=(1, 16, 128), reps=5, ops="ntt,intt,aut,mac,rescale,ks", rotations=32, device=0,
        emit=None) -> list[dict]:
    """Run the config-3 primitives and return one dict per (primitive,
    batch); `emit` (if given) is called on each as it is measured.  Creates
    and deletes its own scheme (the library holds one per process)."""
    import torch

    from helrm_b200 import B200Library, _capi
    from helrm_b200.params import CFG2, CFG2_DNUM

    ops = set(ops.split(",")) if isinstance(ops, str) else set(ops)
    results: list[dict] = []
    lib = B200Library(dnum=CFG2_DNUM, seed=5, device=device)
    lib.setup_bindings(CFG2)
    try:
        lib.GenerateSecretKey()
        info = lib.scheme_info()
        N, L, K, alpha = info["N"], info["L"], info["K"], info["alpha"]
        nq = L
        primes = lib.GetModuliChain()
        beta = (nq + alpha - 1) // alpha
        R = rotations
        if "ks" in ops:
            for k in range(1, R + 1):
                lib.AddRotationKey(k)
        capi = _capi.load()
        limb = N * 8
        peak, src = _peak()
        # an explicit stream: a NULL handle would select the library's own
        # stream, outside the events recorded here
        stream = torch.cuda.Stream()
        sp = ctypes.c_void_p(stream.cuda_stream)
        gen = torch.Generator(device="cuda").manual_seed(1)

        def residues(nct):
            t = torch.empty((nct, 2, nq, N), dtype=torch.int64, device="cuda")
            for i, q in enumerate(primes):
                t[:, :, i].random_(0, q, generator=gen)
            return t

        def timed(fn):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                fn()
            b.record(stream)
            b.synchronize()
            return a.elapsed_time(b) / reps

        def report(op, B, ms, nbytes, extra=None):
            gbs = nbytes / (ms * 1e6)
            line = {"op": op, "batch": B, "ms": ms, "GBps": gbs, "frac_hbm": gbs / peak,
                    "peak": f"{peak} GB/s ({src})"}
            line.update(extra or {})
            results.append(line)
            if emit:
                emit(line)

        ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        with torch.cuda.stream(stream):
            for B in batches:
                x = residues(B)
                rows = B * 2 * nq
                if "ntt" in ops:
                    ms = timed(lambda: _capi.check(capi.helrm_kernel_ntt(ptr(x), rows, nq, nq, 0, sp)))
                    report("ntt_forward", B, ms, 2 * 2 * nq * limb * B,
                           {"Gbutterflies_s": rows * (N // 2) * 16 / (ms * 1e6)})
                if "intt" in ops:
                    ms = timed(lambda: _capi.check(capi.helrm_kernel_ntt(ptr(x), rows, nq, nq, 1, sp)))
                    report("ntt_inverse", B, ms, 2 * 2 * nq * limb * B,
                           {"Gbutterflies_s": rows * (N // 2) * 16 / (ms * 1e6)})
                if "aut" in ops:
                    y = torch.empty_like(x)
                    g = pow(5, 7, 2 * N)
                    ms = timed(lambda: _capi.check(capi.helrm_kernel_automorphism(ptr(x), ptr(y), rows, g, sp)))
                    report("automorphism", B, ms, 2 * 2 * nq * limb * B)
                    del y
                if "rescale" in ops:
                    y = torch.empty((B, 2, nq - 1, N), dtype=torch.int64, device="cuda")
                    ms = timed(lambda: _capi.check(capi.helrm_kernel_rescale(ptr(x), ptr(y), nq, B, sp)))
                    report("rescale", B, ms, (2 * nq + 2 * (nq - 1)) * limb * B)
                    del y
                if "mac" in ops:
                    g = 32
                    cts = residues(g)
                    pts = torch.empty((g, nq, N), dtype=torch.int64, device="cuda")
                    for i, q in enumerate(primes):
                        pts[:, i].random_(0, q, generator=gen)
                    out = torch.empty((2, nq, N), dtype=torch.int64, device="cuda")
                    cp = (ctypes.c_void_p * g)(*[c.data_ptr() for c in cts])
                    pp = (ctypes.c_void_p * g)(*[p.data_ptr() for p in pts])

                    def mac_batch():
                        for _ in range(B):
                            _capi.check(capi.helrm_kernel_mac(cp, pp, g, nq, ptr(out), sp))
                    ms = timed(mac_batch)
                    report("mac_32_pairs", B, ms, (g * 3 * nq + 2 * nq) * limb * B)
                    del cts, pts, out
                if "ks" in ops:
                    # outputs [R][B][2][nq][N]; bound the device memory at ~12 GB
                    sub = max(1, min(B, int(12e9 // (R * 2 * nq * limb))))
                    outs = torch.empty((R, sub, 2, nq, N), dtype=torch.int64, device="cuda")
                    ks = (ctypes.c_int * R)(*range(1, R + 1))

                    def ks_batch():
                        for s0 in range(0, B, sub):
                            nb = min(sub, B - s0)
                            xs = x[s0:s0 + nb]
                            _capi.check(capi.helrm_kernel_rotate_hoisted(ptr(xs), nq, nb, ks, R, ptr(outs), sp))
                    ms = timed(ks_batch)
                    ne = nq + K
                    # algorithmic bytes of ModUp + KeyMult + ModDown, their
                    # NTTs included (each operand read or written once)
                    modup = nq * limb + beta * ne * limb
                    per_rot = beta * ne * limb + 2 * ne * limb + (2 * ne + 2 * nq) * limb + nq * limb
                    evk = 2 * beta * ne * limb * R * ((B + sub - 1) // sub)
                    report("hoisted_keyswitch_R32", B, ms, B * (modup + R * per_rot) + evk,
                           {"rotations": R, "launch_batch": sub})
                    del outs
                del x
                torch.cuda.empty_cache()
        stream.synchronize()
    finally:
        lib.DeleteScheme()
    return results


def run_table_matmul(rows=16, cols=64, level=23, reps=3, device=0) -> dict:
    """The IVE lookup's one-pass table product at LogN 16 (config 2/3
    primes): a rows x cols table of broadcast constants against cols
    ciphertexts, MulConstantMatMulNew (each input read once) against rows
    calls of MulConstantAccumNew (the inputs re-read per row), CUDA events
    on the library stream.  Algorithmic bytes: the inputs once and the
    outputs once."""
    import ctypes

    from helrm_b200 import B200Library, _capi
    from helrm_b200.params import CFG2, CFG2_DNUM

    lib = B200Library(dnum=CFG2_DNUM, seed=9, device=device)
    lib.setup_bindings(CFG2)
    try:
        lib.GenerateSecretKey()
        info = lib.scheme_info()
        slots, N = info["slots"], info["N"]
        rng = np.random.default_rng(0)
        cts = []
        for _ in range(cols):
            pt = lib.Encode(list(rng.uniform(-1, 1, slots)), level, float(1 << CFG2.logscale))
            cts.append(lib.Encrypt(pt))
            lib.DeletePlaintext(pt)
        kids = [lib.EncodeConstantNew(float(v), level, 2.0 ** 20) for v in rng.uniform(-1, 1, rows * cols)]
        tab = lib.PackConstantTableNew(kids, rows)
        capi = _capi.load()

        def timed(fn):
            for _ in range(2):
                for o in fn():
                    lib.DeleteCiphertext(o)
            lib.Synchronize()
            _capi.check(capi.helrm_TimerStart())
            for _ in range(reps):
                for o in fn():
                    lib.DeleteCiphertext(o)
            ms = ctypes.c_double(0)
            _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
            return ms.value / reps

        one = timed(lambda: lib.MulConstantMatMulNew(cts, tab))
        per_row = timed(lambda: [lib.MulConstantAccumNew(cts, kids[r * cols:(r + 1) * cols]) for r in range(rows)])
        limb = N * 8
        nbytes = (cols + rows) * 2 * (level + 1) * limb
        peak, src = _peak()
        lib.DeleteConstantTable(tab)
        return {"op": "ive_table_matmul", "rows": rows, "cols": cols, "level": level, "ms_one_pass": one,
                "ms_row_at_a_time": per_row, "GBps_one_pass": nbytes / (one * 1e6),
                "frac_hbm": nbytes / (one * 1e6) / peak, "peak": f"{peak} GB/s ({src})"}
    finally:
        lib.DeleteScheme()


def run_relu(batches=(1, 8), reps=3, degrees=(15, 15, 27), level=23, device=0) -> list[dict]:
    """Orion's ReLU (orion/nn/activation.py:246-300) at LogN 16 (config 2/3
    primes): the composite step polynomial, stage by stage through
    EvaluatePolynomialBatch (the last stage at scale q[level] so the
    product's rescale is exact), then x * step(x) and its rescale, on
    batches of ciphertexts at `level`.  CUDA events on the library stream;
    reports milliseconds per ciphertext and per ciphertext product."""
    from helrm_b200 import B200Library, _capi
    from helrm_b200.params import CFG2, CFG2_DNUM

    lib = B200Library(dnum=CFG2_DNUM, seed=13, device=device)
    lib.setup_bindings(CFG2)
    out = []
    try:
        lib.GenerateSecretKey()
        lib.GenerateRelinearizationKey()
        info = lib.scheme_info()
        slots = info["slots"]
        scale = float(1 << CFG2.logscale)
        chain = lib.GetModuliChain()
        flat = lib.GenerateMinimaxSignCoeffs(list(degrees), 128, 6, 12, 0)
        stages, o = [], 0
        for d in degrees:
            stages.append(lib.GenerateChebyshev(flat[o:o + d + 1]))
            o += d + 1
        products = sum(lib.PolynomialPlanInfo(p, level, scale)["products"] for p in stages) + 1
        capi = _capi.load()
        rng = np.random.default_rng(1)
        for nb in batches:
            xs = [rng.uniform(-1, 1, slots) for _ in range(nb)]
            cts = []
            for x in xs:
                pt = lib.Encode(list(x), level, scale)
                cts.append(lib.Encrypt(pt))
                lib.DeletePlaintext(pt)

            def relu():
                cur = list(cts)
                for i, p in enumerate(stages):
                    lvl = lib.GetCiphertextLevel(cur[0]) - lib.GetPolyDepth(p)
                    target = float(chain[lvl]) if i == len(stages) - 1 else scale
                    nxt = lib.EvaluatePolynomialBatch(cur, p, target)
                    if cur is not cts and cur[0] not in cts:
                        for c in cur:
                            lib.DeleteCiphertext(c)
                    cur = nxt
                res = []
                for x, s in zip(cts, cur):
                    res.append(lib.Rescale(lib.MulRelinCiphertextNew(x, s)))
                    lib.DeleteCiphertext(s)
                return res

            for r in relu():  # warm-up (plans, pools)
                lib.DeleteCiphertext(r)
            lib.Synchronize()
            _capi.check(capi.helrm_TimerStart())
            last = None
            for _ in range(reps):
                if last:
                    for r in last:
                        lib.DeleteCiphertext(r)
                last = relu()
            ms = ctypes.c_double(0)
            _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
            got = np.array(lib.Decode(lib.Decrypt(last[0])))
            err = float(np.abs(got - np.maximum(xs[0], 0))[np.abs(xs[0]) > 2.0 ** -5].max())
            for r in last:
                lib.DeleteCiphertext(r)
            for c in cts:
                lib.DeleteCiphertext(c)
            per = ms.value / reps / nb
            out.append({"op": "relu_composite", "degrees": list(degrees), "batch": nb, "level_in": level,
                        "level_out": level - sum(math.ceil(math.log2(d + 1)) for d in degrees) - 1,
                        "ms_per_ct": per, "products_per_ct": products, "ms_per_product": per / products,
                        "max_err_outside_gap": err})
    finally:
        lib.DeleteScheme()
    return out


def run_upload(count=64, level=4, reps=3, device=0) -> dict:
    """The selector upload at LogN 16 (config 2/3 primes), server side of
    examples/criteo/bench_sweep.py:355-420: `count` real vectors, device
    encoding one at a time (Encode) and batched (EncodeBatch), and the lane
    split of count/2 packed ciphertexts (UnpackLanes) against the
    reference's op-by-op sequence (conjugate, add, sub, i, negate).  CUDA
    events on the library stream; host-to-device copies of the slot values
    are inside the encode times."""
    from helrm_b200 import B200Library, _capi, lanes
    from helrm_b200.params import CFG2, CFG2_DNUM

    lib = B200Library(dnum=CFG2_DNUM, seed=21, device=device)
    lib.setup_bindings(CFG2)
    try:
        lib.GenerateSecretKey()
        slots = lib.scheme_info()["slots"]
        scale = float(1 << CFG2.logscale)
        capi = _capi.load()
        rng = np.random.default_rng(0)
        vals = rng.uniform(-1, 1, (count, slots))

        def timed(fn):
            # outputs are freed (stream-ordered) after every repetition, so
            # the memory pool stays at its warmed-up size
            for _ in range(2):
                for i, d in fn():
                    d(i)
            lib.Synchronize()
            _capi.check(capi.helrm_TimerStart())
            for _ in range(reps):
                for i, d in fn():
                    d(i)
            ms = ctypes.c_double(0)
            _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
            return ms.value / reps

        dp, dc = lib.DeletePlaintext, lib.DeleteCiphertext
        single = timed(lambda: [(lib.Encode(list(v), level, scale), dp) for v in vals])
        batch = timed(lambda: [(i, dp) for i in lib.EncodeBatch(vals, level, scale)])
        packed_vec, num_real = lanes.pack_lanes(vals.ravel(), slots)
        pts = lanes.encode_packed(lib, packed_vec, slots, level, scale)
        packed = [lib.Encrypt(p) for p in pts]
        fused = timed(lambda: [(i, dc) for i in lib.UnpackLanes(packed, num_real)])

        def op_by_op():
            out = []
            for pid in packed:
                conj = lib.ConjugateNew(pid)
                even = lib.AddCiphertextNew(pid, conj)
                diff = lib.SubCiphertextNew(pid, conj)
                lib.MulImaginaryUnit(diff)
                odd = lib.Negate(diff)
                dc(conj)
                dc(diff)
                out.extend([(even, dc), (odd, dc)])
            return out
        ops = timed(op_by_op)
        return {"op": "selector_upload", "vectors": count, "level": level, "ms_encode_each": single / count,
                "ms_encode_batch_per_vector": batch / count, "ms_unpack_fused": fused,
                "ms_unpack_op_by_op": ops, "packed_cts": len(packed)}
    finally:
        lib.DeleteScheme()


def run_boot(slot_counts=(512,), reps=3, device=0) -> list[dict]:
    """Bootstrapping at LogN 16: the cfg2 chain with a 50-bit q0 (message
    ratio 2^14) under 24 usable levels, the 11 reserved 60-bit primes above it,
    six 60-bit special primes (dnum 6); sparse slot counts as Orion's
    bootstrap layers use for the MLP widths.  CUDA events on the library
    stream around Bootstrap calls on a level-0 ciphertext; the precision
    is the largest slot error after decryption."""
    from helrm_b200 import B200Library, CKKSConfig, _capi

    cfg = CKKSConfig(logn=16, logq=[50] + [36] * 23, logp=[60] * 6, logscale=36, h=192, boot=True)
    lib = B200Library(seed=31, device=device)
    lib.setup_bindings(cfg)
    out = []
    try:
        lib.GenerateSecretKey()
        lib.GenerateRelinearizationKey()
        S = lib.scheme_info()["slots"]
        capi = _capi.load()
        rng = np.random.default_rng(2)
        for n in slot_counts:
            import time
            t0 = time.time()
            lib.NewBootstrapper(None, n)
            lib.Synchronize()
            setup_s = time.time() - t0
            z = rng.uniform(-1, 1, n)
            pt = lib.Encode(list(np.tile(z, S // n)), 0, float(1 << 36))
            ct = lib.Encrypt(pt)
            lib.DeletePlaintext(pt)
            lib.DeleteCiphertext(lib.Bootstrap(ct, n))  # warm-up (plans, pools)
            lib.Synchronize()
            _capi.check(capi.helrm_TimerStart())
            res = None
            for _ in range(reps):
                if res is not None:
                    lib.DeleteCiphertext(res)
                res = lib.Bootstrap(ct, n)
            ms = ctypes.c_double(0)
            _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
            got = np.array(lib.Decode(lib.Decrypt(res)))
            err = float(np.abs(got - np.tile(z, S // n)).max())
            out.append({"op": "bootstrap", "logN": 16, "slots": n, "ms": ms.value / reps,
                        "level_out": lib.GetCiphertextLevel(res), "max_err": err,
                        "setup_s": setup_s, "chain": "50 + 23 x 36 usable, 11 x 60 reserved, 6 x 60 special"})
            lib.DeleteCiphertext(res)
            lib.DeleteCiphertext(ct)
    finally:
        lib.DeleteScheme()
    return out


def run_mac_mixed(reps=3, batch=8, device=0) -> dict:
    """Profiling case of the fused MAC over mixed prime sizes (the
    bootstrapping chain's shape, kept to a few GB): LogN 16, q0 of 50 bits,
    five 36-bit and three 60-bit q primes, three 60-bit special primes at
    dnum 5 (five digits at the top level), one 64-diagonal transform at
    bsgs_ratio 16 (a full chunk of 32 babies, two giant slots), `batch`
    ciphertexts, `reps` evaluations; CUDA events on the library stream."""
    from helrm_b200 import B200Library, CKKSConfig, _capi

    cfg = CKKSConfig(logn=16, logq=[50] + [36] * 5 + [60] * 3, logp=[60] * 3, logscale=36, h=192)
    lib = B200Library(dnum=5, seed=5, device=device)
    lib.setup_bindings(cfg)
    try:
        lib.GenerateSecretKey()
        S = lib.scheme_info()["slots"]
        ks = list(range(64))
        rng = np.random.default_rng(1)
        level = len(cfg.logq) - 1
        lt = lib.GenerateLinearTransform(ks, rng.uniform(-0.5, 0.5, (len(ks), S)).ravel(), level, 16.0, "none")
        for k in lib.GetLinearTransformRotationKeys(lt):
            lib.GenerateLinearTransformRotationKey(k)
        cts = []
        for _ in range(batch):
            pt = lib.Encode(list(rng.uniform(-1, 1, S)), level, float(1 << 36))
            cts.append(lib.Encrypt(pt))
            lib.DeletePlaintext(pt)
        for o in lib.EvaluateLinearTransformBatch(lt, cts):  # warm-up
            lib.DeleteCiphertext(o)
        capi = _capi.load()
        lib.Synchronize()
        _capi.check(capi.helrm_TimerStart())
        for _ in range(reps):
            for o in lib.EvaluateLinearTransformBatch(lt, cts):
                lib.DeleteCiphertext(o)
        ms = ctypes.c_double(0)
        _capi.check(capi.helrm_TimerStop(ctypes.byref(ms)))
        return {"op": "lt_mixed_primes", "logN": 16, "digits": 5, "diagonals": 64, "bs": 32, "batch": batch,
                "ms": ms.value / reps, "peak_device_mb": lib.GetPeakDeviceMemoryMB()}
    finally:
        lib.DeleteScheme()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batches", default="1,16,128")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--ops", default="ntt,intt,aut,mac,rescale,ks")
    ap.add_argument("--rotations", type=int, default=32)
    ap.add_argument("--table", action="store_true", help="also the IVE lookup's one-pass table product")
    ap.add_argument("--relu", action="store_true", help="also Orion's composite ReLU through EvaluatePolynomial")
    ap.add_argument("--upload", action="store_true", help="also the selector upload (device encode, lane split)")
    ap.add_argument("--boot", action="store_true", help="also bootstrapping at LogN 16 (256 and 512 slots)")
    ap.add_argument("--mac-mixed", action="store_true",
                    help="only the mixed-prime fused-MAC profiling case (a few GB on the device)")
    args = ap.parse_args()
    if args.mac_mixed:
        print(json.dumps(run_mac_mixed()), flush=True)
        return
    run([int(b) for b in args.batches.split(",")], args.reps, args.ops, args.rotations,
        emit=lambda line: print(json.dumps(line), flush=True))
    if args.table:
        print(json.dumps(run_table_matmul()), flush=True)
    if args.relu:
        for line in run_relu():
            print(json.dumps(line), flush=True)
    if args.upload:
        print(json.dumps(run_upload()), flush=True)
    if args.boot:
        for line in run_boot(slot_counts=(256, 512)):
            print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
