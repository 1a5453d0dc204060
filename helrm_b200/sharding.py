"""Table sharding of the embedding PCMM, with one exchange of packed
partial ciphertexts (the multi-GPU partition the north star names: the 26
tables split across GPUs, the query batch fixed).

The HE-LRM embedding matrix is block-diagonal: table t's 16 output rows
read only its own selector slots (examples/criteo/dlrm.py:241-248;
examples/criteo/bench_sweep.py:154-188).  A rank that owns a contiguous
group of tables evaluates just those rows:

* its rows R0 .. R0 + n - 1 (n = 16 x tables) form a matrix of block height
  bh = 2^ceil(log2 n) whose row r holds global row R0 + ((r - R0) mod bh),
  over the full selector width, so the input ciphertext is the same
  reference-layout selector every rank holds.  The hybrid diagonal method
  gives bh diagonals (64 at 8 ranks, against 512 for all 26 tables);
* after the transform, the rescale and the log2(slots / bh) fold rotations
  (orion/nn/linear.py:115-117), slot s holds shard row (s - R0) mod bh;
  slots with (s mod P) in [R0, R0 + n), P = 2^ceil(log2 of all rows) = 512,
  hold exactly the values the unsharded transform leaves there;
* a 0/1 mask over those slots, encoded at the modulus of its level (the
  reference's errorless-rescale idiom, orion/nn/embedding.py:104-110), and
  one more rescale keep only them, so the ranks' outputs occupy disjoint
  slots of the unsharded layout.

The exchange is then a sum: the ranks' residues (each below q < 2^61, at
most 8 of them) are summed as 64-bit integers by one NCCL reduce, and the
receiving rank reduces every limb modulo its prime while importing the sum
as a ciphertext (helrm_NewCiphertextsFromDeviceSum).  The result is the
packed embedding ciphertext of all 26 tables, two levels below the input
(one level more than the unsharded transform: the mask).
"""
from __future__ import annotations

import math

import numpy as np

from . import workload as W


def table_shards(ntables: int, nshards: int) -> list[range]:
    """Contiguous, balanced table groups (26 over 8 ranks: 4,4,3,3,3,3,3,3)."""
    if not 1 <= nshards <= ntables:
        raise ValueError("need 1 <= shards <= tables")
    base, extra = divmod(ntables, nshards)
    out, t = [], 0
    for i in range(nshards):
        k = base + (1 if i < extra else 0)
        out.append(range(t, t + k))
        t += k
    return out


def layout_period(total_rows: int) -> int:
    """Output period of the unsharded hybrid transform (block height)."""
    return 2 ** math.ceil(math.log2(total_rows))


def shard_matrix(M: np.ndarray, tables: range, dim: int = W.EMB_DIM):
    """The shard's rows placed for the masked merge.

    Returns (V, bh, R0, n): V has bh rows, row (R0 + i) mod bh = M[R0 + i]."""
    R0, n = dim * tables.start, dim * len(tables)
    bh = layout_period(n)
    if bh > layout_period(M.shape[0]):
        raise ValueError("shard larger than the unsharded block")
    V = np.zeros((bh, M.shape[1]), dtype=np.float32)
    for i in range(n):
        V[(R0 + i) % bh] = M[R0 + i]
    return V, bh, R0, n


def shard_mask(slots: int, period: int, R0: int, n: int) -> np.ndarray:
    """1 on the slots that carry the shard's rows in the unsharded layout."""
    s = np.arange(slots) % period
    return ((s >= R0) & (s < R0 + n)).astype(np.float64)


def cleartext_shard(M: np.ndarray, tables: range, x, slots: int) -> np.ndarray:
    """The shard's masked, folded output on cleartext (reference for tests)."""
    V, bh, R0, n = shard_matrix(M, tables)
    d, rot = W.diagonalize(V, slots, "hybrid")
    y = W.hybrid_fold(W.cleartext_lt(_pad(x, slots), d[(0, 0)], slots), slots, rot)
    return y * shard_mask(slots, layout_period(M.shape[0]), R0, n)


def _pad(x, slots):
    v = np.zeros(slots)
    v[:len(x)] = x
    return v


class ShardedEmbedding:
    """One rank's part of the table-sharded embedding layer, on a
    B200Library scheme: the shard's transform, its rotation keys and the
    mask plaintext, and evaluate() for a batch of selector ciphertexts."""

    def __init__(self, lib, M: np.ndarray, tables: range, level: int, ratio: float | None = None):
        self.lib = lib
        info = lib.scheme_info()
        self.slots = info["slots"]
        self.period = layout_period(M.shape[0])
        V, self.bh, self.R0, self.n = shard_matrix(M, tables)
        d, self.rot = W.diagonalize(V, self.slots, "hybrid")
        diags = d[(0, 0)]
        self.ks = sorted(diags)
        self.diags = diags
        data = np.concatenate([diags[k].astype(np.float64) for k in self.ks])
        self.level = level
        # baby-step stride 32 (ratio 1024 / diagonals, at least the
        # reference's 2): every shard size runs the full-chunk MAC and as
        # few giant-step key switches as the unsharded transform's 16 groups allow
        self.ratio = float(ratio) if ratio else max(2.0, 1024.0 / len(self.ks))
        self.lt = lib.GenerateLinearTransform(self.ks, data, level, self.ratio, "none")
        for k in lib.GetLinearTransformRotationKeys(self.lt):
            lib.GenerateLinearTransformRotationKey(k)
        for i in range(1, self.rot + 1):
            lib.AddRotationKey(self.slots >> i)
        q = lib.GetModuliChain()
        self.mask = shard_mask(self.slots, self.period, self.R0, self.n)
        # errorless rescale: the mask at the scale of the prime the next rescale drops
        self.mask_pt = lib.Encode(list(self.mask), level - 1, float(q[level - 1]))

    def evaluate(self, cts) -> list[int]:
        """Partial packed-embedding ciphertexts (level - 2) of the batch."""
        lib = self.lib
        outs = lib.EvaluateLinearTransformBatch(self.lt, cts)
        lib.RescaleBatch(outs)
        lib.HybridFoldBatch(outs, self.rot)
        for o in outs:
            lib.MulPlaintext(o, self.mask_pt)
        lib.RescaleBatch(outs)
        return outs

    def close(self):
        self.lib.DeleteLinearTransform(self.lt)
        self.lib.DeletePlaintext(self.mask_pt)


def exchange_sum(buf, dist, dst: int = 0):
    """Sum the ranks' partial residues (an int64 torch tensor, 64-bit
    integer sums, exact while the total stays below 2^63) into rank dst
    with one reduce; dist is torch.distributed (NCCL on GPUs, gloo on CPU).
    Returns the tensor (the sum on rank dst)."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.reduce(buf, dst=dst, op=dist.ReduceOp.SUM)
    return buf


def reduce_mod_q(summed: np.ndarray, primes) -> np.ndarray:
    """Host form of the receiving side's reduction: [npoly][nq][N] sums ->
    residues modulo each limb's prime (the library does this on the device
    while importing; tests use this form)."""
    s = np.asarray(summed).view(np.uint64) if summed.dtype == np.int64 else np.asarray(summed, dtype=np.uint64)
    q = np.asarray(primes[:s.shape[-2]], dtype=np.uint64).reshape((1,) * (s.ndim - 2) + (-1, 1))
    return s % q
