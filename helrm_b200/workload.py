"""HE-LRM embedding-PCMM workloads (BASELINE configs 1 and 2), synthetic.

The Criteo dataset is not available, so seeded synthetic inputs with the
reference's shapes and distributions stand in for it:

* cfg1: one V=1024 x 16 table compressed base 32 into 2 digit tables
  (RadixTable, examples/criteo/dlrm.py:100-124), weights N(0, 0.1); the
  plaintext matrix is the 16 x 64 digit-table stack.
* cfg2: 26 vocabularies log-uniform in [3, 1e7] (seed 0 gives W = 4224
  selector slots), each compressed base 64 into ceil(log64 V) one-hot
  digits (dlrm.py:82-90, 202-213); weights N(0, 0.05) in the block-diagonal
  416 x W matrix that export() builds (dlrm.py:241-248; block structure as
  bench_sweep._impose_block_diagonal, examples/criteo/bench_sweep.py:154-188);
  queries Zipf(1.05) per table.

``diagonalize`` restates the hybrid/square diagonal extraction of
orion/core/packing.py:626-865 (without the optional sliced heights), and
``bsgs_plan`` the BSGS split of orion/backend/cheddar/bindings.py:857-862,
893-896, 916-936.
"""
from __future__ import annotations

import math

import numpy as np

EMB_DIM = 16


def radix_width(categories: int, base: int) -> int:
    """dlrm.py:78-79"""
    return math.ceil(math.log(categories, base))


def digits(index: int, base: int, width: int) -> list[int]:
    """dlrm.py:66-75 (least significant digit first)"""
    out = []
    for _ in range(width):
        out.append(index % base)
        index //= base
    return out


# ---------------------------------------------------------------- matrices
def cfg1_matrix(seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    tables = [rng.normal(0.0, 0.1, size=(32, EMB_DIM)) for _ in range(2)]
    return np.concatenate(tables, axis=0).T.astype(np.float32)  # (16, 64)


def cfg2_vocab(seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.floor(np.exp(rng.uniform(np.log(3), np.log(1e7), 26))).astype(np.int64)


def block_diag_matrix(vocab, base: int = 64, dim: int = EMB_DIM, std: float = 0.05, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    widths = [base * radix_width(int(v), base) for v in vocab]
    M = np.zeros((dim * len(vocab), sum(widths)), dtype=np.float32)
    r = c = 0
    for w in widths:
        M[r:r + dim, c:c + w] = rng.normal(0.0, std, size=(dim, w))
        r += dim
        c += w
    return M


def selector(indices, vocab, base: int = 64) -> np.ndarray:
    """Concatenated one-hot digits of every table's index (dlrm.py:202-220)."""
    parts = []
    for idx, v in zip(indices, vocab):
        w = radix_width(int(v), base)
        for d in digits(int(idx), base, w):
            piece = np.zeros(base, dtype=np.float64)
            piece[d] = 1.0
            parts.append(piece)
    return np.concatenate(parts)


def zipf_queries(vocab, n: int, a: float = 1.05, seed: int = 7) -> np.ndarray:
    """n queries x 26 tables of Zipf(a) indices, folded into each vocabulary."""
    rng = np.random.default_rng(seed)
    z = rng.zipf(a, size=(n, len(vocab)))
    return (z - 1) % np.asarray(vocab)[None, :]


def cfg1_queries(n: int, seed: int = 11):
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, 1024, size=n)
    sel = np.zeros((n, 64))
    for i, x in enumerate(idx):
        d0, d1 = digits(int(x), 32, 2)
        sel[i, d0] = 1.0
        sel[i, 32 + d1] = 1.0
    return idx, sel


# ---------------------------------------------------------------- diagonals
def diagonalize(M: np.ndarray, slots: int, method: str = "hybrid", last: bool = False):
    """Generalized diagonals of each (row block, column block).

    Returns ({(br, bc): {k: diag_k (float32, length slots)}}, output_rotations)
    with diag_k[s] = M[row0 + s mod bh, col0 + (s + k) mod slots]."""
    H, W = M.shape
    nbr, nbc = math.ceil(H / slots), math.ceil(W / slots)
    if nbr == 1 and method == "hybrid" and not last:
        bh = 2 ** math.ceil(math.log2(H))
        out_rot = int(math.log2(slots // bh))
    else:
        bh, out_rot = slots, 0
    Mp = np.zeros((max(nbr * bh, slots * (nbr - 1) + bh), nbc * slots), dtype=np.float32)
    Mp[:H, :W] = M
    s = np.arange(slots)
    rows = s % bh
    out = {}
    for br in range(nbr):
        for bc in range(nbc):
            blk = Mp[slots * br: slots * br + bh, bc * slots:(bc + 1) * slots]
            cols = (np.arange(bh)[:, None] + s[None, :]) % slots
            D = blk[rows[None, :], cols]
            nz = {int(i): D[i] for i in range(bh) if np.any(D[i])}
            out[(br, bc)] = nz or {0: np.zeros(slots, dtype=np.float32)}
    return out, out_rot


def bsgs_plan(ks, ratio, slots):
    """Baby-step stride and giant groups for a set of diagonal indices."""
    n = len(ks)
    use_bsgs = ratio not in ("none", None) and float(ratio) > 0 and n > 1
    bs = max(1, math.ceil(math.sqrt(n * float(ratio)))) if use_bsgs else slots
    groups: dict[int, list[tuple[int, int]]] = {}
    for k in ks:
        b, g = (k % bs, k // bs) if use_bsgs else (k, 0)
        groups.setdefault(g, []).append((b, k))
    keys = set()
    for g, grp in groups.items():
        for b, _ in grp:
            if b:
                keys.add(b)
        if g:
            keys.add(g * bs)
    return {"use_bsgs": use_bsgs, "bs": bs if use_bsgs else None, "stride": bs, "groups": groups,
            "rotation_keys": sorted(keys)}


def preroll(values, g: int, bs: int) -> np.ndarray:
    """numpy roll to the right by g*bs (bindings.py:893-896)."""
    v = np.asarray(values)
    return v if g == 0 else np.roll(v, g * bs)


def cleartext_lt(x, diags: dict, slots: int) -> np.ndarray:
    """out[i] = sum_k diag_k[i] * x[(i + k) mod slots] (tests/oracle/test_linear_transform.py:99-100)"""
    x = np.asarray(x, dtype=np.float64)
    out = np.zeros(slots)
    for k, d in diags.items():
        out += np.asarray(d, dtype=np.float64) * np.roll(x, -k)
    return out


def hybrid_fold(v, slots: int, rotations: int) -> np.ndarray:
    """orion/nn/linear.py:115-117 on cleartext."""
    v = np.asarray(v, dtype=np.float64).copy()
    for i in range(1, rotations + 1):
        v = v + np.roll(v, -(slots >> i))
    return v
