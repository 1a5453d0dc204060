"""Host-side workload and plan logic against the reference's golden vectors."""
import hashlib

import numpy as np
import pytest

from helrm_b200 import workload as W


def _check(ks_ref, vals_ref, diags):
    (blk,) = diags.keys()
    d = diags[blk]
    assert sorted(d.keys()) == [int(k) for k in ks_ref]
    got = np.stack([d[int(k)] for k in ks_ref]).astype(np.float32)
    assert np.array_equal(got, vals_ref)


def test_diagonalize_docstring_example(golden_diag):
    m = np.arange(16, dtype=np.float32).reshape(4, 4)
    d, rot = W.diagonalize(m, 4, "hybrid", last=True)
    assert rot == 0
    _check(golden_diag["doc_ks"], golden_diag["doc_vals"], d)


def test_diagonalize_cfg1(golden_diag):
    M = W.cfg1_matrix()
    assert np.array_equal(M, golden_diag["cfg1_matrix"])
    d, rot = W.diagonalize(M, 4096, "hybrid")
    assert rot == int(golden_diag["cfg1_output_rotations"]) == 8
    _check(golden_diag["cfg1_ks"], golden_diag["cfg1_vals"], d)
    assert len(d[(0, 0)]) == 16


def test_diagonalize_block_diagonal_small(golden_diag):
    Ms = golden_diag["small_matrix"]
    d, rot = W.diagonalize(Ms, 2048, "hybrid")
    assert rot == int(golden_diag["small_output_rotations"])
    _check(golden_diag["small_ks"], golden_diag["small_vals"], d)


def test_cfg2_matrix_and_diagonals(golden_diag):
    V = W.cfg2_vocab()
    assert np.array_equal(V, golden_diag["cfg2_vocab"])
    M = W.block_diag_matrix(V, 64, 16, 0.05, seed=0)
    assert M.shape == (416, 4224) and tuple(golden_diag["cfg2_shape"]) == M.shape
    d, rot = W.diagonalize(M, 32768, "hybrid")
    assert rot == int(golden_diag["cfg2_output_rotations"]) == 6
    ks = np.array(sorted(d[(0, 0)].keys()))
    assert np.array_equal(ks, golden_diag["cfg2_ks"]) and len(ks) == 512
    vals = np.stack([d[(0, 0)][int(k)] for k in ks]).astype(np.float32)
    assert hashlib.sha256(vals.tobytes()).digest() == golden_diag["cfg2_sha256"].tobytes()
    plan = W.bsgs_plan(list(ks), 2.0, 32768)
    assert plan["bs"] == 32 and len(plan["groups"]) == 16
    assert len(plan["rotation_keys"]) == 31 + 15


def test_lt_plus_fold_is_matrix_product():
    """diag method + hybrid fold == M @ x on the padded slot vector."""
    rng = np.random.default_rng(0)
    M = rng.normal(size=(12, 40)).astype(np.float32)
    slots = 256
    d, rot = W.diagonalize(M, slots, "hybrid")
    x = np.zeros(slots)
    x[:40] = rng.normal(size=40)
    y = W.hybrid_fold(W.cleartext_lt(x, d[(0, 0)], slots), slots, rot)
    assert np.allclose(y[:12], M.astype(np.float64) @ x[:40], atol=1e-5)


@pytest.mark.parametrize("case", range(6))
def test_bsgs_plan_matches_reference_calls(golden_bsgs, case):
    """bs, rotation keys, pre-rolled plaintexts and the giant-step
    rotations of the reference's Python BSGS (bindings.py:833-1032)."""
    c = golden_bsgs[case]
    plan = W.bsgs_plan(c["ks"], c["ratio"], c["slots"])
    assert plan["use_bsgs"] == c["use_bsgs"]
    assert plan["bs"] == c["bs"]
    assert plan["rotation_keys"] == c["rotation_keys"]
    slots = c["slots"]
    for i, k in enumerate(c["ks"]):
        vals = np.array([float(k + 1 + t / 100.0) for t in range(slots)])
        g = k // plan["stride"] if plan["use_bsgs"] else 0
        ref = np.array(c["pt_values"][str(c["pt_ids"][str(k)])])
        assert np.array_equal(W.preroll(vals, g, plan["stride"]), ref)
    mac_out = {x[3] for x in c["eval_calls"] if x[0] == "MulPlaintextAccumNew"}
    giant_rot = sorted(x[2] for x in c["eval_calls"] if x[0] == "RotateNew" and x[1] in mac_out)
    want = sorted(g * plan["stride"] for g in plan["groups"] if g)
    if c["use_bsgs"]:
        assert giant_rot == want
    baby_calls = [x for x in c["eval_calls"] if x[0] == "RotateBatchNew"]
    if baby_calls:
        babies = sorted({b for grp in plan["groups"].values() for b, _ in grp if b})
        assert sorted(baby_calls[0][2]) == babies


def test_selector_and_queries():
    V = W.cfg2_vocab()
    q = W.zipf_queries(V, 8)
    assert q.shape == (8, 26) and (q >= 0).all() and (q < V[None, :]).all()
    s = W.selector(q[0], V)
    assert s.shape == (4224,)
    assert s.sum() == sum(W.radix_width(int(v), 64) for v in V)
