"""bench.py's command line and the fixed parts of its JSON line (no GPU):
the defaults the driver runs with, the modes, the workload descriptions
and the tolerances the correctness checks use."""
import sys

import pytest

import bench


def _parse(argv):
    old = sys.argv
    sys.argv = ["bench.py"] + argv
    try:
        return bench.parse()
    finally:
        sys.argv = old


def test_defaults_are_one_gpu_and_the_config2_step():
    a = _parse([])
    assert (a.gpus, a.steps, a.warmup, a.impl, a.mode, a.batch, a.level) == (1, 5, 3, "b200", "dp", 64, 23)
    assert a.bsgs_ratio == 8.0 and not a.no_cfg4 and not a.small


@pytest.mark.parametrize("mode", ["dp", "tables", "helrm"])
def test_modes(mode):
    assert _parse(["--mode", mode]).mode == mode


def test_small_case_caps_the_level():
    assert _parse(["--small"]).level == 7


def test_workload_descriptions():
    a = _parse([])
    c2 = bench.cfg_dict(a, a.batch)
    assert c2["workload"].startswith("cfg2") and c2["bs"] == 64 and c2["giant_groups"] == 8
    assert "model" not in c2
    c4 = bench.helrm_config(a)
    assert c4["workload"].startswith("cfg4") and c4["bottom"] == [13, 512, 256, 64, 16]
    assert c4["top"] == [432, 512, 256, 1] and c4["batch_ciphertexts"] == 64


def test_tolerances():
    assert bench.REL_TOL == 2.0 ** -15 and bench.LOGIT_TOL == 1e-3
    assert bench.bs_of(2.0) == 32 and bench.bs_of(8.0) == 64
