"""The router's B200 step-time model of the device-side schedule against the
step times measured on a B200 (profiles/router_sweep_b200.json: configs 1-5,
eight group counts each, L2 flushed before every step).  The constants of
pkv_router_params_b200 come from persistentkv_attention_b200/calibrate.py
on that file."""

import json

import numpy as np
import pytest

from persistentkv_attention_b200 import calibrate
from persistentkv_attention_b200.scheduler import Router
from tests.conftest import REPO

SWEEP = json.loads((REPO / "profiles" / "router_sweep_b200.json").read_text())


def _params():
    p = Router.b200(32, 8, sm_count=SWEEP["sm_count"]).params
    return {k: getattr(p, k) for k in ("read_gbps", "dev_cta_gbps", "dev_fixed_us",
                                       "dev_merge_us", "dev_merge_piece_us")}


def test_model_matches_the_measured_step_times():
    params = _params()
    rel = [(calibrate.predict(params, s, SWEEP["hkv"]) - s.us) / s.us
           for s in calibrate.samples(SWEEP)]
    assert np.sqrt(np.mean(np.square(rel))) < 0.05
    assert np.max(np.abs(rel)) < 0.12


def test_router_picks_a_measured_near_best_group_count():
    router = Router.b200(32, 8, sm_count=SWEEP["sm_count"])
    for name, c in SWEEP["configs"].items():
        measured = {int(g): us for g, us in c["us_median"].items()}
        best = min(measured.values())
        choices = [router.choose_groups(lens)[0] for lens in c["lengths"]]
        for ng in set(choices):
            # the nearest measured group count to the choice
            near = min(measured, key=lambda g: abs(g - ng))
            assert measured[near] <= best * 1.06, (name, ng, measured)


def test_fit_reproduces_the_committed_constants():
    fitted, err = calibrate.fit(SWEEP)
    params = _params()
    assert err ** 0.5 < 0.05
    for key in ("read_gbps", "dev_cta_gbps"):
        assert abs(fitted[key] - params[key]) <= 0.02 * params[key], key


def _choose_groups_exhaustive(params, lengths, sms=148, hkv=8):
    """The step-time model over every candidate group count, every row."""
    ng_max = max(1, (2 * sms) // hkv)
    bytes_ = float(sum(max(0, int(n)) for n in lengths)) * hkv * 128 * 2 * 2
    best, best_us = ng_max, float("inf")
    for ng in range(ng_max, max(1, ng_max // 8) - 1, -1):
        s = calibrate.Sample("x", ng, 0.0, bytes_, calibrate.max_pieces(lengths, ng))
        us = calibrate.predict(params, s, hkv)
        if us < best_us:
            best, best_us = ng, us
    return best, best_us


@pytest.mark.parametrize("seed", range(6))
def test_choose_groups_matches_the_exhaustive_model(seed):
    """pkv_choose_groups visits only the rows that can hold the most pieces;
    its choice and estimate equal the model evaluated over every row."""
    rng = np.random.default_rng(seed)
    router = Router.b200(32, 8, sm_count=148)
    params = _params()
    for n in (1, 3, 8, 64, 500):
        lens = rng.choice([0, 1, 31, 33, 512, 4096, 30000], size=n).tolist()
        if not any(lens):
            lens[0] = 100
        ng, est = router.choose_groups(lens)
        want_ng, want_us = _choose_groups_exhaustive(params, lens)
        assert ng == want_ng, (n, ng, want_ng)
        assert abs(est - want_us) < 1e-9 * max(1.0, want_us)
