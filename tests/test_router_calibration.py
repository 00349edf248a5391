"""The router's B200 step-time model of the device-side schedule against the
step times measured on a B200 (profiles/router_sweep_b200.json: configs 1-5,
eight group counts each, L2 flushed before every step).  The constants of
pkv_router_params_b200 come from persistentkv_attention_b200/calibrate.py
on that file."""

import json

import numpy as np

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
