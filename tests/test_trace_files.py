"""External trace files: the loader and the requests /
steps built from it match the reference's own ``load_trace_specs`` /
``build_requests(trace_file=...)`` / ``build_steps`` on the committed files
(golden outputs from ``tests/golden/make_golden.py``)."""

import json

import pytest

from persistentkv_attention_b200 import trace as tr
from tests.conftest import GOLDEN


@pytest.fixture(scope="module")
def trace_files_golden():
    return json.loads((GOLDEN / "trace_files.json").read_text())


def test_trace_files_match_reference(trace_files_golden):
    for case in trace_files_golden:
        specs = tr.load_trace_specs(GOLDEN / case["file"], case["limit"])
        assert [list(s) for s in specs] == case["specs"]
        reqs, physical = tr.build_requests("uniform", case["limit"], case["max_active"],
                                           case["seed"], case["hole"], specs=specs)
        assert physical == case["physical_pages"]
        assert [list(r.physical_pages) for r in reqs] == case["pages"]
        steps = tr.build_steps(reqs, case["max_active"])
        assert [[s.step, list(s.active_ids), list(s.lengths)] for s in steps] == case["steps"]


def test_trace_file_errors(tmp_path):
    bad_json = tmp_path / "t.json"
    bad_json.write_text('{"prompt": 5}')
    with pytest.raises(ValueError, match="list of request objects"):
        tr.load_trace_specs(bad_json, 10)
    bad_csv = tmp_path / "t.csv"
    bad_csv.write_text("prompt_len,decode_len\n12,x\n")
    with pytest.raises(ValueError, match="integer prompt_len/prompt"):
        tr.load_trace_specs(bad_csv, 10)
    empty = tmp_path / "e.csv"
    empty.write_text("prompt_len,decode_len\n")
    with pytest.raises(ValueError, match="produced no requests"):
        tr.load_trace_specs(empty, 10)
    # limit and defaults: arrival = row index, prompt rounded up to whole pages
    ok = tmp_path / "ok.csv"
    ok.write_text("prompt,decode\n1,2\n17,3\n40,4\n")
    assert tr.load_trace_specs(ok, 2) == [(0, 16, 2), (1, 32, 3)]
