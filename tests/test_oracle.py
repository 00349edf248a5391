"""The CPU oracle against the reference's own golden outputs (no GPU)."""

import ctypes

import numpy as np
import pytest

from oracle import pkv_oracle as po
from tests.golden.make_golden import SMOKE_CASES, smoke_inputs


def test_glibc_rand_matches_libc():
    try:
        libc = ctypes.CDLL("libc.so.6")
    except OSError:
        pytest.skip("no glibc")
    for seed in (42, 7, 2**31 + 5):
        libc.srand(seed)
        want = np.array([libc.rand() for _ in range(2000)])
        got = po.GlibcRand(seed).rand_array(2000)
        assert np.array_equal(want, got)


def test_smoke_replay_matches_fixture(smoke_kat):
    # the first values of every case pin the replayed srand(42) stream
    for i, (_, q, _, _) in enumerate(smoke_inputs()):
        assert np.array_equal(q.reshape(-1)[:8], smoke_kat[f"q_head_{i}"])


def test_oracle_matches_reference_cpu_gqa_attention(smoke_kat):
    """numpy restatement vs outputs of the reference's compiled cpu_gqa_attention."""
    for i, (case, q, k, v) in enumerate(smoke_inputs()):
        want = smoke_kat[f"out_{i}"]
        got = po.cpu_gqa_attention(q, k, v)
        assert np.abs(got - want).max() < 2e-6, case


def _to_paged(k, v, page_size, order="reversed"):
    """Pages a contiguous [B,Hkv,N,D] cache like tests/smoke_test.cu:239-258."""
    b, hkv, n, d = k.shape
    per = (n + page_size - 1) // page_size
    kp = np.zeros((b * per, hkv, page_size, d), np.float32)
    vp = np.zeros_like(kp)
    table = np.zeros((b, per), np.int32)
    for bi in range(b):
        for lp in range(per):
            phys = bi * per + (per - 1 - lp if order == "reversed" else lp)
            table[bi, lp] = phys
            t0, t1 = lp * page_size, min(n, (lp + 1) * page_size)
            kp[phys, :, : t1 - t0] = k[bi, :, t0:t1]
            vp[phys, :, : t1 - t0] = v[bi, :, t0:t1]
    return kp, vp, table


def test_paged_oracle_equals_contiguous(smoke_kat):
    for i, (case, q, k, v) in enumerate(smoke_inputs()):
        page = case[6] or 16
        kp, vp, table = _to_paged(k, v, page)
        got = po.paged_decode(q, kp, vp, table, context=k.shape[2])
        assert np.abs(got - smoke_kat[f"out_{i}"]).max() < 2e-6, case


def test_masked_indexed_semantics():
    rng = np.random.default_rng(3)
    hq, hkv, page = 8, 2, 16
    pool = 40
    kp = po.quantize(rng.standard_normal((pool, hkv, page, 128)))
    vp = po.quantize(rng.standard_normal((pool, hkv, page, 128)))
    table = rng.permutation(pool)[:30].reshape(3, 10).astype(np.int32)
    seq = np.array([5, 0, 160], np.int32)
    q_src = po.quantize(rng.standard_normal((5, hq, 128)))
    q_idx = np.array([4, 0, 2], np.int32)
    o_idx = np.array([1, 3, 0], np.int32)
    out = po.paged_decode(q_src, kp, vp, table, seq_lens=seq, q_indices=q_idx,
                          out_indices=o_idx, out_rows=4)
    assert np.isnan(out[2]).all()            # row never written
    assert np.all(out[3] == 0)               # empty sequence -> zeros
    k, v = po.gather_row(kp, vp, table[2], 160)
    assert np.allclose(out[0], po.attend_row(q_src[2].astype(np.float64), k, v))


def test_state_combine_is_exact_split():
    rng = np.random.default_rng(4)
    q = rng.standard_normal((8, 128))
    k = rng.standard_normal((2, 300, 128))
    v = rng.standard_normal((2, 300, 128))
    parts = [po.row_state(q, k[:, a:b], v[:, a:b]) for a, b in ((0, 37), (37, 37), (37, 300))]
    merged = po.combine_states([p[0] for p in parts], [p[1] for p in parts],
                               [p[2] for p in parts])
    assert np.abs(merged - po.attend_row(q, k, v)).max() < 1e-12


def test_bf16_quantize_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-3, 3.0e38], np.float32)
    q = po.quantize(x, "bf16")
    assert q[0] == 1.0 and q[1] == 1.0 and q[2] == np.float32(1.0078125)
    assert np.abs(q[3] - x[3]) / abs(x[3]) < 2 ** -8
    assert len(SMOKE_CASES) == 8


def test_torch_repack_forms_match_numpy_oracle():
    """The repack + SDPA forms (benchmark_torch_paged_sdpa.py:90-109) agree
    with the numpy oracle: torch's fp32 SDPA (the CPU baseline) to fp32
    rounding, the float64 checker to 1e-9 (the numpy oracle keeps the
    reference's ``/(l + 1e-8)`` normalisation, the torch checker divides by l:
    they differ by o * 1e-8 / l, l >= 1)."""
    import torch

    rng = np.random.default_rng(11)
    hq, hkv, page, pool = 32, 8, 16, 40
    kp = po.quantize(rng.standard_normal((pool, hkv, page, 128)))
    vp = po.quantize(rng.standard_normal((pool, hkv, page, 128)))
    table = rng.permutation(pool)[:24].reshape(3, 8).astype(np.int32)
    seq = np.array([100, 0, 128], np.int32)
    q = po.quantize(rng.standard_normal((3, hq, 128)))
    want = po.paged_decode(q, kp, vp, table, seq_lens=seq)
    got64 = po.torch_paged_decode(torch.from_numpy(q), torch.from_numpy(kp),
                                  torch.from_numpy(vp), table, seq)
    assert np.abs(got64.numpy() - want).max() < 1e-9
    kt, vt = torch.from_numpy(kp), torch.from_numpy(vp)
    for r in (0, 2):
        n = int(seq[r])
        pages = torch.from_numpy(table[r, : (n + page - 1) // page]).long()
        got = po.sdpa_repack_row(torch.from_numpy(q[r]), kt, vt, pages, n).numpy()
        assert np.abs(got - want[r]).max() < 1e-5
