"""The oracle's e4m3 rounding (written from the OCP 8-bit floating point
spec) pinned against two independent implementations: CUDA's host-side
saturating conversion (cuda_fp8.h) and torch's float8_e4m3fn cast. Also the
block quantiser and block-scaled GEMM definitions against float64."""
import numpy as np
import torch

import oracle
from helpers import rel_err


def _probe_values():
    rng = np.random.default_rng(0)
    # every e4m3 value, the midpoints between neighbours (ties), +-1 ulp around
    # them, random magnitudes across the whole range, and specials
    vals = oracle.e4m3_to_f32(np.arange(256, dtype=np.uint8))
    finite = np.unique(vals[np.isfinite(vals)])
    mids = (finite[:-1].astype(np.float64) + finite[1:]) / 2
    mids = mids.astype(np.float32)
    around = np.concatenate([np.nextafter(mids, np.float32(np.inf)),
                             np.nextafter(mids, np.float32(-np.inf))])
    rand = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 100,
        (rng.random(200000).astype(np.float32) * 2 - 1) * 0.02,
        np.exp(rng.uniform(-30, 8, 100000)).astype(np.float32),
    ])
    special = np.array([0.0, -0.0, 448.0, 449.0, 464.0, 480.0, 1e6, np.inf, -np.inf,
                        2 ** -9, 2 ** -10, 3 * 2 ** -11, 2 ** -6, -2 ** -6, 1e-30],
                       dtype=np.float32)
    return np.concatenate([finite, -finite, mids, -mids, around, -around, rand, special])


def test_e4m3_rounding_matches_cuda_host_conversion():
    x = _probe_values()
    ours = oracle.f32_to_e4m3(x)
    cuda = oracle.cuda_host_e4m3(x)
    bad = np.nonzero(ours != cuda)[0]
    assert bad.size == 0, [(float(x[i]), int(ours[i]), int(cuda[i])) for i in bad[:10]]
    nan = oracle.f32_to_e4m3(np.array([np.nan], dtype=np.float32))
    assert (nan[0] & 0x7F) == 0x7F


def test_e4m3_rounding_matches_torch_within_range():
    x = _probe_values()
    x = x[np.abs(x) < 448]            # torch does not saturate
    ours = oracle.f32_to_e4m3(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)


def test_e4m3_decode_round_trips():
    codes = np.arange(256, dtype=np.uint8)
    vals = oracle.e4m3_to_f32(codes)
    ok = np.isfinite(vals)
    assert ok.sum() == 254 and vals[0x7E] == 448.0 and vals[0x01] == 2 ** -9
    assert np.array_equal(oracle.f32_to_e4m3(vals[ok]), codes[ok])


def test_block_quantiser_definition():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((200, 300)).astype(np.float32)
    x[0:128, 128:256] = 0.0                      # an all-zero block
    q, s = oracle.quantize_e4m3_block128(x)
    assert s.shape == (2, 3) and s[0, 1] == 1.0
    blk = np.abs(x[128:200, 256:300]).max()
    assert s[1, 2] == np.float32(blk) / np.float32(448.0)
    deq = oracle.e4m3_to_f32(q) * np.repeat(np.repeat(s, 128, 0), 128, 1)[:200, :300]
    assert rel_err(deq, x) < 0.05
    assert np.abs(oracle.e4m3_to_f32(q)).max() <= 448.0


def test_blockscaled_gemm_matches_float64():
    rng = np.random.default_rng(2)
    M, N, K = 130, 256, 384
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    aq, sa = oracle.quantize_e4m3_block128(a)
    wq, sw = oracle.quantize_e4m3_block128(w)
    d = oracle.bf16_to_f32(oracle.gemm_fp8_blockscaled(aq, sa, wq, sw))
    ad = oracle.e4m3_to_f32(aq).astype(np.float64) * np.repeat(np.repeat(sa, 128, 0), 128, 1)[:M]
    wd = oracle.e4m3_to_f32(wq).astype(np.float64) * np.repeat(np.repeat(sw, 128, 0), 128, 1)[:N]
    assert rel_err(d, ad @ wd.T) < 4e-3
