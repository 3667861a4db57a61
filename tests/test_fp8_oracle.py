"""The oracle's fp8 E4M3 restatement against torch's float8_e4m3fn conversion (CPU)."""
import numpy as np
import torch

import paged_ref as ref


def test_fp8_encode_matches_torch_cast():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        (rng.standard_normal(200000) * 60).astype(np.float32),
        (rng.standard_normal(20000) * 1e-3).astype(np.float32),          # subnormal range
        np.array([0.0, -0.0, 448.0, -448.0, 447.99, 2.0 ** -10, 2.0 ** -9 * 1.5, 240.0, 232.0],
                 np.float32)])                                              # exact ties included
    ours = ref.fp8_e4m3_encode(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)


def test_fp8_decode_round_trip_and_saturation():
    every = np.arange(256, dtype=np.uint8)
    vals = ref.fp8_e4m3_decode(every)
    finite = ~np.isnan(vals)
    assert np.array_equal(np.isnan(vals), np.isin(every, [0x7F, 0xFF]))
    assert np.array_equal(ref.fp8_e4m3_encode(vals[finite]), every[finite])
    assert np.array_equal(vals, torch.from_numpy(every).view(torch.float8_e4m3fn).float().numpy(),
                          equal_nan=True)
    big = np.array([449.0, 1e6, -5000.0], np.float32)
    assert ref.fp8_e4m3_encode(big).tolist() == [0x7E, 0x7E, 0xFE]
    assert ref.fp8_e4m3_encode(np.array([np.nan], np.float32)).tolist() == [0x7F]
