"""The oracle's restatement of the true-e4m3 tier (a separately named, non-parity storage mode; the
reference's "FP8" tier is the int8-with-wrap simulation): the e4m3 encoder pinned against torch's
own float8_e4m3fn conversion (round to nearest even) over every finite fp16 value in range and a
dense sweep of fp32 values, the spec's landmark codes, saturation and the tier's row arithmetic."""
import numpy as np
import torch

import oracle


def torch_codes(v):
    return torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def test_encoder_matches_torch_on_every_fp16_value_in_range():
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    h = h[np.isfinite(h) & (np.abs(h) <= 448.0)]
    assert (oracle.e4m3_encode(h) == torch_codes(h)).all()


def test_encoder_matches_torch_on_a_dense_fp32_sweep():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.uniform(-448, 448, 200_000), rng.standard_normal(200_000) * 2.0 ** rng.integers(-12, 8, 200_000),
                        # midpoints between neighbouring codes: ties to even
                        (torch.arange(0, 127, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()[:-1]
                         + torch.arange(1, 127, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()) / 2]).astype(np.float32)
    v = v[np.abs(v) <= 448.0]
    assert (oracle.e4m3_encode(v) == torch_codes(v)).all()


def test_landmarks_saturation_and_nan():
    v = np.array([0.0, -0.0, 1.0, 448.0, 2 ** -9, 2 ** -6, 240.0, 449.0, 464.0, 1e30, np.inf, -np.inf, np.nan],
                 np.float32)
    assert [int(c) for c in oracle.e4m3_encode(v)] == [0x00, 0x80, 0x38, 0x7E, 0x01, 0x08, 0x77, 0x7E, 0x7E, 0x7E,
                                                       0x7E, 0xFE, 0x00]


def test_tier_rows_round_trip():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 128)) * 3).astype(np.float16)
    x[5] = 0.0                               # zero row: scale 0, codes 0, values 0
    q, s = oracle.quantize_to_e4m3(x)
    assert s.dtype == np.float16 and q.dtype == np.uint8
    # the scale is fp16(amax / 448) and the row's largest magnitude lands on 448 (or 1 ulp off)
    amax = np.abs(x.astype(np.float32)).max(1)
    assert (s[:, 0] == (amax / np.float32(448)).astype(np.float16)).all()
    y = oracle.dequantize_from_e4m3(q, s)
    assert (y[5] == 0).all() and (q[5] == 0).all()
    live = np.arange(64) != 5
    rel = np.abs(y[live].astype(np.float32) - x[live].astype(np.float32)) / amax[live, None]
    assert rel.max() < 2.0 ** -4 + 1e-3      # 3 mantissa bits over the row's range
    # decoding is exact: e4m3 values times the fp16 scale, rounded once to fp16
    dec = torch.from_numpy(q).view(torch.float8_e4m3fn).float().numpy()
    assert (y == (dec * s.astype(np.float32)).astype(np.float16)).all()
