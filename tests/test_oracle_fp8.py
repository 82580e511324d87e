"""Pins the FP8 oracle (oracle/oracle.c) before it is trusted as the checker.

Golden vectors come from the reference's own codec (include/fp8.hpp:15-63,
compiled from its sources by oracle/Makefile) and are committed in
tests/golden/fp8_e4m3_ref_codec.json (generator: tests/golden/make_golden.py).
"""
import json
from pathlib import Path

import numpy as np
import pytest

GOLD = json.loads((Path(__file__).parent / "golden" / "fp8_e4m3_ref_codec.json").read_text())


def test_decode_table_matches_reference_codec(oracle_lib):
    dec = oracle_lib.e4m3_decode_table()
    for code, want in enumerate(GOLD["decode"]):
        if want is None:
            assert np.isnan(dec[code]), code
        else:
            assert dec[code] == np.float32(want), (code, dec[code], want)


def test_decode_table_matches_torch():
    import torch
    import oracle
    dec = oracle.e4m3_decode_table()
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    same = (dec == t) | (np.isnan(dec) & np.isnan(t))
    assert same.all()
    # signed zero: 0x80 decodes to -0.0
    assert np.signbit(dec[0x80]) and dec[0x80] == 0


def test_ampcompat_mode_reproduces_reference_codec_goldens(oracle_lib):
    for key in ("verify_fixes_probes", "midpoints", "edges"):
        x = np.asarray(GOLD[key]["x"], np.float32)
        got = oracle_lib.e4m3_encode(x, mode="amp")
        assert got.tolist() == GOLD[key]["amp"], key
    xs = np.array([int(h, 16) for h in GOLD["sample"]["x_f32_hex"]], np.uint32).view(np.float32)
    assert oracle_lib.e4m3_encode(xs, mode="amp").tolist() == GOLD["sample"]["amp"]


def test_rne_mode_matches_torch_goldens(oracle_lib):
    for key in ("verify_fixes_probes", "midpoints"):
        x = np.asarray(GOLD[key]["x"], np.float32)
        assert oracle_lib.e4m3_encode(x).tolist() == GOLD[key]["torch_rne"], key
    xs = np.array([int(h, 16) for h in GOLD["sample"]["x_f32_hex"]], np.uint32).view(np.float32)
    got = oracle_lib.e4m3_encode(xs)
    want = np.asarray(GOLD["sample"]["torch_rne"])
    fin = np.abs(xs) < 464  # torch's cast does not saturate; saturation checked below
    assert (got[fin] == want[fin]).all()
    assert ((got[~fin] & 0x7F) == 0x7E).all()


def test_rne_and_reference_differ_only_where_documented(oracle_lib):
    """AMP's codec rounds ties away from zero; on the 125 positive midpoints
    about half disagree with RNE (the deviation the oracle documents)."""
    m = GOLD["midpoints"]
    diff = sum(a != b for a, b in zip(m["amp"], m["torch_rne"]))
    assert 55 <= diff <= 70


def test_verify_fixes_roundtrip_property(oracle_lib):
    """tests/verify_fixes.cpp:29-46: >=5 distinct codes over [256,448], <=10% error."""
    x = np.asarray(GOLD["verify_fixes_probes"]["x"], np.float32)
    q = oracle_lib.e4m3_encode(x)
    back = oracle_lib.e4m3_decode_table()[q]
    assert len(set(q.tolist())) >= 5
    assert (np.abs(back - x) / x <= 0.10).all()


def test_rne_exhaustive_sweep_vs_torch(oracle_lib):
    import torch
    pats = np.arange(0, 2 ** 32, 4099, dtype=np.uint64).astype(np.uint32)
    x = pats.view(np.float32)
    got = oracle_lib.e4m3_encode(x)
    t = torch.from_numpy(x.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    nan = np.isnan(x)
    fin = ~nan & (np.abs(x) < 464)
    assert (got[fin] == t[fin]).all()
    assert (got[nan] == 0x7F).all()
    sat = ~nan & ~fin
    assert ((got[sat] & 0x7F) == 0x7E).all()
    assert ((got[sat] & 0x80) == ((pats[sat] >> 24) & 0x80)).all()


def test_ampcompat_sweep_vs_live_reference_codec(oracle_lib):
    r = oracle_lib.ref_lib()
    if r is None:
        pytest.skip("AMP's codec is not built from its sources (make -C oracle ref)")
    pats = np.arange(0, 2 ** 32, 8191, dtype=np.uint64).astype(np.uint32)
    x = pats.view(np.float32)
    q_ref = np.empty(x.size, np.uint8)
    r.ref_f32_to_e4m3_n(x.ctypes.data, x.size, q_ref.ctypes.data)
    assert (oracle_lib.e4m3_encode(x, mode="amp") == q_ref).all()


def test_quant_pipeline_semantics(oracle_lib):
    x = np.array([0.0, 1.0, -2.0, 448.0, 3.5, -0.0], np.float32)
    xb = oracle_lib.f32_to_bf16_bits(x)
    q, s, a = oracle_lib.quant_e4m3(xb)
    assert a == 448.0 and s == np.float32(1.0)
    assert q.tolist() == oracle_lib.e4m3_encode(x).tolist()
    y = oracle_lib.bf16_bits_to_f32(oracle_lib.dequant_e4m3(q, s))
    assert (y == x).all() and np.signbit(y[-1])
    # all-zero tensor: scale 1 by definition
    q0, s0, a0 = oracle_lib.quant_e4m3(np.zeros(7, np.uint16))
    assert a0 == 0.0 and s0 == 1.0 and (q0 == 0).all()
    # empty tensor
    qe, se, ae = oracle_lib.quant_e4m3(np.zeros(0, np.uint16))
    assert qe.size == 0 and se == 1.0


def test_rowwise_and_colwise_are_per_slice_tensors(oracle_lib):
    rng = np.random.default_rng(1)
    x = oracle_lib.f32_to_bf16_bits(rng.standard_normal((5, 9)).astype(np.float32))
    qr, sr = oracle_lib.quant_e4m3_rows(x)
    for r in range(5):
        q, s, _ = oracle_lib.quant_e4m3(x[r])
        assert (qr[r] == q).all() and sr[r] == np.float32(s)
    qc, sc = oracle_lib.quant_e4m3_cols(x)
    for c in range(9):
        q, s, _ = oracle_lib.quant_e4m3(np.ascontiguousarray(x[:, c]))
        assert (qc[:, c] == q).all() and sc[c] == np.float32(s)


def test_subnormal_scale_survives_the_reciprocal_clamp(oracle_lib):
    """A tiny amax gives a subnormal scale whose reciprocal overflows and is clamped
    to FLT_MAX; the scale itself must stay amax/448 (a compiler that infers
    scale == 0 from an infinite reciprocal would return 0)."""
    for a in (1e-38, 3e-39, 1e-39, 2e-40):   # all nonzero in bf16 (min 2^-133)
        x16 = oracle_lib.f32_to_bf16_bits(np.array([a, -a / 2, 0.0], np.float32))
        amax = oracle_lib.bf16_bits_to_f32(x16[:1])[0]
        q, s, got_amax = oracle_lib.quant_e4m3(x16)
        assert got_amax == amax
        assert s == np.float32(amax) / np.float32(448) and s > 0, (a, s)
        # the reciprocal is clamped, so the codes are those of x * FLT_MAX
        big = np.float32(np.finfo(np.float32).max)
        assert np.array_equal(q, oracle_lib.e4m3_encode(oracle_lib.bf16_bits_to_f32(x16) * big))
