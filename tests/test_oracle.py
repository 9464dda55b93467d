"""CPU: the oracle restatements against the reference's golden vectors (no GPU)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import c_oracle
from oracle import iq3s_oracle as O


def test_codebook_magnitudes_and_fp8_encoding():
    # test_iq3_s_fp8.py:71-81: every E4M3 byte decodes to its magnitude, |0x80 to its negation.
    raw = O.iq3s_grid_u32()
    enc = O.iq3s_fp8_table()
    assert raw.shape == enc.shape == (512,) and raw.dtype == enc.dtype == np.uint32
    shifts = (0, 8, 16, 24)
    mags = np.stack([(raw >> s) & 0xFF for s in shifts], -1).astype(np.float32)
    bits = np.stack([(enc >> s) & 0xFF for s in shifts], -1).astype(np.uint8)
    assert set(np.unique(mags)) == {1, 3, 5, 7, 9, 11, 13, 15}
    np.testing.assert_array_equal(O.decode_e4m3(bits), mags)
    np.testing.assert_array_equal(O.decode_e4m3(bits | np.uint8(0x80)), -mags)


def test_codebook_known_entries():
    # First entries of ggml's iq3s_grid (all magnitudes 1, then 3,1,1,1 ...).
    raw = O.iq3s_grid_u32()
    assert raw[0] == 0x01010101 and raw[1] == 0x01010103


def test_decode_matches_gguf_golden(golden):
    g = golden["iq3s_decode"]
    np.testing.assert_array_equal(O.dequantize_iq3s(g["synth_raw"]), g["synth_deq"])


def test_decode_all_codes_and_sign_nibbles_bit_exact(golden):
    g = golden["iq3s_decode"]
    np.testing.assert_array_equal(O.dequantize_iq3s(g["allcodes_raw"]), g["allcodes_deq"])
    q, s = O.decode_iq3s_fp8(g["allcodes_raw"])
    np.testing.assert_array_equal(O.decode_e4m3(q) * np.repeat(s, 32, axis=1), g["allcodes_deq"])
    # the generator reproduces the fixture
    np.testing.assert_array_equal(O.make_all_codes_iq3s(), g["allcodes_raw"])


def test_c_oracle_decode_matches(golden):
    g = golden["iq3s_decode"]
    for key in ("synth", "allcodes"):
        np.testing.assert_array_equal(c_oracle.dequantize_iq3s(g[f"{key}_raw"]), g[f"{key}_deq"])


def test_soa_fields_preserve_every_byte(golden):
    raw = golden["iq3s_decode"]["soa_raw"]
    n, b, _ = raw.shape
    f = O.prepare_fields(raw)
    rec = np.empty_like(raw)
    for name, start, size in O.FIELD_LAYOUT:
        rec[..., start:start + size] = f[name].view(np.uint8).reshape(b, n, size).transpose(1, 0, 2)
    np.testing.assert_array_equal(rec, raw)
    assert f["qs"].shape == (b, n, 16) and f["qh"].shape == (b, n, 4) and f["signs"].shape == (b, n, 8)


@pytest.mark.parametrize("m", [5, 33, 128])
def test_mxfp8_matches_reference_oracle(golden, m):
    g = golden["mxfp8"]
    x = g[f"x_{m}"]
    for rounding in ("rne", "ties_down"):
        q, s = O.quantize_mxfp8(x, rounding)
        np.testing.assert_array_equal(q, g[f"q_{m}"])  # tie-free f32 inputs: both rules agree
        np.testing.assert_array_equal(s, g[f"s_{m}"])
    np.testing.assert_array_equal(O.quantize_mxfp8(x)[0], g[f"q_rne_{m}"])
    qc, sc = c_oracle.quantize_mxfp8(x, "rne")
    np.testing.assert_array_equal(qc, g[f"q_{m}"])
    np.testing.assert_array_equal(sc, g[f"s_{m}"])
    assert np.count_nonzero(O.decode_mxfp8(*O.quantize_mxfp8(x))[0]) == 0


def test_mxfp8_bf16_tie_rules(golden):
    g = golden["mxfp8"]
    x = (g["xbf16_bits"].astype(np.uint32) << 16).view(np.float32)
    q_rne, s = O.quantize_mxfp8(x, "rne")
    q_td, s2 = O.quantize_mxfp8(x, "ties_down")
    np.testing.assert_array_equal(s, g["s_bf16"])
    np.testing.assert_array_equal(s2, g["s_bf16"])
    np.testing.assert_array_equal(q_rne, g["q_bf16_rne"])
    np.testing.assert_array_equal(q_td, g["q_bf16_ties_down"])
    np.testing.assert_array_equal(c_oracle.quantize_mxfp8(x, "ties_down")[0], g["q_bf16_ties_down"])
    # bf16 inputs hit exact ties often; the two rules then differ by one code.
    diff = np.mean(q_rne != q_td)
    assert 0.01 < diff < 0.06


def test_mxfp8_exponent_edges():
    amax = np.array([0.0, 448.0, 448.0000305, 1.0, 2.0 ** -130, 3.0e38, 1.75 * 2.0 ** -119, 1.75 * 2.0 ** -118])
    e = O.mxfp8_exponent(amax)
    assert list(e[:4]) == [0, 0, 1, -8]
    assert e[4] == -127 and e[5] == 120 and e[6] == -127 and e[7] == -126


@pytest.mark.parametrize("m", [3, 4, 5, 8, 9, 33, 128, 129])
def test_linear_oracle_matches_golden(golden, m):
    g = golden["linear"]
    rng = np.random.default_rng(20261016)
    x = rng.standard_normal((m, 768), dtype=np.float32)
    import hashlib

    assert hashlib.sha256(x.tobytes()).hexdigest().encode() == g[f"x_sha_{m}"].tobytes()
    q, s = O.quantize_mxfp8(x)
    np.testing.assert_array_equal(q, g[f"q_{m}"])
    np.testing.assert_array_equal(s, g[f"s_{m}"])
    out = O.iq3s_linear_f64(q, s, g["raw"])
    np.testing.assert_allclose(out, g[f"out_{m}"], rtol=1e-6, atol=1e-6)
    out_c = c_oracle.iq3s_linear_f64(q, s, g["raw"], threads=2)
    np.testing.assert_allclose(out_c, out, rtol=1e-12, atol=1e-12)


def test_oracle_planted_mistake_is_caught(golden):
    # A decode with one flipped sign bit must not pass the bit-exact check.
    raw = golden["iq3s_decode"]["allcodes_raw"].copy()
    raw[0, 0, 74] ^= 1
    assert not np.array_equal(O.dequantize_iq3s(raw), golden["iq3s_decode"]["allcodes_deq"])
