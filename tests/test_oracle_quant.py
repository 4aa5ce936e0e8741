"""The oracle's dequant pinned by the reference's known-answer tests
(tests/quant.test.ts:6-49 of ahpah-dev/WebGPU 0.9.0, restated with the same
byte fixtures and expected values), and cross-checked against the gguf Python
package's independent K-quant decoder."""
import math

import numpy as np
import pytest

import oracle
from webgpu_b200 import synth


def test_half_to_float_signs_subnormals_inf_nan():
    # quant.test.ts:6-10
    assert oracle.half_to_float(0x3C00) == 1
    assert oracle.half_to_float(0xC000) == -2
    assert oracle.half_to_float(1) == 2 ** -24
    assert oracle.half_to_float(0x7C00) == math.inf
    assert math.isnan(oracle.half_to_float(0x7E00))


def test_q4_0_and_q8_0_signed_blocks_across_blocks():
    # quant.test.ts:11-18
    q4 = np.zeros(36, np.uint8)
    q4[1] = q4[19] = 0x3C
    for i in range(16):
        q4[2 + i] = q4[20 + i] = i | (15 - i) << 4
    got = oracle.decode(q4, 2, 64)
    for i in range(64):
        assert got[i] == (i % 16 - 8 if i % 32 < 16 else 7 - i % 16)
    assert np.array_equal(oracle.decode_f32(q4, 2, 64), got.astype(np.float32))
    q8 = np.zeros(68, np.uint8)
    q8[1] = q8[35] = 0x3C
    for i in range(32):
        q8[2 + i] = q8[36 + i] = (240 + i) & 255  # Uint8Array wraps
    got = oracle.decode(q8, 8, 64)
    for i in range(64):
        assert got[i] == i % 32 - 16
    assert np.array_equal(oracle.decode_f32(q8, 8, 64), got.astype(np.float32))


def kquant_fixture(ttype):
    # quant.test.ts:19-31
    data = np.zeros(144 if ttype == 12 else 176, np.uint8)
    data[1] = data[3] = 0x3C
    scales = [1, 17, 35, 63, 49, 21, 38, 54]
    mins = [62, 34, 18, 2, 57, 43, 29, 15]
    for s in range(8):
        if s < 4:
            data[4 + s] = scales[s]
            data[8 + s] = mins[s]
        else:
            data[8 + s] = (scales[s] & 15) | ((mins[s] & 15) << 4)
            data[s] |= (scales[s] >> 4) << 6
            data[4 + s] |= (mins[s] >> 4) << 6
    base = 16 if ttype == 12 else 48
    for group in range(4):
        for lane in range(32):
            data[base + group * 32 + lane] = (lane & 15) | ((15 - (lane & 15)) << 4)
    if ttype == 13:
        data[16:48] = 0xA5
    expected = []
    for i in range(256):
        s = i // 32
        q = (15 - i % 16 if s % 2 else i % 16) + (16 if ttype == 13 and ((0xA5 >> s) & 1) else 0)
        expected.append(scales[s] * q - mins[s])
    return data, expected


@pytest.mark.parametrize("ttype", [12, 13])
def test_k_quants_six_bit_scales_and_minima(ttype):
    data, expected = kquant_fixture(ttype)
    got = oracle.decode(data, ttype, 256)
    assert list(got) == expected
    assert np.array_equal(oracle.decode_f32(data, ttype, 256), np.array(expected, np.float32))


def q6k_fixture():
    # quant.test.ts:32-45
    data = np.zeros(420, np.uint8)
    expected = np.zeros(512, np.float32)
    for block in range(2):
        base = block * 210
        data[base + 209] = 0x3C
        for j in range(16):
            data[base + 192 + j] = (j - 8) & 255
        for i in range(256):
            value = (i * 7 + block) % 64
            segment, quarter, lane = i // 128, (i % 128) // 32, i % 32
            data[base + segment * 64 + quarter % 2 * 32 + lane] |= (value & 15) << ((quarter // 2) * 4)
            data[base + 128 + segment * 32 + lane] |= (value >> 4) << (quarter * 2)
            expected[block * 256 + i] = (value - 32) * (i // 16 - 8)
    return data, expected


def test_q6_k_quarters_and_signed_scales():
    data, expected = q6k_fixture()
    got = oracle.decode(data, 14, 512)
    assert np.array_equal(got, expected.astype(np.float64))
    assert np.array_equal(oracle.decode_f32(data, 14, 512), expected)


def test_greedy_skips_nan_and_reports_all_nonfinite():
    # quant.test.ts:46-49
    assert oracle.greedy(np.array([np.nan, -2, 7, 3], np.float32)) == 2
    assert oracle.greedy(np.array([np.nan, -np.inf], np.float32)) == -1


GGUF_TYPES = {2: "Q4_0", 8: "Q8_0", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}


@pytest.mark.parametrize("ttype", sorted(GGUF_TYPES))
def test_cross_check_with_gguf_package(ttype):
    """Independent decoder (gguf-py's numpy dequantize) on random blocks."""
    gq = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType
    nblocks = 64
    raw = synth.random_blocks(ttype, nblocks, seed=5, stream=ttype, scale_std=1e-2)
    be = synth.BLOCK[ttype][0]
    ours = oracle.decode(raw, ttype, nblocks * be)
    theirs = gq.dequantize(raw.reshape(1, -1), GGMLQuantizationType[GGUF_TYPES[ttype]]).astype(np.float64).reshape(-1)
    # gguf-py computes in f32; our f64 values rounded to f32 must agree to f32 rounding.
    np.testing.assert_allclose(ours, theirs, rtol=2e-6, atol=1e-9)


@pytest.mark.parametrize("ttype", [0, 1, 2, 8, 12, 13, 14])
def test_f32_twin_within_one_ulp_of_f64(ttype):
    """The WGSL-order fp32 dequant is the f64 value rounded once or twice: within 1 ulp."""
    be = synth.BLOCK[ttype][0]
    nblocks = 256 // be * 8 if be < 256 else 8
    raw = synth.random_blocks(ttype, nblocks, seed=9, stream=ttype)
    n = nblocks * be
    f64 = oracle.decode(raw, ttype, n)
    f32 = oracle.decode_f32(raw, ttype, n).astype(np.float64)
    finite = np.isfinite(f64)
    ulp = np.spacing(np.abs(f64[finite]).astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(f32[finite] - f64[finite]) <= ulp + 1e-45)


@pytest.mark.parametrize("ttype", [0, 1, 2, 8, 12, 13, 14])
def test_hoisted_row_decoder_is_bit_identical(ttype):
    """The oracle's fast row decoder equals the literal decodeWeight restatement bitwise."""
    import ctypes
    L = oracle.lib()
    L.or_dequant_row_matches.restype = ctypes.c_int
    L.or_dequant_row_matches.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64]
    cols = 2048
    be = synth.BLOCK[ttype][0]
    raw = synth.random_blocks(ttype, cols // be, seed=21, stream=ttype)
    assert L.or_dequant_row_matches(ctypes.c_void_p(raw.ctypes.data), ttype, cols) == 1
