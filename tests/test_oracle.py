"""CPU tests that pin the oracle (oracle/gemm_oracle.c) to the reference.

The reference (Zig + Bazel) cannot be built here, so the oracle is pinned by
(1) the known-answer values in the reference's own tests (tests/golden/
reference_kats.json, each entry citing its source line), and (2) the
second, independent restatements those tests carry (`referenceReal`,
tests/gemm_correctness.zig:243-286; the f32 loop of
tests/gemm_correctness.zig:210-218), re-stated here in numpy float32 /
Python float arithmetic.
"""
import json
import os
import re

import numpy as np
import pytest

import oracle as orc

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))
HEADER = os.path.join(os.path.dirname(HERE), "include", "gemm_sm100.h")

F32 = np.float32


def layout_idx(layout, ld, r, c):
    return r * ld + c if layout == orc.ROW_MAJOR else r + c * ld


def len_for(layout, rows, cols, ld):
    return (rows - 1) * ld + cols if layout == orc.ROW_MAJOR else (cols - 1) * ld + rows


def min_ld(layout, rows, cols):
    return max(1, cols if layout == orc.ROW_MAJOR else rows)


def reference_real(op_a, op_b, m, n, k, alpha, a, al, sa, b, bl, sb, beta, c, cl, sc, batch):
    """`referenceReal` of tests/gemm_correctness.zig:243-286 in float32 scalar arithmetic."""
    def idx(l, r, col):
        return l[0] + r * l[1] + col * l[2]

    alpha, beta = F32(alpha), F32(beta)
    for bt in range(batch):
        for row in range(m):
            for col in range(n):
                s = F32(0)
                for kk in range(k):
                    av = a[bt * sa + (idx(al, row, kk) if op_a == 0 else idx(al, kk, row))]
                    bv = b[bt * sb + (idx(bl, kk, col) if op_b == 0 else idx(bl, col, kk))]
                    s = F32(s + F32(av * bv))
                ci = bt * sc + idx(cl, row, col)
                c[ci] = F32(F32(alpha * s) + F32(beta * c[ci]))


# ---- enums and codecs ------------------------------------------------------

def test_enum_values_match_reference():
    kat = KATS["enum_values"]
    text = open(HEADER).read()

    def hdr(name):
        return int(re.search(rf"\b{name}\s*=\s*(-?\d+)", text).group(1))

    assert hdr("GS_R_32F") == kat["r_32f"] == orc.R_32F
    assert hdr("GS_R_64F") == kat["r_64f"] == orc.R_64F
    assert hdr("GS_R_16F") == kat["r_16f"] == orc.R_16F
    assert hdr("GS_R_16BF") == kat["r_16bf"] == orc.R_16BF
    assert orc.R_8F_E4M3 == kat["r_8f_e4m3"] and orc.R_4F_E2M1 == kat["r_4f_e2m1"]
    assert hdr("GS_COMPUTE_32F") == kat["compute_f32"]
    assert hdr("GS_GEMM_DEFAULT") == kat["algo_default"]
    ops = KATS["op_values"]
    assert (hdr("GS_OP_N"), hdr("GS_OP_T"), hdr("GS_OP_C")) == (ops["n"], ops["t"], ops["c"])


def test_low_precision_decoders_finite():
    for dtype, bits in KATS["decoders_finite"]["cases"]:
        re_, im = orc.read_scalar(bytes([bits]), dtype, 0)
        assert np.isfinite(re_) and im == 0.0


def test_f16_codec_matches_ieee_rne():
    rng = np.random.default_rng(1)
    xs = np.concatenate([
        rng.standard_normal(20000).astype(F32) * F32(4),
        (rng.standard_normal(5000) * 1e-5).astype(F32),      # subnormal range of f16
        (rng.standard_normal(2000) * 7e4).astype(F32),       # overflow range
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08,
                  np.inf, -np.inf], dtype=F32),
    ])
    ours = np.array([orc.f32_to_f16_bits(float(x)) for x in xs], dtype=np.uint16)
    np.testing.assert_array_equal(ours, xs.astype(np.float16).view(np.uint16))
    bits = np.arange(0, 65536, 7, dtype=np.uint16)
    bits = bits[(bits & 0x7C00) != 0x7C00]  # finite only
    back = np.array([orc.f16_bits_to_f32(int(b)) for b in bits], dtype=F32)
    np.testing.assert_array_equal(back, bits.view(np.float16).astype(F32))


def test_bf16_codec_is_reference_formula():
    rng = np.random.default_rng(2)
    xs = rng.standard_normal(5000).astype(F32)
    ours = np.array([orc.f32_to_bf16_bits(float(x)) for x in xs], dtype=np.uint16)
    raw = xs.view(np.uint32).astype(np.uint64)
    expect = (((raw + 0x7FFF + ((raw >> 16) & 1)) & 0xFFFFFFFF) >> 16).astype(np.uint16)
    np.testing.assert_array_equal(ours, expect)
    np.testing.assert_array_equal(orc.bf16_round_array(xs), expect)
    for b in (0x3F80, 0xBF80, 0x0001, 0x7F7F):
        assert orc.bf16_bits_to_f32(b) == np.array([b << 16], dtype=np.uint32).view(F32)[0]


# ---- known answers ---------------------------------------------------------

def test_alpha_beta_zero_kat():
    kat = KATS["alpha_beta_zero"]
    a = np.array(kat["a"], dtype=F32)
    b = np.array(kat["b"], dtype=F32)
    for case in kat["cases"]:
        c = np.array(kat["c"], dtype=F32)
        rc = orc.sgemm(orc.ROW_MAJOR, 0, 0, kat["m"], kat["n"], kat["k"], case["alpha"], a, kat["lda"], b,
                       kat["ldb"], case["beta"], c, kat["ldc"])
        assert rc == orc.OK
        np.testing.assert_array_equal(c, np.array(case["expected"], dtype=F32))


@pytest.mark.parametrize("op_a", [0, 1, 2])
@pytest.mark.parametrize("op_b", [0, 1, 2])
def test_sgemm_transpose_variants_bit_exact(op_a, op_b):
    kat = KATS["real_transpose_variants"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    for run in kat["runs"]:
        layout = orc.ROW_MAJOR if run["layout"] == "row_major" else orc.COL_MAJOR
        ar, ac = (m, k) if op_a == 0 else (k, m)
        br, bc = (k, n) if op_b == 0 else (n, k)
        lda = min_ld(layout, ar, ac) + kat["lda_pad"]
        ldb = min_ld(layout, br, bc) + kat["ldb_pad"]
        ldc = min_ld(layout, m, n) + kat["ldc_pad"]
        a = orc.value_for(np.arange(len_for(layout, ar, ac, lda)), kat["fill_bias"]["a"])
        b = orc.value_for(np.arange(len_for(layout, br, bc, ldb)), kat["fill_bias"]["b"])
        c = orc.value_for(np.arange(len_for(layout, m, n, ldc)), kat["fill_bias"]["c"])
        expected = c.copy()
        lay = lambda ld: (0, ld, 1) if layout == orc.ROW_MAJOR else (0, 1, ld)  # noqa: E731
        reference_real(op_a, op_b, m, n, k, run["alpha"], a, lay(lda), 0, b, lay(ldb), 0, run["beta"], expected,
                       lay(ldc), 0, 1)
        assert orc.sgemm(layout, op_a, op_b, m, n, k, run["alpha"], a, lda, b, ldb, run["beta"], c, ldc) == orc.OK
        np.testing.assert_array_equal(c, expected)  # identical f32 operation order => bit-exact
        assert np.max(np.abs(c - expected)) <= kat["tol_f32"]


def test_strided_batched_descriptor():
    kat = KATS["strided_batched_descriptor"]
    m, n, k, batch = kat["m"], kat["n"], kat["k"], kat["batch"]
    sa, sb, sc = kat["stride_a"], kat["stride_b"], kat["stride_c"]
    a = orc.value_for(np.arange(sa * batch), kat["fill_bias"]["a"])
    b = orc.value_for(np.arange(sb * batch), kat["fill_bias"]["b"])
    c = orc.value_for(np.arange(sc * batch), kat["fill_bias"]["c"])
    expected = c.copy()
    reference_real(0, 1, m, n, k, kat["alpha"], a, kat["a_layout"], sa, b, kat["b_layout"], sb, kat["beta"],
                   expected, kat["c_layout"], sc, batch)
    rc = orc.gemm_f32(0, 1, m, n, k, kat["alpha"], a, kat["a_layout"], b, kat["b_layout"], kat["beta"], c,
                      kat["c_layout"], batch, sa, sb, sc)
    assert rc == orc.OK
    np.testing.assert_array_equal(c, expected)


@pytest.mark.parametrize("bf16", [False, True])
def test_gemm_ex_legacy_and_generic_lowp(bf16):
    kat = KATS["gemm_ex_legacy"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    tol = kat["tol"]["bf16" if bf16 else "f16"]
    enc = (lambda x: orc.bf16_round_array(x)) if bf16 else (lambda x: x.astype(np.float16).view(np.uint16))
    dec = (lambda u: orc.bf16_bits_to_f32_array(u)) if bf16 else (lambda u: u.view(np.float16).astype(F32))
    a = enc(orc.value_for(np.arange(m * k), kat["fill_bias"]["a"]))
    b = enc(orc.value_for(np.arange(k * n), kat["fill_bias"]["b"]))
    c0 = orc.value_for(np.arange(m * n), kat["fill_bias"]["c"])
    # the test's own expected values: f32 accumulation over decoded inputs (tests/gemm_correctness.zig:210-218)
    ad, bd = dec(a), dec(b)
    expected = np.empty(m * n, dtype=F32)
    for row in range(m):
        for col in range(n):
            s = F32(0)
            for kk in range(k):
                s = F32(s + F32(ad[row * k + kk] * bd[kk * n + col]))
            expected[row * n + col] = F32(F32(F32(kat["alpha"]) * s) - F32(F32(0.5) * c0[row * n + col]))
    c = c0.copy()
    rc = orc.gemm_ex_legacy(bf16, 0, 0, m, n, k, a, (0, k, 1), b, (0, n, 1), c, (0, n, 1), kat["alpha"], kat["beta"])
    assert rc == orc.OK
    assert np.max(np.abs(c - expected)) <= tol
    # generic gemmEx (f64 accumulation) agrees within the same tolerance
    c2 = c0.copy()
    dt = orc.R_16BF if bf16 else orc.R_16F
    rc = orc.gemm_ex(0, 0, m, n, k, kat["alpha"], a, dt, k, b, dt, n, kat["beta"], c2, orc.R_32F, n,
                     layout=orc.ROW_MAJOR)
    assert rc == orc.OK
    assert np.max(np.abs(c2 - expected)) <= tol


def test_generic_gemm_ex_f32_bytes_matches_sgemm():
    kat = KATS["gemm_ex_f32_bytes_equals_sgemm"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    a = orc.value_for(np.arange(m * k), kat["fill_bias"]["a"])
    b = orc.value_for(np.arange(k * n), kat["fill_bias"]["b"])
    c = orc.value_for(np.arange(m * n), kat["fill_bias"]["c"])
    expected = c.copy()
    assert orc.sgemm(orc.ROW_MAJOR, 0, 0, m, n, k, kat["alpha"], a, k, b, n, kat["beta"], expected, n) == orc.OK
    assert orc.gemm_ex(0, 0, m, n, k, kat["alpha"], a, orc.R_32F, k, b, orc.R_32F, n, kat["beta"], c, orc.R_32F, n,
                       layout=orc.ROW_MAJOR) == orc.OK
    assert np.max(np.abs(c - expected)) <= kat["tol"]


@pytest.mark.parametrize("dt", [orc.R_16F, orc.R_16BF])
def test_strided_lowp_equals_per_batch(dt):
    kat = KATS["strided_lowp_equals_per_batch"]
    m, n, k, batch = kat["m"], kat["n"], kat["k"], kat["batch"]
    tol = kat["tol"]["f16" if dt == orc.R_16F else "bf16"]
    enc = (lambda x: x.astype(np.float16).view(np.uint16)) if dt == orc.R_16F else orc.bf16_round_array
    sa, sb, sc = m * k, k * n, m * n
    a = enc(orc.value_for(np.arange(sa * batch), kat["fill_bias"]["a"]))
    b = enc(orc.value_for(np.arange(sb * batch), kat["fill_bias"]["b"]))
    c = orc.value_for(np.arange(sc * batch), kat["fill_bias"]["c"])
    expected = c.copy()
    for bt in range(batch):
        ea = a[bt * sa:(bt + 1) * sa].copy()
        eb = b[bt * sb:(bt + 1) * sb].copy()
        ec = expected[bt * sc:(bt + 1) * sc].copy()
        assert orc.gemm_ex_legacy(dt == orc.R_16BF, 0, 0, m, n, k, ea, (0, k, 1), eb, (0, n, 1), ec, (0, n, 1),
                                  1.0, 0.0) == orc.OK
        expected[bt * sc:(bt + 1) * sc] = ec
    assert orc.gemm_ex(0, 0, m, n, k, 1.0, a, dt, k, b, dt, n, 0.0, c, orc.R_32F, n, layout=orc.ROW_MAJOR,
                       batch=batch, sa=sa, sb=sb, sc=sc) == orc.OK
    assert np.max(np.abs(c - expected)) <= tol


def test_pointer_array_batched_ex():
    kat = KATS["pointer_array_batched"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    fb = kat["fill_bias"]
    a = [orc.value_for(np.arange(m * k), fb["a0"]), orc.value_for(np.arange(m * k), fb["a1"])]
    b = [orc.value_for(np.arange(k * n), fb["b0"]), orc.value_for(np.arange(k * n), fb["b1"])]
    c = [orc.value_for(np.arange(m * n), fb["c0"]), orc.value_for(np.arange(m * n), fb["c1"])]
    e = [x.copy() for x in c]
    for i in range(2):
        assert orc.sgemm(orc.ROW_MAJOR, 0, 0, m, n, k, 1.0, a[i], k, b[i], n, 0.0, e[i], n) == orc.OK
    assert orc.gemm_batched_ex(0, 0, m, n, k, 1.0, a, orc.R_32F, k, b, orc.R_32F, n, 0.0, c, orc.R_32F, n,
                               layout=orc.ROW_MAJOR) == orc.OK
    for i in range(2):
        assert np.max(np.abs(c[i] - e[i])) <= kat["tol"]
    # length mismatch -> InvalidBatchCount (src/gemm.zig:637)
    assert orc.gemm_batched_ex(0, 0, m, n, k, 1.0, a, orc.R_32F, k, b[:1], orc.R_32F, n, 0.0, c, orc.R_32F, n,
                               layout=orc.ROW_MAJOR) == orc.ERR_INVALID_BATCH_COUNT


def test_padded_ld_column_major_shapes():
    kat = KATS["cublas_padded_ld_shapes"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    for op_a in (0, 1, 2):
        for op_b in (0, 1, 2):
            ar, ac = (m, k) if op_a == 0 else (k, m)
            br, bc = (k, n) if op_b == 0 else (n, k)
            lda, ldb, ldc = ar + kat["lda_pad"], br + kat["ldb_pad"], m + kat["ldc_pad"]
            a = orc.value_for(np.arange((ac - 1) * lda + ar), kat["fill_bias"]["a"])
            b = orc.value_for(np.arange((bc - 1) * ldb + br), kat["fill_bias"]["b"])
            c = orc.value_for(np.arange((n - 1) * ldc + m), kat["fill_bias"]["c"])
            expected = c.copy()
            reference_real(op_a, op_b, m, n, k, kat["alpha"], a, (0, 1, lda), 0, b, (0, 1, ldb), 0, kat["beta"],
                           expected, (0, 1, ldc), 0, 1)
            assert orc.sgemm(orc.COL_MAJOR, op_a, op_b, m, n, k, kat["alpha"], a, lda, b, ldb, kat["beta"], c,
                             ldc) == orc.OK
            np.testing.assert_array_equal(c, expected)


# ---- gemmExCuda arithmetic, restated independently -----------------------

def py_gemm_ex(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, dec, batch=1, sa=0, sb=0, sc=0,
               layout=orc.COL_MAJOR):
    """gemmExCuda (src/gemm.zig:671-706) in Python floats (f64): sequential-k sum, then alpha*sum + beta*old."""
    out = {}
    for bt in range(batch):
        for row in range(m):
            for col in range(n):
                s = 0.0
                for kk in range(k):
                    ia = layout_idx(layout, lda, row, kk) if op_a == 0 else layout_idx(layout, lda, kk, row)
                    ib = layout_idx(layout, ldb, kk, col) if op_b == 0 else layout_idx(layout, ldb, col, kk)
                    s += float(dec(a[bt * sa + ia])) * float(dec(b[bt * sb + ib]))
                ci = bt * sc + layout_idx(layout, ldc, row, col)
                out[ci] = alpha * s + beta * float(c[ci])
    return out


@pytest.mark.parametrize("dt", [orc.R_16F, orc.R_16BF, orc.R_8I])
@pytest.mark.parametrize("layout", [orc.COL_MAJOR, orc.ROW_MAJOR])
def test_gemm_ex_matches_python_restatement(dt, layout):
    rng = np.random.default_rng(10 + dt + layout)
    m, n, k, batch = 7, 5, 9, 2
    for op_a in (0, 1):
        for op_b in (0, 1):
            ar, ac = (m, k) if op_a == 0 else (k, m)
            br, bc = (k, n) if op_b == 0 else (n, k)
            lda, ldb, ldc = min_ld(layout, ar, ac) + 1, min_ld(layout, br, bc) + 2, min_ld(layout, m, n) + 3
            sa, sb, sc = len_for(layout, ar, ac, lda) + 4, len_for(layout, br, bc, ldb), len_for(layout, m, n, ldc)
            if dt == orc.R_8I:
                a = rng.integers(-128, 128, sa * batch).astype(np.int8)
                b = rng.integers(-128, 128, sb * batch).astype(np.int8)
                c = rng.integers(-1000, 1000, sc * batch).astype(np.int32)
                ct, alpha, beta = orc.R_32I, 3.0, -2.0
                dec = int
            else:
                a = orc.randn_lowp(rng, sa * batch, dt)
                b = orc.randn_lowp(rng, sb * batch, dt)
                c = rng.standard_normal(sc * batch).astype(F32)
                ct, alpha, beta = orc.R_32F, 1.5, 0.5
                dec = (lambda u: np.array([u], np.uint16).view(np.float16)[0]) if dt == orc.R_16F else \
                    (lambda u: orc.bf16_bits_to_f32_array(np.array([u], np.uint16))[0])
            exp = py_gemm_ex(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, dec, batch, sa, sb, sc, layout)
            got = c.copy()
            rc = orc.gemm_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, got, ct, ldc,
                             compute_type=72 if dt == orc.R_8I else 68, layout=layout, batch=batch, sa=sa, sb=sb,
                             sc=sc)
            assert rc == orc.OK
            for ci, v in exp.items():
                if ct == orc.R_32I:
                    assert got[ci] == int(np.clip(np.sign(v) * np.floor(abs(v) + 0.5), -2**31, 2**31 - 1))
                else:
                    assert got[ci] == np.float32(v)  # single rounding f64 -> f32
            untouched = np.ones(c.size, bool)
            untouched[list(exp.keys())] = False
            np.testing.assert_array_equal(got[untouched], c[untouched])


def test_i32_output_rounds_half_away_and_clamps():
    # alpha = 0.5 on odd sums exercises clampInt's @round (half away from zero)
    a = np.array([3, -3, 1, 127], dtype=np.int8)  # 4x1 column
    b = np.array([1], dtype=np.int8)
    c = np.zeros(4, dtype=np.int32)
    assert orc.gemm_ex(0, 0, 4, 1, 1, 0.5, a, orc.R_8I, 4, b, orc.R_8I, 1, 0.0, c, orc.R_32I, 4,
                       compute_type=72) == orc.OK
    np.testing.assert_array_equal(c, [2, -2, 1, 64])
    c = np.array([2**31 - 1, -2**31, 0, 0], dtype=np.int32)
    assert orc.gemm_ex(0, 0, 4, 1, 1, 1.0, a, orc.R_8I, 4, b, orc.R_8I, 1, 1.0, c, orc.R_32I, 4,
                       compute_type=72) == orc.OK
    np.testing.assert_array_equal(c, [2**31 - 1, -2**31, 1, 127])


def test_validation_errors():
    a = np.zeros(6, np.uint16)
    b = np.zeros(6, np.uint16)
    c = np.zeros(4, F32)
    assert orc.gemm_ex(0, 0, 2, 2, 3, 1.0, a, orc.R_16F, 2, b, orc.R_16F, 3, 0.0, c, orc.R_32F, 2,
                       batch=0) == orc.ERR_INVALID_BATCH_COUNT
    assert orc.gemm_ex(0, 0, 2, 2, 3, 1.0, a, orc.R_16F, 2, b, orc.R_16F, 3, 0.0, c, orc.R_32F, 2, batch=2,
                       sa=3) == orc.ERR_INVALID_STRIDE
    assert orc.gemm_ex(0, 0, 2, 2, 3, 1.0, a, orc.R_16F, 2, b, orc.R_16F, 3, 0.0, c, orc.R_32F, 2,
                       batch=2) == orc.ERR_BUFFER_TOO_SMALL
    assert orc.gemm_ex(0, 0, 0, 0, 0, 1.0, a, orc.R_16F, 1, b, orc.R_16F, 1, 0.0, c, orc.R_32F, 1) == orc.OK


@pytest.mark.parametrize("dt", [orc.R_16F, orc.R_8I])
def test_multithreaded_oracle_is_bit_identical(dt):
    rng = np.random.default_rng(5)
    m, n, k, batch = 33, 29, 41, 3
    if dt == orc.R_8I:
        a = rng.integers(-128, 128, m * k * batch).astype(np.int8)
        b = rng.integers(-128, 128, k * n * batch).astype(np.int8)
        c = rng.integers(-50, 50, m * n * batch).astype(np.int32)
        ct, comp = orc.R_32I, 72
    else:
        a = orc.randn_lowp(rng, m * k * batch, dt)
        b = orc.randn_lowp(rng, k * n * batch, dt)
        c = rng.standard_normal(m * n * batch).astype(F32)
        ct, comp = orc.R_32F, 68
    c1, c2 = c.copy(), c.copy()
    args = (1, 0, m, n, k, 1.25, a, dt, k, b, dt, k, -0.75)
    assert orc.gemm_ex(*args, c1, ct, m, compute_type=comp, batch=batch) == orc.OK
    assert orc.gemm_ex(*args, c2, ct, m, compute_type=comp, batch=batch, threads=4) == orc.OK
    np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))
    # sampled checker gives the same entries without modifying C
    rows = rng.integers(0, m, 50)
    cols = rng.integers(0, n, 50)
    bts = rng.integers(0, batch, 50)
    c3 = c.copy()
    rc, vals = orc.gemm_ex_entries(args + (c3, ct, m), dict(compute_type=comp, batch=batch), bts, rows, cols,
                                   c.dtype)
    assert rc == orc.OK
    np.testing.assert_array_equal(c3, c)
    np.testing.assert_array_equal(vals, c1[bts * m * n + rows + cols * m])


def test_sgemm_mt_is_bit_identical():
    rng = np.random.default_rng(6)
    m, n, k = 40, 37, 50
    a = rng.standard_normal(m * k).astype(F32)
    b = rng.standard_normal(k * n).astype(F32)
    c = rng.standard_normal(m * n).astype(F32)
    c1, c2 = c.copy(), c.copy()
    assert orc.sgemm(orc.COL_MAJOR, 0, 1, m, n, k, 1.5, a, m, b, n, 0.5, c1, m) == orc.OK
    assert orc.sgemm_strided_batched_mt(orc.COL_MAJOR, 0, 1, m, n, k, 1.5, a, m, 0, b, n, 0, 0.5, c2, m, 0, 1,
                                        3) == orc.OK
    np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))


def test_hgemm_rounds_to_f16():
    rng = np.random.default_rng(7)
    m, n, k = 6, 5, 8
    a = orc.randn_lowp(rng, m * k, orc.R_16F)
    b = orc.randn_lowp(rng, k * n, orc.R_16F)
    c = orc.randn_lowp(rng, m * n, orc.R_16F)
    got = c.copy()
    alpha, beta = orc.f32_to_f16_bits(1.5), orc.f32_to_f16_bits(-0.5)
    assert orc.hgemm(orc.COL_MAJOR, 0, 0, m, n, k, alpha, a, m, b, k, beta, got, m) == orc.OK
    ad, bd, cd = (x.view(np.float16).astype(F32) for x in (a, b, c))
    for row in range(m):
        for col in range(n):
            s = F32(0)
            for kk in range(k):
                s = F32(s + F32(ad[row + kk * m] * bd[kk + col * k]))
            v = F32(F32(F32(1.5) * s) + F32(F32(-0.5) * cd[row + col * m]))
            assert got[row + col * m] == np.array([v], F32).astype(np.float16).view(np.uint16)[0]


@pytest.mark.parametrize("op_a", [0, 1])
@pytest.mark.parametrize("op_b", [0, 1])
def test_int8_checksum_identities_and_layout_duality_are_exact(op_a, op_b):
    """The size-independent properties the full-size GPU tests check, pinned on the oracle itself: with
    alpha 1 and beta 0 an INT8 GEMM is exact, so the column sums of C equal (1^T op(A)) op(B) and the row
    sums equal op(A) (op(B) 1) in int64; and a row-major call equals the column-major call on the same
    bytes with the operands swapped (C^T = op(B)^T op(A)^T), element for element."""
    rng = np.random.default_rng(20 + 2 * op_a + op_b)
    m, n, k = 23, 17, 300  # |sums| reach 128 * 128 * 300, far beyond int16
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    a = rng.integers(-128, 128, ar * ac).astype(np.int8)
    b = rng.integers(-128, 128, br * bc).astype(np.int8)
    c = np.zeros(m * n, np.int32)
    assert orc.gemm_ex(op_a, op_b, m, n, k, 1.0, a, orc.R_8I, ar, b, orc.R_8I, br, 0.0, c, orc.R_32I, m,
                       compute_type=72) == orc.OK
    am = a.astype(np.int64).reshape(ac, ar).T  # stored column-major, ar x ac
    bm = b.astype(np.int64).reshape(bc, br).T
    opa, opb = (am if op_a == 0 else am.T), (bm if op_b == 0 else bm.T)
    cm = c.astype(np.int64).reshape(n, m).T
    np.testing.assert_array_equal(cm.sum(axis=0), opa.sum(axis=0) @ opb)
    np.testing.assert_array_equal(cm.sum(axis=1), opa @ opb.sum(axis=1))
    # The same matrices stored row-major (leading dimension = stored columns) give the same C, row-major.
    a_rm = np.ascontiguousarray(am).astype(np.int8).ravel()
    b_rm = np.ascontiguousarray(bm).astype(np.int8).ravel()
    c_rm = np.zeros(m * n, np.int32)
    assert orc.gemm_ex(op_a, op_b, m, n, k, 1.0, a_rm, orc.R_8I, ac, b_rm, orc.R_8I, bc, 0.0, c_rm,
                       orc.R_32I, n, compute_type=72, layout=orc.ROW_MAJOR) == orc.OK
    np.testing.assert_array_equal(c_rm.reshape(m, n), cm)
    # Column-major bytes of A and B read as the swapped call C^T = op(B)^T op(A)^T give C^T column-major.
    c_sw = np.zeros(m * n, np.int32)
    assert orc.gemm_ex(1 - op_b, 1 - op_a, n, m, k, 1.0, b, orc.R_8I, br, a, orc.R_8I, ar, 0.0, c_sw, orc.R_32I,
                       n, compute_type=72) == orc.OK
    np.testing.assert_array_equal(c_sw.astype(np.int64).reshape(m, n), cm)
