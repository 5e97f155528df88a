"""Helpers shared by the GPU parity tests: seeded inputs, device upload and the
comparison metrics the north star fixes (normwise relative error for floats,
bit equality for INT8 -> INT32)."""
import numpy as np

import gemm_sm100 as gs
import oracle as orc

TOL = {gs.R_32F: 1e-5, gs.R_16F: 2e-3, gs.R_16BF: 1e-2}
COMPUTE = {gs.R_16F: gs.COMPUTE_32F, gs.R_16BF: gs.COMPUTE_32F, gs.R_8I: gs.COMPUTE_32I, gs.R_32F: gs.COMPUTE_32F}
OUT_OF = {gs.R_16F: gs.R_32F, gs.R_16BF: gs.R_32F, gs.R_8I: gs.R_32I, gs.R_32F: gs.R_32F}
NP_OF = {gs.R_16F: np.uint16, gs.R_16BF: np.uint16, gs.R_8I: np.int8, gs.R_32F: np.float32, gs.R_32I: np.int32}


def to_dev(x: np.ndarray):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def to_host(t) -> np.ndarray:
    return t.cpu().numpy()


def make_input(rng, count: int, dt: int) -> np.ndarray:
    if dt in (gs.R_16F, gs.R_16BF):
        return orc.randn_lowp(rng, count, dt)
    if dt == gs.R_8I:
        return rng.integers(-128, 128, count, dtype=np.int64).astype(np.int8)
    return rng.uniform(-1.0, 1.0, count).astype(np.float32)


def make_c(rng, count: int, ct: int) -> np.ndarray:
    if ct == gs.R_32I:
        return rng.integers(-1000, 1000, count, dtype=np.int64).astype(np.int32)
    if ct == gs.R_16F:
        return rng.uniform(-1, 1, count).astype(np.float32).astype(np.float16).view(np.uint16)
    if ct == gs.R_16BF:
        return orc.bf16_round_array(rng.uniform(-1, 1, count).astype(np.float32))
    return rng.uniform(-1.0, 1.0, count).astype(np.float32)


def decode_out(c: np.ndarray, ct: int) -> np.ndarray:
    if ct == gs.R_16F:
        return c.view(np.float16).astype(np.float64)
    if ct == gs.R_16BF:
        return orc.bf16_bits_to_f32_array(c).astype(np.float64)
    return c.astype(np.float64)


def normwise_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    g = got.astype(np.float64)
    r = ref.astype(np.float64)
    den = np.linalg.norm(r)
    return float(np.linalg.norm(g - r) / (den if den > 0 else 1.0))


def matrix_mask(m: int, n: int, ld: int, batch: int, stride: int, total: int) -> np.ndarray:
    """Boolean mask of the elements of a batched column-major matrix that the GEMM writes."""
    mask = np.zeros(total, dtype=bool)
    rows = np.arange(m)
    for b in range(batch):
        for col in range(n):
            mask[b * stride + col * ld + rows] = True
    return mask


def assert_parity(got: np.ndarray, ref: np.ndarray, ct: int, tol_dt: int, mask=None, c_before=None):
    """INT32 outputs must match bit for bit; float outputs within the normwise tolerance.
    Elements outside `mask` (padding between columns / batches) must be untouched."""
    if mask is not None and c_before is not None:
        np.testing.assert_array_equal(got[~mask], c_before[~mask])
        got, ref = got[mask], ref[mask]
    if ct == gs.R_32I:
        np.testing.assert_array_equal(got, ref)
        return 0.0
    err = normwise_rel_err(decode_out(got, ct), decode_out(ref, ct))
    assert err <= TOL[tol_dt], f"normwise relative error {err:.3e} > {TOL[tol_dt]:.1e}"
    return err
