// gs_epilogue.cuh -- alpha/beta epilogue shared by every kernel.
//
// Output rounding follows slang-gemm's writeScalar (src/gemm.zig:837-896):
//  - r_32i: the value alpha*acc + beta*old is formed in f64 (each product and
//    the sum rounded separately, no FMA), rounded half away from zero and
//    clamped to int32 (clampInt, src/gemm.zig:1002-1010). With alpha == 1 and
//    beta == 0 the exact s32 accumulator is stored as is.
//  - r_16bf: rounded with the reference's bit formula raw + 0x7fff + lsb
//    (f32ToBf16Bits, src/gemm.zig:924-928).
//  - r_16f: IEEE round-to-nearest-even from f32.
// beta == 0 never reads C (cuBLAS semantics; identical to the reference for
// finite C).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gs_internal.h"

namespace gs {

__device__ __forceinline__ uint16_t bf16_bits_ref_round(float v) {
    const uint32_t raw = __float_as_uint(v);
    const uint32_t rounded = raw + 0x7fffu + ((raw >> 16) & 1u);
    return static_cast<uint16_t>(rounded >> 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// Store one element of a float-accumulated result.
template <int OUT>
__device__ __forceinline__ void store_facc(void *C, size_t i, float acc, const Epilogue &ep) {
    if constexpr (OUT == OUT_F32) {
        float *c = static_cast<float *>(C);
        float v = ep.identity ? acc : ep.alpha_f * acc;
        if (!ep.beta_zero) v = __fadd_rn(v, __fmul_rn(ep.beta_f, c[i]));
        c[i] = v;
    } else if constexpr (OUT == OUT_F16) {
        __half *c = static_cast<__half *>(C);
        float v = ep.identity ? acc : ep.alpha_f * acc;
        if (!ep.beta_zero) v = __fadd_rn(v, __fmul_rn(ep.beta_f, __half2float(c[i])));
        c[i] = __float2half_rn(v);
    } else if constexpr (OUT == OUT_BF16) {
        uint16_t *c = static_cast<uint16_t *>(C);
        float v = ep.identity ? acc : ep.alpha_f * acc;
        if (!ep.beta_zero) v = __fadd_rn(v, __fmul_rn(ep.beta_f, bf16_bits_to_f32(c[i])));
        c[i] = bf16_bits_ref_round(v);
    }
}

// Store one element of an s32-accumulated result into an int32 C.
__device__ __forceinline__ void store_iacc(void *C, size_t i, int32_t acc, const Epilogue &ep) {
    int32_t *c = static_cast<int32_t *>(C);
    if (ep.identity) {
        c[i] = acc;
        return;
    }
    double v = __dmul_rn(static_cast<double>(ep.alpha_i), static_cast<double>(acc));
    if (!ep.beta_zero) v = __dadd_rn(v, __dmul_rn(static_cast<double>(ep.beta_i), static_cast<double>(c[i])));
    v = round(v);
    v = fmin(2147483647.0, fmax(-2147483648.0, v));
    c[i] = static_cast<int32_t>(v);
}

}  // namespace gs
