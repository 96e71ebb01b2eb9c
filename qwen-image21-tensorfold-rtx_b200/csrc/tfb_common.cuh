// Shared device/host helpers for libtfb (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tfb.h"

namespace tfb {

// ------------------------------------------------------------------------------------------------ host plumbing
tfb_status fail(tfb_status st, const char* fmt, ...);
tfb_status cuda_fail(cudaError_t e, const char* what);
#define TFB_CUDA(call)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return ::tfb::cuda_fail(e_, #call); \
  } while (0)

struct DeviceInfo {
  int device;
  int sm_count;
  int* err_word;  // device address of the kernel error word
};
// Per-device cache (filled once per device: SM count, arch check, error-word address).
tfb_status device_info(const DeviceInfo** out);

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// 2-D uint8 tensor map for TMA: inner dimension `inner_bytes` (contiguous), `rows` rows `row_stride` bytes apart,
// box `box_inner` x `box_rows`, 128-byte swizzle, zero fill out of bounds.
tfb_status make_tmap_u8(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t row_stride,
                        uint32_t box_inner, uint32_t box_rows);
// Same for 1- or 2-byte elements: `inner` elements per row, box `box_inner` elements, 128-byte swizzle or none.
tfb_status make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                        uint64_t row_stride, uint32_t box_inner, uint32_t box_rows, bool swizzle);

// NVFP4 row quantizer launch (quant.cu); shared by the fused MLP entry point.
// Launch with programmatic stream serialization (see pdl_trigger / pdl_wait). Launch errors are picked up by the
// cudaGetLastError() check that follows every launch site.
#define TFB_LAUNCH(kernel, grid, block, stream, ...) \
  (void)::tfb::launch_pdl(kernel, dim3(grid), dim3(block), 0, stream, __VA_ARGS__)
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

tfb_status quant_nvfp4(const void* x, int64_t M, int64_t K, int64_t ldx, float g, uint8_t* codes, uint8_t* sf,
                       int layout, cudaStream_t s);

constexpr long long kWaitLimitNs = 1000000000LL;  // 1 s: a pipeline wait that takes longer is a bug, not a load

// ------------------------------------------------------------------------------------------------ device helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// E4M3 byte (sign, 4 exponent bits bias 7, 3 mantissa bits) -> fp32, by assembling the fp32 bit pattern.
// Only finite codes are passed (NaN 0x7F never reaches it: scales are produced by a saturating conversion).
__device__ __forceinline__ float e4m3_to_f32(uint32_t c) {
  uint32_t e = (c >> 3) & 15u, m = c & 7u;
  float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20)) : static_cast<float>(m) * 0.001953125f;
  return (c & 0x80u) ? -v : v;
}

// fp32 -> E4M3, round to nearest even, finite values saturate to +-448.
__device__ __forceinline__ uint32_t f32_to_e4m3_sat(float v) {
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// 8 fp32 -> 8 E2M1 nibbles (round to nearest even, saturate at 6), element 0 in the lowest nibble.
__device__ __forceinline__ uint32_t e2m1x8(float v0, float v1, float v2, float v3, float v4, float v5, float v6,
                                           float v7) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(v0), "f"(v1), "f"(v2), "f"(v3), "f"(v4), "f"(v5), "f"(v6), "f"(v7));
  return out;
}

// NVFP4 encoder constants for one global scale g: inv6g = 1 / (6 g) in fp32 round-to-nearest.
struct Nvfp4Enc {
  float g;
  float inv6g;
};
__device__ __forceinline__ Nvfp4Enc nvfp4_enc(float g) { return {g, __frcp_rn(__fmul_rn(6.0f, g))}; }

// Scale byte of a 16-element block from its amax: e4m3_rne_satfinite(amax * inv6g).
__device__ __forceinline__ uint32_t nvfp4_scale(float amax, Nvfp4Enc e) { return f32_to_e4m3_sat(__fmul_rn(amax, e.inv6g)); }

// Multiplier that maps block values onto the E2M1 grid: 1 / (float(sf) * g), or 0 for an all-zero block.
__device__ __forceinline__ float nvfp4_inv(uint32_t sf, Nvfp4Enc e) {
  float d = __fmul_rn(e4m3_to_f32(sf), e.g);
  return d == 0.0f ? 0.0f : __frcp_rn(d);
}

// Codes of 8 values under multiplier inv (each value: e2m1(x * inv), RN multiply).
__device__ __forceinline__ uint32_t nvfp4_codes8(const float* x, float inv) {
  return e2m1x8(__fmul_rn(x[0], inv), __fmul_rn(x[1], inv), __fmul_rn(x[2], inv), __fmul_rn(x[3], inv),
                __fmul_rn(x[4], inv), __fmul_rn(x[5], inv), __fmul_rn(x[6], inv), __fmul_rn(x[7], inv));
}

// Byte offset of (row, scale column j) in the tiled scale layout with `chunks` = K/64 chunks per 128-row group.
__device__ __forceinline__ size_t sf_tiled_offset(int64_t row, int64_t j, int64_t chunks) {
  return (static_cast<size_t>(row >> 7) * chunks + (j >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (j & 3);
}

// Programmatic dependent launch. Every kernel of the library is launched with programmatic stream serialization,
// lets the next kernel launch as soon as all of its own CTAs are running (pdl_trigger), and waits for the previous
// kernel of the stream to complete -- with its memory visible -- before its first read of anything that kernel may
// have written (pdl_wait). What runs before pdl_wait (barrier set-up, TMEM allocation, tensor-map prefetch) overlaps
// the previous kernel's tail. Without a programmatic predecessor both are no-ops.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// silu(g) = g / (1 + e^-g), rounded to bf16 (kernels.py:80 rounds silu to bf16 before the product) CORRECTLY: the
// result is the round-to-nearest-even bf16 of the exact silu(g), so every implementation that rounds correctly --
// the float64 oracle included -- agrees bit for bit (the standalone SwiGLU kernel). Two parts:
//   * silu_fast_flag: branch-free fp32 with the hardware approximations, plus a flag. __expf(x) is within
//     2 + floor(1.173 |x|) ulp of e^x (CUDA's documented bound), the add within 1/2 ulp, __fdividef within 2 ulp,
//     so s is within 9 + 2.35 |g| ulp of the exact value: 19 ulp for |g| <= 4, 47 ulp for |g| <= 16. bf16
//     rounding depends only on the low 16 bits of the fp32 pattern; when those lie more than 20 (|g| <= 4) or 60
//     (|g| <= 16) ulp from the rounding midpoint 0x8000, the exact value rounds the same way. Otherwise, and for
//     every |g| > 16, the flag is set (about one value in 1600 for typical gate values);
//   * silu_f64_rto: the flagged values in fp64, rounded to fp32 by round-to-odd (truncate, set the last bit if
//     inexact). fp32 keeps 16 more significand bits than bf16, so the later round-to-nearest-even to bf16 equals a
//     single rounding of the fp64 value.
__device__ __forceinline__ float silu_fast_flag(float g, bool& flag) {
  const float s = __fdividef(g, 1.0f + __expf(-g));
  const float a = fabsf(g);
  const uint32_t w = a <= 4.0f ? 20u : 60u;
  flag = ((__float_as_uint(s) & 0xFFFFu) - (0x8000u - w)) <= 2u * w || a > 16.0f;
  return s;
}
static __device__ __noinline__ float silu_f64_rto(float g) {
  const double d = (double)g / (1.0 + exp(-(double)g));
  float f = __double2float_rz(d);
  if ((double)f != d) f = __uint_as_float(__float_as_uint(f) | 1u);
  return f;
}
// One value: an fp32 number whose bf16 rounding is the correctly rounded silu(g).
__device__ __forceinline__ float silu_for_bf16(float g) {
  bool flag;
  const float s = silu_fast_flag(g, flag);
  return flag ? silu_f64_rto(g) : s;
}

__device__ __forceinline__ void unpack_bf16x8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// RMSNorm over a 128-wide head + RoPE on interleaved pairs, shared by the standalone kernel (16 lanes x 8 values per
// head row) and the qkv GEMM epilogue (one thread per head row), so both produce the same bits. Every rounding is
// spelled out (no compiler contraction choices): the sum of squares of 8 values is a chain of fused multiply-adds
// from 0; the 16 such partial sums of a row are added in the xor-butterfly order of a 16-lane shuffle reduction.
__device__ __forceinline__ float sumsq8(const float* x) {
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss = __fmaf_rn(x[k], x[k], ss);
  return ss;
}
__device__ __forceinline__ float rms_rr(float ss, float eps) { return rsqrtf(__fadd_rn(__fmul_rn(ss, 0.0078125f), eps)); }
// 8 values (4 pairs) normalised by rr, scaled by w, rotated by (c, s): (c x0 - s x1, s x0 + c x1), to bf16.
__device__ __forceinline__ uint4 norm_rope8(const float* x, float rr, const float* wv, const float* cv,
                                            const float* sv) {
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float x0 = __fmul_rn(__fmul_rn(x[2 * p], rr), wv[2 * p]);
    const float x1 = __fmul_rn(__fmul_rn(x[2 * p + 1], rr), wv[2 * p + 1]);
    o[p] = pack_bf16x2(__fmaf_rn(cv[p], x0, -__fmul_rn(sv[p], x1)), __fmaf_rn(sv[p], x0, __fmul_rn(cv[p], x1)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}


}  // namespace tfb
