// Activation quantizers and amax reductions (HBM-bound; 16-byte vector loads, one 16-element block per thread).
#include "tfb_common.cuh"

namespace tfb {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------------------------------------- amax reduction
__global__ void __launch_bounds__(kThreads) absmax_kernel(const uint4* __restrict__ x, int64_t nvec,
                                                         const __nv_bfloat16* __restrict__ tail, int ntail,
                                                         unsigned int* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  float m = 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * kThreads) {
    float f[8];
    unpack_bf16x8(__ldg(x + i), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(f[k]));
  }
  if (blockIdx.x == 0 && threadIdx.x < ntail) m = fmaxf(m, fabsf(__bfloat162float(tail[threadIdx.x])));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red[w]);
    atomicMax(out, __float_as_uint(m));  // non-negative floats order like their bit patterns
  }
}

// a = max(amax / 448, 1e-12) (tfimage/linear.py:86)
__global__ void fp8_scale_finalize(float* a) {
  pdl_trigger();
  pdl_wait();
  *a = fmaxf(__fdiv_rn(*a, 448.0f), 1e-12f);
}

tfb_status launch_absmax(const void* x, int64_t n, float* out, cudaStream_t s) {
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (n < 0) return fail(TFB_BAD_SHAPE, "absmax: n < 0");
  if (!aligned(x, 16) || !aligned(out, 4)) return fail(TFB_BAD_ALIGN, "absmax: x must be 16-byte aligned");
  TFB_CUDA(cudaMemsetAsync(out, 0, sizeof(float), s));
  int64_t nvec = n / 8;
  int ntail = static_cast<int>(n - nvec * 8);
  int64_t want = (nvec + kThreads - 1) / kThreads;
  int grid = static_cast<int>(want < (int64_t)di->sm_count * 8 ? (want > 0 ? want : 1) : (int64_t)di->sm_count * 8);
  TFB_LAUNCH(absmax_kernel, grid, kThreads, s, static_cast<const uint4*>(x), nvec,
                                          static_cast<const __nv_bfloat16*>(x) + nvec * 8, ntail,
                                          reinterpret_cast<unsigned int*>(out));
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

// ------------------------------------------------------------------------------------------ NVFP4 row quantizer
// One thread per 16-element block: two 16-byte loads, 8 bytes of codes, one scale byte. In the tiled scale layout
// four consecutive blocks of a row share one 32-bit word, written by the first of the four lanes.
template <bool TILED>
__global__ void __launch_bounds__(kThreads) quant_nvfp4_kernel(const __nv_bfloat16* __restrict__ x, int64_t M,
                                                              int64_t rows_total, int64_t K, int64_t ldx, float g,
                                                              uint8_t* __restrict__ codes, uint8_t* __restrict__ sf) {
  pdl_trigger();
  pdl_wait();
  const int64_t nb = K >> 4;
  const int64_t blk = blockIdx.x * (int64_t)kThreads + threadIdx.x;
  const int64_t row = blk / nb, j = blk - row * nb;
  const bool live = row < rows_total;
  uint32_t s = 0;
  if (live && row < M) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx + j * 16);
    float f[16];
    unpack_bf16x8(__ldg(src), f);
    unpack_bf16x8(__ldg(src + 1), f + 8);
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(f[k]));
    const Nvfp4Enc e = nvfp4_enc(g);
    s = nvfp4_scale(amax, e);
    const float inv = nvfp4_inv(s, e);
    uint2 c;
    c.x = nvfp4_codes8(f, inv);
    c.y = nvfp4_codes8(f + 8, inv);
    *reinterpret_cast<uint2*>(codes + row * (K >> 1) + j * 8) = c;
  }
  if (TILED) {
    const int lane = threadIdx.x & 31;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, s, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, s, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, s, 3);
    if (live && (j & 3) == 0) {
      (void)lane;
      *reinterpret_cast<uint32_t*>(sf + sf_tiled_offset(row, j, K >> 6)) = s | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
  } else if (live) {
    sf[row * nb + j] = static_cast<uint8_t>(s);
  }
}

// ------------------------------------------------------------------------------------------ FP8 row quantizer
// q = e4m3(clamp(x / a, -448, 448)) with an IEEE division (tfimage/linear.py:95); 16 elements per thread.
__global__ void __launch_bounds__(kThreads) quant_fp8_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K,
                                                            int64_t ldx, const float* __restrict__ a_dev,
                                                            uint8_t* __restrict__ q) {
  pdl_trigger();
  pdl_wait();
  const int64_t nb = K >> 4;
  const int64_t blk = blockIdx.x * (int64_t)kThreads + threadIdx.x;
  const int64_t row = blk / nb, j = blk - row * nb;
  if (row >= M) return;
  const float a = __ldg(a_dev);
  const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx + j * 16);
  float f[16];
  unpack_bf16x8(__ldg(src), f);
  unpack_bf16x8(__ldg(src + 1), f + 8);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t b = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v = fminf(fmaxf(__fdiv_rn(f[4 * i + k], a), -448.0f), 448.0f);
      b |= f32_to_e4m3_sat(v) << (8 * k);
    }
    w[i] = b;
  }
  *reinterpret_cast<uint4*>(q + row * K + j * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace

tfb_status quant_nvfp4(const void* x, int64_t M, int64_t K, int64_t ldx, float g, uint8_t* codes, uint8_t* sf,
                       int layout, cudaStream_t s) {
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (M < 0 || K <= 0 || ldx < K) return fail(TFB_BAD_SHAPE, "quant_nvfp4: bad shape M=%lld K=%lld ldx=%lld",
                                               (long long)M, (long long)K, (long long)ldx);
  if (layout != TFB_SF_ROWS && layout != TFB_SF_TILED) return fail(TFB_BAD_ARG, "quant_nvfp4: unknown scale layout");
  if (K % (layout == TFB_SF_TILED ? 64 : 16)) return fail(TFB_BAD_SHAPE, "quant_nvfp4: K=%lld not a multiple of %d",
                                                          (long long)K, layout == TFB_SF_TILED ? 64 : 16);
  if (!aligned(x, 16) || ldx % 8 || !aligned(codes, 8) || !aligned(sf, 4))
    return fail(TFB_BAD_ALIGN, "quant_nvfp4: x/ldx must be 16-byte aligned, codes 8-byte, scales 4-byte");
  if (!(g > 0.0f) || !isfinite(g)) return fail(TFB_BAD_ARG, "quant_nvfp4: global scale must be positive and finite");
  const int64_t rows_total = layout == TFB_SF_TILED ? (M + 127) / 128 * 128 : M;
  const int64_t blocks = rows_total * (K / 16);
  if (blocks == 0) return TFB_OK;
  const int64_t grid = (blocks + kThreads - 1) / kThreads;
  if (layout == TFB_SF_TILED)
    TFB_LAUNCH(quant_nvfp4_kernel<true>, grid, kThreads, s, static_cast<const __nv_bfloat16*>(x), M, rows_total, K, ldx,
                                                       g, codes, sf);
  else
    TFB_LAUNCH(quant_nvfp4_kernel<false>, grid, kThreads, s, static_cast<const __nv_bfloat16*>(x), M, rows_total, K, ldx,
                                                        g, codes, sf);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

}  // namespace tfb

extern "C" {

tfb_status tfb_absmax_bf16(const void* x, int64_t n, float* amax_dev, void* stream) {
  return tfb::launch_absmax(x, n, amax_dev, static_cast<cudaStream_t>(stream));
}

tfb_status tfb_fp8_act_scale(const void* x, int64_t n, float* a_dev, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  tfb_status st = tfb::launch_absmax(x, n, a_dev, s);
  if (st != TFB_OK) return st;
  TFB_LAUNCH(tfb::fp8_scale_finalize, 1, 1, s, a_dev);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

tfb_status tfb_quant_nvfp4(const void* x, int64_t M, int64_t K, int64_t ldx, float global, uint8_t* codes,
                           uint8_t* sf, int sf_layout, void* stream) {
  return tfb::quant_nvfp4(x, M, K, ldx, global, codes, sf, sf_layout, static_cast<cudaStream_t>(stream));
}

tfb_status tfb_quant_fp8(const void* x, int64_t M, int64_t K, int64_t ldx, const float* a_dev, uint8_t* q,
                         void* stream) {
  const tfb::DeviceInfo* di;
  tfb_status st = tfb::device_info(&di);
  if (st != TFB_OK) return st;
  if (M < 0 || K <= 0 || K % 16 || ldx < K)
    return tfb::fail(TFB_BAD_SHAPE, "quant_fp8: K must be a positive multiple of 16 and ldx >= K");
  if (!tfb::aligned(x, 16) || ldx % 8 || !tfb::aligned(q, 16) || !tfb::aligned(a_dev, 4))
    return tfb::fail(TFB_BAD_ALIGN, "quant_fp8: x, ldx and q must be 16-byte aligned");
  const int64_t blocks = M * (K / 16);
  if (blocks == 0) return TFB_OK;
  TFB_LAUNCH(tfb::quant_fp8_kernel, (blocks + 255) / 256, 256, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(x), M, K, ldx, a_dev, q);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

}  // extern "C"
