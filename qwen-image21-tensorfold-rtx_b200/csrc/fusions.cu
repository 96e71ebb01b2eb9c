// Fused elementwise kernels of a DiT block: AdaLN modulate (+ NVFP4 quantize), RMSNorm + RoPE, SwiGLU.
// All are HBM-bound: 16-byte coalesced loads/stores, statistics in fp32 registers, one pass over the input.
#include "tfb_common.cuh"

namespace tfb {
namespace {

// ------------------------------------------------------------------------------------------------------- AdaLN
// WPR warps share a row (D = 256 * NCH): warp w of the row, lane l holds columns (i * WPR + w) * 256 + l * 8 .. +7
// for its CPT = NCH / WPR chunks i, so every warp load / store covers 512 contiguous bytes and a 16-element
// quantization block is the lane pair (2q, 2q+1). Row statistics: warp shuffles, then the WPR partial sums through
// shared memory. Splitting the row keeps a thread's values in few registers (24 floats at D = 3072): with one warp
// per row (96 floats per lane) only 16 warps fitted on an SM and the kernel ran at a third of HBM bandwidth.
constexpr int kAdaThreads = 256;

template <int NCH>
struct AdaSplit {
  static constexpr int WPR = NCH % 4 == 0 ? 4 : NCH % 3 == 0 ? 3 : NCH % 2 == 0 ? 2 : 1;   // warps per row
  static constexpr int CPT = NCH / WPR;                                                    // chunks per thread
  static constexpr int RPB = (kAdaThreads / 32) / WPR;                                     // rows per block
};

template <int NCH>
__global__ void __launch_bounds__(kAdaThreads) adaln_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                            int64_t rows_total, int64_t rows_per_b,
                                                            const float* __restrict__ scale,
                                                            const float* __restrict__ shift, float eps,
                                                            __nv_bfloat16* __restrict__ out, float qg,
                                                            uint8_t* __restrict__ codes, uint8_t* __restrict__ sf) {
  pdl_trigger();
  pdl_wait();
  using S = AdaSplit<NCH>;
  constexpr int D = NCH * 256, WPR = S::WPR, CPT = S::CPT, RPB = S::RPB;
  __shared__ float red[2][RPB][WPR];
  // NVFP4 multiplier per scale byte, 1 / (e4m3(sf) * g) (0 for sf = 0): scales of non-negative amax are 0..0x7E,
  // so 128 entries cover them; one exact reciprocal per entry instead of one per 8 values
  __shared__ float inv_tab[128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rib = warp / WPR, wr = warp % WPR;             // row inside the block, warp inside the row
  if (codes && threadIdx.x < 128) inv_tab[threadIdx.x] = nvfp4_inv(threadIdx.x, nvfp4_enc(qg));
  const bool warp_live = warp < RPB * WPR;                 // WPR = 3 leaves spare warps in the block
  const int64_t row = blockIdx.x * (int64_t)RPB + rib;
  const bool live = warp_live && row < rows;
  float v[CPT][8];
  float sum = 0.0f;
  if (live) {
    const __nv_bfloat16* xr = x + row * D;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(xr + (i * WPR + wr) * 256 + lane * 8)), v[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) sum += v[i][k];
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (warp_live && lane == 0) red[0][rib][wr] = sum;
  __syncthreads();
  float mean = 0.0f;
  if (warp_live) {
#pragma unroll
    for (int w = 0; w < WPR; ++w) mean += red[0][rib][w];
    mean /= D;
  }
  float var = 0.0f;
  if (live) {
#pragma unroll
    for (int i = 0; i < CPT; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[i][k] -= mean;
        var += v[i][k] * v[i][k];
      }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  if (warp_live && lane == 0) red[1][rib][wr] = var;
  __syncthreads();
  if (!warp_live || row >= rows_total) return;
  if (!live) {  // padding rows of the tiled scale layout: zero scales
    if (sf && (lane & 7) == 0)
#pragma unroll
      for (int i = 0; i < CPT; ++i)
        *reinterpret_cast<uint32_t*>(sf + sf_tiled_offset(row, (i * WPR + wr) * 16 + (lane >> 1), D >> 6)) = 0u;
    return;
  }
  float vs = 0.0f;
#pragma unroll
  for (int w = 0; w < WPR; ++w) vs += red[1][rib][w];
  const float rstd = rsqrtf(vs / D + eps);
  const int64_t b = row / rows_per_b;
  const float* sc = scale + b * D;
  const float* sh = shift ? shift + b * D : nullptr;
  const Nvfp4Enc enc = nvfp4_enc(qg);
  // this row's part of the tiled scale offset; chunk ch's word for lanes 8t adds (4 ch + t) * 512
  const size_t sf_row = sf ? (static_cast<size_t>(row >> 7) * (D >> 6)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4
                           : 0;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int ch = i * WPR + wr;
    const int c0 = ch * 256 + lane * 8;
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(sc + c0));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(sc + c0 + 4));
    float s8[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float y[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] = v[i][k] * rstd * (1.0f + s8[k]);
    if (sh) {
      const float4 h0 = __ldg(reinterpret_cast<const float4*>(sh + c0));
      const float4 h1 = __ldg(reinterpret_cast<const float4*>(sh + c0 + 4));
      const float h[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] += h[k];
    }
    uint4 packed = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                              pack_bf16x2(y[6], y[7]));
    if (out) *reinterpret_cast<uint4*>(out + row * D + c0) = packed;
    if (codes) {
      float q[8];
      unpack_bf16x8(packed, q);  // quantize the bf16-rounded result
      float amax = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(q[k]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      const uint32_t sfb = nvfp4_scale(amax, enc);
      *reinterpret_cast<uint32_t*>(codes + row * (D >> 1) + (c0 >> 1)) = nvfp4_codes8(q, inv_tab[sfb]);
      // lanes 8t, 8t+2, 8t+4, 8t+6 hold blocks 4t..4t+3 of this chunk: one 32-bit word of the tiled layout
      const uint32_t b1 = __shfl_down_sync(0xffffffffu, sfb, 2);
      const uint32_t b2 = __shfl_down_sync(0xffffffffu, sfb, 4);
      const uint32_t b3 = __shfl_down_sync(0xffffffffu, sfb, 6);
      if ((lane & 7) == 0)
        *reinterpret_cast<uint32_t*>(sf + sf_row + (size_t)(ch * 4 + (lane >> 3)) * 512) =
            sfb | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
  }
}
template <int NCH>
void launch_adaln(const void* x, int64_t rows, int64_t rows_total, int64_t rows_per_b, const float* scale,
                  const float* shift, float eps, void* out, float qg, uint8_t* codes, uint8_t* sf, cudaStream_t s) {
  constexpr int RPB = AdaSplit<NCH>::RPB;
  const int64_t grid = (rows_total + RPB - 1) / RPB;
  TFB_LAUNCH(adaln_kernel<NCH>, grid, kAdaThreads, s, static_cast<const __nv_bfloat16*>(x), rows, rows_total, rows_per_b,
                                                 scale, shift, eps, static_cast<__nv_bfloat16*>(out), qg, codes, sf);
}

// --------------------------------------------------------------------------------------------- RMSNorm + RoPE
// Half a warp per (b, n, h) with D = 128: lane holds 8 elements (four interleaved pairs), 16-byte accesses.
// One lane's 8 elements of a head: RMSNorm over the half-warp's 128 (weight w), then RoPE on the pairs.
__device__ __forceinline__ uint4 rms_rope_piece(uint4 raw, const float* __restrict__ w, int l, const float* cv,
                                                const float* sv, float eps) {
  float x[8];
  unpack_bf16x8(raw, x);
  float ss = sumsq8(x);
#pragma unroll
  for (int o = 8; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float rr = rms_rr(ss, eps);
  const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + l * 8));
  const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + l * 8 + 4));
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  return norm_rope8(x, rr, wv, cv, sv);
}

__global__ void __launch_bounds__(256) rms_rope_kernel(const __nv_bfloat16* __restrict__ src, int64_t units, int64_t N,
                                                       int64_t H, int64_t src_sb, int64_t src_sn, int64_t src_off,
                                                       const float* __restrict__ w, const float* __restrict__ cosp,
                                                       const float* __restrict__ sinp, float eps,
                                                       __nv_bfloat16* __restrict__ dst, int64_t dst_sb,
                                                       int64_t dst_sn) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128;
  const int64_t unit = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;
  const int l = threadIdx.x & 15;
  const bool live = unit < units;
  const int64_t uu = live ? unit : 0;
  const int64_t h = uu % H, bn = uu / H, n = bn % N, b = bn / N;
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src + b * src_sb + n * src_sn + src_off + h * D + l * 8));
  const float4 c = __ldg(reinterpret_cast<const float4*>(cosp + n * (D / 2) + l * 4));
  const float4 s = __ldg(reinterpret_cast<const float4*>(sinp + n * (D / 2) + l * 4));
  const float cv[4] = {c.x, c.y, c.z, c.w}, sv[4] = {s.x, s.y, s.z, s.w};
  const uint4 o = rms_rope_piece(raw, w, l, cv, sv, eps);
  if (live) *reinterpret_cast<uint4*>(dst + b * dst_sb + n * dst_sn + h * D + l * 8) = o;
}

// q, k and v of a fused qkv row [B, N, 3, H, D] in one pass: q and k normalised + rotated (one cos / sin read for
// both), v copied; each goes to its own strided destination (k and v typically behind a kept prefix).
__global__ void __launch_bounds__(256) rms_rope_qkv_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t units, int64_t N, int64_t H, int64_t src_sb, int64_t src_sn,
    const float* __restrict__ wq, const float* __restrict__ wk, const float* __restrict__ cosp,
    const float* __restrict__ sinp, float eps, __nv_bfloat16* __restrict__ qd, int64_t q_sb, int64_t q_sn,
    __nv_bfloat16* __restrict__ kd, int64_t k_sb, int64_t k_sn, __nv_bfloat16* __restrict__ vd, int64_t v_sb,
    int64_t v_sn) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128;
  const int64_t unit = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;
  const int l = threadIdx.x & 15;
  const bool live = unit < units;
  const int64_t uu = live ? unit : 0;
  const int64_t h = uu % H, bn = uu / H, n = bn % N, b = bn / N;
  const __nv_bfloat16* sp = src + b * src_sb + n * src_sn + h * D + l * 8;
  const uint4 rq = __ldg(reinterpret_cast<const uint4*>(sp));
  const uint4 rk = __ldg(reinterpret_cast<const uint4*>(sp + H * D));
  const uint4 rv = __ldg(reinterpret_cast<const uint4*>(sp + 2 * H * D));
  const float4 c = __ldg(reinterpret_cast<const float4*>(cosp + n * (D / 2) + l * 4));
  const float4 s = __ldg(reinterpret_cast<const float4*>(sinp + n * (D / 2) + l * 4));
  const float cv[4] = {c.x, c.y, c.z, c.w}, sv[4] = {s.x, s.y, s.z, s.w};
  const uint4 oq = rms_rope_piece(rq, wq, l, cv, sv, eps);
  const uint4 ok = rms_rope_piece(rk, wk, l, cv, sv, eps);
  if (live) {
    const int64_t col = h * D + l * 8;
    *reinterpret_cast<uint4*>(qd + b * q_sb + n * q_sn + col) = oq;
    *reinterpret_cast<uint4*>(kd + b * k_sb + n * k_sn + col) = ok;
    *reinterpret_cast<uint4*>(vd + b * v_sb + n * v_sn + col) = rv;
  }
}

// ------------------------------------------------------------------------------------------------------ SwiGLU
// bf16(bf16(silu(g)) * u), 8 columns per thread.
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gu, int64_t M, int64_t F,
                                                     __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t per_row = F >> 3;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= M * per_row) return;
  const int64_t m = t / per_row, c = (t - m * per_row) * 8;
  float g[8], u[8];
  unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(gu + m * 2 * F + c)), g);
  unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(gu + m * 2 * F + F + c)), u);
  float y[8];
#pragma unroll
  for (int k = 0; k < 8; k += 2) {   // silu rounded to bf16 two at a time (one paired conversion)
    const uint32_t sp = pack_bf16x2(__fdiv_rn(g[k], 1.0f + expf(-g[k])), __fdiv_rn(g[k + 1], 1.0f + expf(-g[k + 1])));
    y[k] = __uint_as_float(sp << 16) * u[k];
    y[k + 1] = __uint_as_float(sp & 0xFFFF0000u) * u[k + 1];
  }
  *reinterpret_cast<uint4*>(out + m * F + c) =
      make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
}

}  // namespace
}  // namespace tfb

extern "C" {

tfb_status tfb_adaln(const void* x, int64_t B, int64_t N, int64_t D, const float* scale, const float* shift, float eps,
                     void* out, float q_global, uint8_t* codes, uint8_t* sf, void* stream) {
  using namespace tfb;
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (B <= 0 || N < 0 || D <= 0 || D % 256 || D > 8192)
    return fail(TFB_BAD_SHAPE, "adaln: need D %% 256 == 0 and D <= 8192 (D=%lld)", (long long)D);
  if (!out && !codes) return fail(TFB_BAD_ARG, "adaln: no output requested");
  if ((codes == nullptr) != (sf == nullptr)) return fail(TFB_BAD_ARG, "adaln: codes and scales go together");
  if (codes && (!(q_global > 0.0f) || !isfinite(q_global)))
    return fail(TFB_BAD_ARG, "adaln: quantization global must be positive and finite");
  if (!aligned(x, 16) || (out && !aligned(out, 16)) || !aligned(scale, 16) || (shift && !aligned(shift, 16)) ||
      (codes && (!aligned(codes, 4) || !aligned(sf, 4))))
    return fail(TFB_BAD_ALIGN, "adaln: x/out/scale/shift must be 16-byte aligned");
  const int64_t rows = B * N;
  const int64_t rows_total = codes ? (rows + 127) / 128 * 128 : rows;
  if (rows_total == 0) return TFB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (D / 256) {
#define TFB_ADA(n) \
  case n: launch_adaln<n>(x, rows, rows_total, N, scale, shift, eps, out, q_global, codes, sf, s); break;
    TFB_ADA(1) TFB_ADA(2) TFB_ADA(3) TFB_ADA(4) TFB_ADA(6) TFB_ADA(8) TFB_ADA(12) TFB_ADA(16) TFB_ADA(24) TFB_ADA(32)
#undef TFB_ADA
    default:
      return fail(TFB_BAD_SHAPE, "adaln: D=%lld not instantiated (256 x {1,2,3,4,6,8,12,16,24,32})", (long long)D);
  }
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

tfb_status tfb_rms_rope(const void* src, int64_t B, int64_t N, int64_t H, int64_t D, int64_t src_sb, int64_t src_sn,
                        int64_t src_off, const float* w, const float* cos, const float* sin, float eps, void* dst,
                        int64_t dst_sb, int64_t dst_sn, void* stream) {
  using namespace tfb;
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (D != 128 || B < 0 || N < 0 || H <= 0) return fail(TFB_BAD_SHAPE, "rms_rope: head dim must be 128");
  if (!aligned(src, 16) || !aligned(dst, 16) || src_sb % 8 || src_sn % 8 || src_off % 8 || dst_sb % 8 ||
      dst_sn % 8 || !aligned(w, 16) || !aligned(cos, 16) || !aligned(sin, 16))
    return fail(TFB_BAD_ALIGN, "rms_rope: pointers and element strides must be 16-byte aligned");
  const int64_t units = B * N * H;
  if (units == 0) return TFB_OK;
  const int64_t threads = units * 16;
  TFB_LAUNCH(rms_rope_kernel, (threads + 255) / 256, 256, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(src), units, N, H, src_sb, src_sn, src_off, w, cos, sin, eps,
      static_cast<__nv_bfloat16*>(dst), dst_sb, dst_sn);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

tfb_status tfb_rms_rope_qkv(const void* src, int64_t B, int64_t N, int64_t H, int64_t D, int64_t src_sb,
                            int64_t src_sn, const float* wq, const float* wk, const float* cos, const float* sin,
                            float eps, void* q, int64_t q_sb, int64_t q_sn, void* k, int64_t k_sb, int64_t k_sn,
                            void* v, int64_t v_sb, int64_t v_sn, void* stream) {
  using namespace tfb;
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (D != 128 || B < 0 || N < 0 || H <= 0) return fail(TFB_BAD_SHAPE, "rms_rope_qkv: head dim must be 128");
  if (!aligned(src, 16) || !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || src_sb % 8 || src_sn % 8 ||
      q_sb % 8 || q_sn % 8 || k_sb % 8 || k_sn % 8 || v_sb % 8 || v_sn % 8 || !aligned(wq, 16) || !aligned(wk, 16) ||
      !aligned(cos, 16) || !aligned(sin, 16))
    return fail(TFB_BAD_ALIGN, "rms_rope_qkv: pointers and element strides must be 16-byte aligned");
  const int64_t units = B * N * H;
  if (units == 0) return TFB_OK;
  const int64_t threads = units * 16;
  TFB_LAUNCH(rms_rope_qkv_kernel, (threads + 255) / 256, 256, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(src), units, N, H, src_sb, src_sn, wq, wk, cos, sin, eps,
      static_cast<__nv_bfloat16*>(q), q_sb, q_sn, static_cast<__nv_bfloat16*>(k), k_sb, k_sn,
      static_cast<__nv_bfloat16*>(v), v_sb, v_sn);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

tfb_status tfb_swiglu(const void* gu, int64_t M, int64_t F, void* out, void* stream) {
  using namespace tfb;
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (M < 0 || F <= 0 || F % 8) return fail(TFB_BAD_SHAPE, "swiglu: F must be a positive multiple of 8");
  if (!aligned(gu, 16) || !aligned(out, 16)) return fail(TFB_BAD_ALIGN, "swiglu: buffers must be 16-byte aligned");
  const int64_t threads = M * (F / 8);
  if (threads == 0) return TFB_OK;
  TFB_LAUNCH(swiglu_kernel, (threads + 255) / 256, 256, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(gu), M, F, static_cast<__nv_bfloat16*>(out));
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

}  // extern "C"
