// Fused elementwise kernels of a DiT block: AdaLN modulate (+ NVFP4 quantize), RMSNorm + RoPE, SwiGLU.
// All are HBM-bound: 16-byte coalesced loads/stores, statistics in fp32 registers, one pass over the input.
#include <algorithm>
#include <atomic>

#include "tfb_common.cuh"

namespace tfb {
namespace {

// ------------------------------------------------------------------------------------------------------- AdaLN
// WPR warps share a row (D = 256 * NCH): warp w of the row, lane l holds columns (i * WPR + w) * 256 + l * 8 .. +7
// for its CPT = NCH / WPR chunks i, so every warp load / store covers 512 contiguous bytes and a 16-element
// quantization block is the lane pair (2q, 2q+1). Row statistics: warp shuffles, then the WPR partial sums through
// shared memory (two passes over the register-held row: mean, then the centred sum of squares).
//
// A block (RPB row slots of WPR warps) walks a contiguous range of rows of ONE batch element, so the modulation of
// its columns -- (1 + scale) and shift -- is staged once per block in shared memory ([chunk][half][lane][4] floats:
// each 16-byte read of a warp is contiguous, no bank conflicts) instead of being re-read and re-added per element;
// the next row's x is loaded into registers before the current row is computed. The arithmetic runs on packed fp32
// pairs (sm_100 FFMA2 / FADD2 / FMUL2) and the NVFP4 block maximum on packed bf16 pairs. The previous form (one row
// per warp group, per-element scale / shift loads, scalar math) was issue-bound at ~27 instructions per element.
constexpr int kAdaThreads = 256;

template <int NCH>
struct AdaSplit {
  static constexpr int WPR = NCH % 4 == 0 ? 4 : NCH % 3 == 0 ? 3 : NCH % 2 == 0 ? 2 : 1;   // warps per row
  static constexpr int CPT = NCH / WPR;                                                    // chunks per thread
  static constexpr int RPB = (kAdaThreads / 32) / WPR;                                     // rows per block
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

template <int NCH>
__global__ void __launch_bounds__(kAdaThreads) adaln_kernel(const __nv_bfloat16* __restrict__ x, int64_t B,
                                                            int64_t N, int64_t rows_total, int chunks_per_b,
                                                            const float* __restrict__ scale,
                                                            const float* __restrict__ shift, float eps,
                                                            __nv_bfloat16* __restrict__ out, float qg,
                                                            uint8_t* __restrict__ codes, uint8_t* __restrict__ sf) {
  using S = AdaSplit<NCH>;
  constexpr int D = NCH * 256, WPR = S::WPR, CPT = S::CPT, RPB = S::RPB;
  extern __shared__ float4 ada_tab[];                      // [2][NCH][2][32] float4: (1 + scale), then shift
  __shared__ float red[2][RPB][WPR];
  // NVFP4 multiplier per scale byte, 1 / (e4m3(sf) * g) (0 for sf = 0): scales of non-negative amax are 0..0x7E,
  // so 128 entries cover them; one exact reciprocal per entry instead of one per 8 values
  __shared__ float inv_tab[128];
  pdl_trigger();
  pdl_wait();                                              // before any access to global memory
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rib = warp / WPR, wr = warp % WPR;             // row slot inside the block, warp inside the row
  const bool warp_live = warp < RPB * WPR;                 // WPR = 3 leaves spare warps in the block
  if (codes && threadIdx.x < 128) inv_tab[threadIdx.x] = nvfp4_inv(threadIdx.x, nvfp4_enc(qg));
  // this block's rows: chunk blockIdx.x of batch element blockIdx.y (y == B: the padding rows of the tiled scales)
  const int64_t b = blockIdx.y;
  const int64_t first = b < B ? b * N : B * N, count = b < B ? N : rows_total - B * N;
  const int64_t per = (count + chunks_per_b - 1) / chunks_per_b;
  const int64_t r0 = first + (int64_t)blockIdx.x * per, r1 = min(first + count, r0 + per);
  const size_t sf_chunks = D >> 6;
  if (b == B) {                                            // padding rows: zero scale words, nothing else
    if (!warp_live) return;
    for (int64_t row = r0 + rib; row < r1; row += RPB)
      if ((lane & 7) == 0)
#pragma unroll
        for (int i = 0; i < CPT; ++i)
          *reinterpret_cast<uint32_t*>(sf + sf_tiled_offset(row, (i * WPR + wr) * 16 + (lane >> 1), sf_chunks)) = 0u;
    return;
  }
  const Nvfp4Enc enc = nvfp4_enc(qg);
  uint4 nxt[CPT];
  auto load_row = [&](int64_t row) {
#pragma unroll
    for (int i = 0; i < CPT; ++i)
      nxt[i] = row < r1 ? __ldg(reinterpret_cast<const uint4*>(x + row * D + (i * WPR + wr) * 256 + lane * 8))
                        : make_uint4(0, 0, 0, 0);
  };
  int64_t row = r0 + rib;
  if (warp_live) load_row(row);                            // the first row's loads go out before the table's
  {
    // 4 consecutive columns c..c+3 are one float4 of the [chunk][half][lane][4] layout; every load of the fill is
    // in flight before the first store
    constexpr int kV = (D / 4 + kAdaThreads - 1) / kAdaThreads;   // float4 per thread (the last may be past D)
    float4 sv[kV], hv[kV];
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const int c = (k * kAdaThreads + threadIdx.x) * 4;
      const bool in = c < D;
      sv[k] = in ? __ldg(reinterpret_cast<const float4*>(scale + b * D + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
      hv[k] = in && shift ? __ldg(reinterpret_cast<const float4*>(shift + b * D + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const int c = (k * kAdaThreads + threadIdx.x) * 4, ch = c >> 8, r = c & 255;
      if (c >= D) continue;
      const int q = ch * 64 + ((r >> 2) & 1) * 32 + (r >> 3);
      ada_tab[q] = make_float4(1.0f + sv[k].x, 1.0f + sv[k].y, 1.0f + sv[k].z, 1.0f + sv[k].w);
      ada_tab[NCH * 64 + q] = hv[k];
    }
  }
  __syncthreads();                                         // the modulation table and inv_tab are in place
  const int iters = (int)((r1 - r0 + RPB - 1) / RPB);
  for (int it = 0; it < iters; ++it, row += RPB) {
    const bool live = warp_live && row < r1;
    float2 v[CPT][4];
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      v[i][0] = bf16x2_to_f2(nxt[i].x);
      v[i][1] = bf16x2_to_f2(nxt[i].y);
      v[i][2] = bf16x2_to_f2(nxt[i].z);
      v[i][3] = bf16x2_to_f2(nxt[i].w);
    }
    if (warp_live) load_row(row + RPB);                   // the next row's loads are in flight during this row
    float2 s2 = f2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < CPT; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) s2 = __fadd2_rn(s2, v[i][k]);
    float sum = s2.x + s2.y;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (warp_live && lane == 0) red[0][rib][wr] = sum;
    __syncthreads();
    float mean = 0.0f;
#pragma unroll
    for (int w = 0; w < WPR; ++w) mean += warp_live ? red[0][rib][w] : 0.0f;
    mean /= D;
    const float2 nm = f2(-mean, -mean);
    float2 q2 = f2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < CPT; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[i][k] = __fadd2_rn(v[i][k], nm);
        q2 = __ffma2_rn(v[i][k], v[i][k], q2);
      }
    float var = q2.x + q2.y;
#pragma unroll
    for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    if (warp_live && lane == 0) red[1][rib][wr] = var;
    __syncthreads();
    if (live) {
      float vs = 0.0f;
#pragma unroll
      for (int w = 0; w < WPR; ++w) vs += red[1][rib][w];
      const float rstd = rsqrtf(vs / D + eps);
      const float2 r2 = f2(rstd, rstd);
      // this row's part of the tiled scale offset
      const size_t sf_row = (static_cast<size_t>(row >> 7) * sf_chunks) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
#pragma unroll
      for (int i = 0; i < CPT; ++i) {
        const int ch = i * WPR + wr;
        const int c0 = ch * 256 + lane * 8;
        const float4 a0 = ada_tab[ch * 64 + lane], a1 = ada_tab[ch * 64 + 32 + lane];
        const float4 h0 = ada_tab[NCH * 64 + ch * 64 + lane], h1 = ada_tab[NCH * 64 + ch * 64 + 32 + lane];
        const float2 y0 = __ffma2_rn(__fmul2_rn(v[i][0], r2), f2(a0.x, a0.y), f2(h0.x, h0.y));
        const float2 y1 = __ffma2_rn(__fmul2_rn(v[i][1], r2), f2(a0.z, a0.w), f2(h0.z, h0.w));
        const float2 y2 = __ffma2_rn(__fmul2_rn(v[i][2], r2), f2(a1.x, a1.y), f2(h1.x, h1.y));
        const float2 y3 = __ffma2_rn(__fmul2_rn(v[i][3], r2), f2(a1.z, a1.w), f2(h1.z, h1.w));
        const uint4 packed = make_uint4(pack_bf16x2(y0.x, y0.y), pack_bf16x2(y1.x, y1.y), pack_bf16x2(y2.x, y2.y),
                                        pack_bf16x2(y3.x, y3.y));
        if (out) *reinterpret_cast<uint4*>(out + row * D + c0) = packed;
        if (codes) {
          // the bf16-rounded result is what gets quantized: block max on packed bf16 magnitudes, then the lane pair
          const uint32_t ax = packed.x & 0x7FFF7FFFu, ay = packed.y & 0x7FFF7FFFu;
          const uint32_t az = packed.z & 0x7FFF7FFFu, aw = packed.w & 0x7FFF7FFFu;
          const __nv_bfloat162 mm = __hmax2(__hmax2(*reinterpret_cast<const __nv_bfloat162*>(&ax),
                                                    *reinterpret_cast<const __nv_bfloat162*>(&ay)),
                                            __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&az),
                                                    *reinterpret_cast<const __nv_bfloat162*>(&aw)));
          const uint32_t mw = *reinterpret_cast<const uint32_t*>(&mm);
          float amax = fmaxf(__uint_as_float(mw << 16), __uint_as_float(mw & 0xFFFF0000u));
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
          const uint32_t sfb = nvfp4_scale(amax, enc);
          const float inv = inv_tab[sfb];
          const float2 i2 = f2(inv, inv);
          const float2 p0 = __fmul2_rn(bf16x2_to_f2(packed.x), i2), p1 = __fmul2_rn(bf16x2_to_f2(packed.y), i2);
          const float2 p2 = __fmul2_rn(bf16x2_to_f2(packed.z), i2), p3 = __fmul2_rn(bf16x2_to_f2(packed.w), i2);
          *reinterpret_cast<uint32_t*>(codes + row * (D >> 1) + (c0 >> 1)) =
              e2m1x8(p0.x, p0.y, p1.x, p1.y, p2.x, p2.y, p3.x, p3.y);
          // lane 2q holds block ch * 16 + q: byte (q % 4) of word ch * 4 + q / 4 of the row in the tiled layout
          if ((lane & 1) == 0) sf[sf_row + (size_t)(ch * 4 + (lane >> 3)) * 512 + ((lane >> 1) & 3)] = (uint8_t)sfb;
        }
      }
    }
  }
}

template <int NCH>
tfb_status launch_adaln(const DeviceInfo* di, const void* x, int64_t B, int64_t N, int64_t rows_total,
                        const float* scale, const float* shift, float eps, void* out, float qg, uint8_t* codes,
                        uint8_t* sf, cudaStream_t s) {
  constexpr int RPB = AdaSplit<NCH>::RPB;
  constexpr int kSmem = 2 * NCH * 256 * 4;                // (1 + scale) and shift, fp32
  // blocks of this instantiation one SM holds at once, per device (set-up calls may race: they store the same value)
  static std::atomic<int> resident[64];
  int per_sm = resident[di->device].load(std::memory_order_acquire);
  if (!per_sm) {
    TFB_CUDA(cudaFuncSetAttribute(adaln_kernel<NCH>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    int n = 0;
    TFB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, adaln_kernel<NCH>, kAdaThreads, kSmem));
    per_sm = std::max(1, n);
    resident[di->device].store(per_sm, std::memory_order_release);
  }
  // one resident wave of blocks over all batch elements, each walking at least RPB rows
  const int64_t want = (int64_t)di->sm_count * per_sm;
  const int64_t by_rows = (N + RPB - 1) / RPB;
  const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>(by_rows, (want + B - 1) / B));
  const int pad_blocks = rows_total > B * N ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(chunks, (unsigned)(B + pad_blocks));
  cfg.blockDim = dim3(kAdaThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TFB_CUDA(cudaLaunchKernelEx(&cfg, adaln_kernel<NCH>, static_cast<const __nv_bfloat16*>(x), B, N, rows_total,
                              chunks, scale, shift, eps, static_cast<__nv_bfloat16*>(out), qg, codes, sf));
  return TFB_OK;
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

// UPT units per half-warp: unit hw + k * span for k < UPT (span = the grid's half-warps), so consecutive half-warps
// read consecutive heads; every unit's loads are issued before the first unit's math.
template <int UPT>
__global__ void __launch_bounds__(256) rms_rope_kernel(const __nv_bfloat16* __restrict__ src, int64_t units, int64_t N,
                                                       int64_t H, int64_t src_sb, int64_t src_sn, int64_t src_off,
                                                       const float* __restrict__ w, const float* __restrict__ cosp,
                                                       const float* __restrict__ sinp, float eps,
                                                       __nv_bfloat16* __restrict__ dst, int64_t dst_sb,
                                                       int64_t dst_sn) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128;
  const int64_t hw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;
  const int64_t span = (int64_t)gridDim.x * (blockDim.x >> 4);
  const int l = threadIdx.x & 15;
  uint4 raw[UPT];
  float4 c[UPT], s[UPT];
  int64_t doff[UPT];
  bool live[UPT];
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const int64_t unit = hw + k * span;
    live[k] = unit < units;
    const int64_t uu = live[k] ? unit : 0;              // dead lanes still take part in the row shuffles
    const int64_t h = uu % H, bn = uu / H, n = bn % N, b = bn / N;
    raw[k] = __ldg(reinterpret_cast<const uint4*>(src + b * src_sb + n * src_sn + src_off + h * D + l * 8));
    c[k] = __ldg(reinterpret_cast<const float4*>(cosp + n * (D / 2) + l * 4));
    s[k] = __ldg(reinterpret_cast<const float4*>(sinp + n * (D / 2) + l * 4));
    doff[k] = b * dst_sb + n * dst_sn + h * D + l * 8;
  }
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const float cv[4] = {c[k].x, c[k].y, c[k].z, c[k].w}, sv[4] = {s[k].x, s[k].y, s[k].z, s[k].w};
    const uint4 o = rms_rope_piece(raw[k], w, l, cv, sv, eps);
    if (live[k]) *reinterpret_cast<uint4*>(dst + doff[k]) = o;
  }
}

// q, k and v of a fused qkv row [B, N, 3, H, D] in one pass: q and k normalised + rotated (one cos / sin read for
// both), v copied; each goes to its own strided destination (k and v typically behind a kept prefix).
template <int UPT>
__global__ void __launch_bounds__(256) rms_rope_qkv_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t units, int64_t N, int64_t H, int64_t src_sb, int64_t src_sn,
    const float* __restrict__ wq, const float* __restrict__ wk, const float* __restrict__ cosp,
    const float* __restrict__ sinp, float eps, __nv_bfloat16* __restrict__ qd, int64_t q_sb, int64_t q_sn,
    __nv_bfloat16* __restrict__ kd, int64_t k_sb, int64_t k_sn, __nv_bfloat16* __restrict__ vd, int64_t v_sb,
    int64_t v_sn) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128;
  const int64_t hw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;
  const int64_t span = (int64_t)gridDim.x * (blockDim.x >> 4);
  const int l = threadIdx.x & 15;
  uint4 rq[UPT], rk[UPT], rv[UPT];
  float4 c[UPT], s[UPT];
  int64_t bb[UPT], nn[UPT], col[UPT];
  bool live[UPT];
#pragma unroll
  for (int k = 0; k < UPT; ++k) {                      // every unit's loads first (see rms_rope_kernel)
    const int64_t unit = hw + k * span;
    live[k] = unit < units;
    const int64_t uu = live[k] ? unit : 0;
    const int64_t h = uu % H, bn = uu / H, n = bn % N, b = bn / N;
    const __nv_bfloat16* sp = src + b * src_sb + n * src_sn + h * D + l * 8;
    rq[k] = __ldg(reinterpret_cast<const uint4*>(sp));
    rk[k] = __ldg(reinterpret_cast<const uint4*>(sp + H * D));
    rv[k] = __ldg(reinterpret_cast<const uint4*>(sp + 2 * H * D));
    c[k] = __ldg(reinterpret_cast<const float4*>(cosp + n * (D / 2) + l * 4));
    s[k] = __ldg(reinterpret_cast<const float4*>(sinp + n * (D / 2) + l * 4));
    bb[k] = b;
    nn[k] = n;
    col[k] = h * D + l * 8;
  }
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const float cv[4] = {c[k].x, c[k].y, c[k].z, c[k].w}, sv[4] = {s[k].x, s[k].y, s[k].z, s[k].w};
    const uint4 oq = rms_rope_piece(rq[k], wq, l, cv, sv, eps);
    const uint4 ok = rms_rope_piece(rk[k], wk, l, cv, sv, eps);
    if (live[k]) {
      *reinterpret_cast<uint4*>(qd + bb[k] * q_sb + nn[k] * q_sn + col[k]) = oq;
      *reinterpret_cast<uint4*>(kd + bb[k] * k_sb + nn[k] * k_sn + col[k]) = ok;
      *reinterpret_cast<uint4*>(vd + bb[k] * v_sb + nn[k] * v_sn + col[k]) = rv[k];
    }
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
  for (int k = 0; k < 8; k += 2) {   // silu correctly rounded to bf16, two at a time (one paired conversion)
    const uint32_t sp = pack_bf16x2(silu_for_bf16(g[k]), silu_for_bf16(g[k + 1]));
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
  if (B > 65535) return fail(TFB_BAD_SHAPE, "adaln: at most 65535 batch elements (B=%lld)", (long long)B);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (D / 256) {
#define TFB_ADA(n) \
  case n: st = launch_adaln<n>(di, x, B, N, rows_total, scale, shift, eps, out, q_global, codes, sf, s); break;
    TFB_ADA(1) TFB_ADA(2) TFB_ADA(3) TFB_ADA(4) TFB_ADA(6) TFB_ADA(8) TFB_ADA(12) TFB_ADA(16) TFB_ADA(24) TFB_ADA(32)
#undef TFB_ADA
    default:
      return fail(TFB_BAD_SHAPE, "adaln: D=%lld not instantiated (256 x {1,2,3,4,6,8,12,16,24,32})", (long long)D);
  }
  if (st != TFB_OK) return st;
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
  // one unit per half-warp: at configs[2] size (4352 x 24 heads) 2 units ran in the same time and 4 or 8 slower
  constexpr int kUpt = 1;
  const int64_t threads = (units + kUpt - 1) / kUpt * 16;
  TFB_LAUNCH(rms_rope_kernel<kUpt>, (threads + 255) / 256, 256, static_cast<cudaStream_t>(stream), 
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
  // two units per half-warp (six 16-byte loads in flight per lane): 36.9 -> 32.8 us at configs[2] size on one
  // box; four were slower (47 us, 161 registers)
  constexpr int kUpt = 2;
  const int64_t threads = (units + kUpt - 1) / kUpt * 16;
  TFB_LAUNCH(rms_rope_qkv_kernel<kUpt>, (threads + 255) / 256, 256, static_cast<cudaStream_t>(stream), 
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
