// GGUF block decoders on the GPU: Q8_0, Q4_K, Q5_K, Q6_K raw blocks -> f32 / f16 / bf16 values.
//
// The reference decodes these with a chain of torch ops per tensor (tfimage/gguf_load.py:17-73: byte views, shifts,
// stacks, a float multiply per op, then .to(dtype)); every op reads and writes a full-size temporary in HBM. Here one
// kernel reads each block once and writes each value once. The arithmetic is the reference's, one IEEE rounding per
// operation in its order (__fmul_rn / __fsub_rn keep nvcc from contracting into an FMA, which would round once):
//   Q8_0  y = f16(d) * q                                   Q4_K/Q5_K  y = (f16(d) * sc) * q - (f16(dmin) * m)
//   Q6_K  y = (f16(d) * sc) * (q - 32)
// then one round-to-nearest-even to the output type.
//
// Work split: a CTA of 256 threads decodes a tile of 2048 values (8 super-blocks, or 64 Q8_0 blocks). The tile's
// raw bytes (a multiple of 16 for every type) are staged in shared memory with 16-byte loads; each thread then
// decodes 8 consecutive values and writes them with one 16-byte (f16/bf16) or two 16-byte (f32) stores, so a warp
// writes 256 or 512 contiguous bytes. Grid-stride over tiles, up to 8 CTAs per SM, each with the raw bytes of its
// next two tiles in flight (register prefetch) while it decodes the current one. HBM-bound: per value the kernel
// moves the block bytes / values (1.06 / 0.56 / 0.69 / 0.82 B for Q8_0 / Q4_K / Q5_K / Q6_K) plus the output.
#include "tfb_common.cuh"

#include <cuda_fp16.h>

namespace tfb {
namespace {

constexpr int kThreads = 256;
constexpr int kTileValues = kThreads * 8;

template <int TYPE>
struct Fmt;
template <>
struct Fmt<TFB_GGUF_Q8_0> {
  static constexpr int kValues = 32, kBytes = 34;
};
template <>
struct Fmt<TFB_GGUF_Q4_K> {
  static constexpr int kValues = 256, kBytes = 144;
};
template <>
struct Fmt<TFB_GGUF_Q5_K> {
  static constexpr int kValues = 256, kBytes = 176;
};
template <>
struct Fmt<TFB_GGUF_Q6_K> {
  static constexpr int kValues = 256, kBytes = 210;
};

__device__ __forceinline__ float f16_at(const uint8_t* p) {
  const unsigned short b = static_cast<unsigned short>(p[0] | (p[1] << 8));
  return __half2float(__ushort_as_half(b));
}

// Exact float of a small non-negative integer (v < 2^23) on the FP32 pipe: 2^23 + v has v in its mantissa, and
// subtracting 2^23 is exact. Same value as an int-to-float conversion, without the conversion pipe's lower rate.
__device__ __forceinline__ float small_u2f(uint32_t v) {
  return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.0f);
}

// Exact float of a signed byte: (b ^ 0x80) = b + 128 as an unsigned value, then subtract 2^23 + 128.
__device__ __forceinline__ float i8_to_f(uint32_t byte) {
  return __fsub_rn(__uint_as_float(0x4B000000u | ((byte & 0xFFu) ^ 0x80u)), 8388736.0f);
}

// 8 bytes at an 8-byte aligned shared-memory address.
__device__ __forceinline__ void bytes8(const uint8_t* p, uint32_t* b) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    b[i] = (w.x >> (8 * i)) & 0xFF;
    b[4 + i] = (w.y >> (8 * i)) & 0xFF;
  }
}

// Six-bit scale and min number `j` (0-7) of a K-quant block from its 12 packed bytes (ggml get_scale_min_k4).
__device__ __forceinline__ void scale_min_k4(const uint8_t* s, int j, float& sc, float& m) {
  if (j < 4) {
    sc = small_u2f(s[j] & 63);
    m = small_u2f(s[j + 4] & 63);
  } else {
    sc = small_u2f((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
    m = small_u2f((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

// Values o .. o+7 (o a multiple of 8) of one block staged at `blk`.
template <int TYPE>
__device__ __forceinline__ void decode8(const uint8_t* blk, int o, float* y) {
  if constexpr (TYPE == TFB_GGUF_Q8_0) {
    const float d = f16_at(blk);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fmul_rn(d, i8_to_f(blk[2 + o + i]));
  } else if constexpr (TYPE == TFB_GGUF_Q4_K || TYPE == TFB_GGUF_Q5_K) {
    const int j = o >> 6, hi = (o >> 5) & 1, p = o & 31, sub = 2 * j + hi;
    float sc, m;
    scale_min_k4(blk + 4, sub, sc, m);
    const float ds = __fmul_rn(f16_at(blk), sc);
    const float dm = __fmul_rn(f16_at(blk + 2), m);
    constexpr int kQs = TYPE == TFB_GGUF_Q4_K ? 16 : 48;
    uint32_t q[8];
    bytes8(blk + kQs + 32 * j + p, q);
    uint32_t h[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if constexpr (TYPE == TFB_GGUF_Q5_K) bytes8(blk + 16 + p, h);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t v = hi ? (q[i] >> 4) : (q[i] & 15);
      if constexpr (TYPE == TFB_GGUF_Q5_K) v |= ((h[i] >> sub) & 1) << 4;
      y[i] = __fsub_rn(__fmul_rn(ds, small_u2f(v)), dm);
    }
  } else {  // Q6_K: half h, run r of 32 values, position p within the run
    const int h = o >> 7, r = (o >> 5) & 3, p = o & 31;
    const float ds = __fmul_rn(f16_at(blk + 208), i8_to_f(blk[192 + 8 * h + 2 * r + (p >> 4)]));
    const uint8_t* ql = blk + 64 * h + 32 * (r & 1) + p;
    const uint8_t* qh = blk + 128 + 32 * h + p;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = r < 2 ? (ql[i] & 15) : (ql[i] >> 4);
      const float v = __fsub_rn(small_u2f(lo | (((qh[i] >> (2 * r)) & 3) << 4)), 32.0f);   // q - 32, exact
      y[i] = __fmul_rn(ds, v);
    }
  }
}

template <int OUT>
__device__ __forceinline__ void store8(void* out, int64_t idx, const float* y) {
  if constexpr (OUT == TFB_DT_F32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + idx);
    p[0] = make_float4(y[0], y[1], y[2], y[3]);
    p[1] = make_float4(y[4], y[5], y[6], y[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (OUT == TFB_DT_BF16) {
        w[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
      } else {
        __half2 hv = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&hv);
      }
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + idx) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int TYPE, int OUT>
__global__ void __launch_bounds__(kThreads, 8) gguf_kernel(const uint8_t* __restrict__ raw, int64_t n_blocks,
                                                          void* __restrict__ out) {
  using F = Fmt<TYPE>;
  constexpr int kBlocksPerTile = kTileValues / F::kValues;
  constexpr int kTileBytes = kBlocksPerTile * F::kBytes;
  constexpr int kVecs = kTileBytes / 16;          // 16-byte pieces of a full tile: at most one per thread
  static_assert(kTileBytes % 16 == 0 && kVecs <= kThreads, "a full tile stages with one 16-byte load per thread");
  __shared__ __align__(16) uint8_t stage[kTileBytes];
  pdl_trigger();
  pdl_wait();
  const int t = threadIdx.x;
  const int v0 = 8 * t;                 // this thread's first value within the tile
  const int blk = v0 / F::kValues;
  const int64_t step = gridDim.x;
  // The raw bytes of the next two tiles of this CTA are loaded into registers while the current tile decodes
  // (two tiles in flight per CTA), so the HBM reads of a CTA overlap its decode and stores.
  auto prefetch = [&](int64_t tile, uint4& r) {
    if (t < kVecs && (tile + 1) * kBlocksPerTile <= n_blocks)
      r = __ldg(reinterpret_cast<const uint4*>(raw + tile * kBlocksPerTile * F::kBytes) + t);
  };
  auto body = [&](int64_t tile, uint4& r) {
    const int64_t b0 = tile * kBlocksPerTile;
    const int nb = n_blocks - b0 < kBlocksPerTile ? static_cast<int>(n_blocks - b0) : kBlocksPerTile;
    if (nb == kBlocksPerTile) {
      if (t < kVecs) reinterpret_cast<uint4*>(stage)[t] = r;
    } else {                            // the ragged last tile: byte loads, no prefetch
      const uint8_t* src = raw + b0 * F::kBytes;
      for (int i = t; i < nb * F::kBytes; i += kThreads) stage[i] = __ldg(src + i);
    }
    __syncthreads();
    prefetch(tile + 2 * step, r);
    if (blk < nb) {
      float y[8];
      decode8<TYPE>(stage + blk * F::kBytes, v0 % F::kValues, y);
      store8<OUT>(out, b0 * F::kValues + v0, y);
    }
    __syncthreads();
  };
  uint4 r0 = make_uint4(0, 0, 0, 0), r1 = r0;
  int64_t tile = blockIdx.x;
  prefetch(tile, r0);
  prefetch(tile + step, r1);
  while (tile * kBlocksPerTile < n_blocks) {
    body(tile, r0);
    tile += step;
    if (tile * kBlocksPerTile >= n_blocks) break;
    body(tile, r1);
    tile += step;
  }
}

template <int TYPE>
tfb_status launch_type(const uint8_t* raw, int64_t n_values, void* out, int out_dtype, int grid_cap,
                       cudaStream_t s) {
  using F = Fmt<TYPE>;
  if (n_values % F::kValues)
    return fail(TFB_BAD_SHAPE, "gguf_dequant: %lld values is not a whole number of %d-value blocks",
                (long long)n_values, F::kValues);
  const int64_t n_blocks = n_values / F::kValues;
  const int64_t tiles = (n_blocks + kTileValues / F::kValues - 1) / (kTileValues / F::kValues);
  const int grid = static_cast<int>(tiles < grid_cap ? tiles : grid_cap);
  if (out_dtype == TFB_DT_F32)
    TFB_LAUNCH((gguf_kernel<TYPE, TFB_DT_F32>), grid, kThreads, s, raw, n_blocks, out);
  else if (out_dtype == TFB_DT_F16)
    TFB_LAUNCH((gguf_kernel<TYPE, TFB_DT_F16>), grid, kThreads, s, raw, n_blocks, out);
  else
    TFB_LAUNCH((gguf_kernel<TYPE, TFB_DT_BF16>), grid, kThreads, s, raw, n_blocks, out);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

}  // namespace
}  // namespace tfb

extern "C" {

int64_t tfb_gguf_block_bytes(int type, int64_t* values_per_block) {
  int64_t v = 0, b = 0;
  switch (type) {
    case TFB_GGUF_Q8_0: v = 32, b = 34; break;
    case TFB_GGUF_Q4_K: v = 256, b = 144; break;
    case TFB_GGUF_Q5_K: v = 256, b = 176; break;
    case TFB_GGUF_Q6_K: v = 256, b = 210; break;
    default: return -1;
  }
  if (values_per_block) *values_per_block = v;
  return b;
}

tfb_status tfb_gguf_dequant(int type, const uint8_t* raw, int64_t n_values, void* out, int out_dtype,
                            void* stream) {
  using namespace tfb;
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  if (tfb_gguf_block_bytes(type, nullptr) < 0)
    return fail(TFB_BAD_ARG, "gguf_dequant: ggml type %d is not decoded here (decoded: Q8_0=8, Q4_K=12, Q5_K=13, "
                             "Q6_K=14)", type);
  if (out_dtype != TFB_DT_F32 && out_dtype != TFB_DT_F16 && out_dtype != TFB_DT_BF16)
    return fail(TFB_BAD_ARG, "gguf_dequant: output type %d (f32=0, f16=1, bf16=2)", out_dtype);
  if (n_values < 0) return fail(TFB_BAD_SHAPE, "gguf_dequant: negative value count");
  if (!aligned(raw, 16) || !aligned(out, 16))
    return fail(TFB_BAD_ALIGN, "gguf_dequant: raw blocks and output must be 16-byte aligned");
  if (n_values == 0) return TFB_OK;
  const int cap = di->sm_count * 8;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (type) {
    case TFB_GGUF_Q8_0: return launch_type<TFB_GGUF_Q8_0>(raw, n_values, out, out_dtype, cap, s);
    case TFB_GGUF_Q4_K: return launch_type<TFB_GGUF_Q4_K>(raw, n_values, out, out_dtype, cap, s);
    case TFB_GGUF_Q5_K: return launch_type<TFB_GGUF_Q5_K>(raw, n_values, out, out_dtype, cap, s);
    default: return launch_type<TFB_GGUF_Q6_K>(raw, n_values, out, out_dtype, cap, s);
  }
}

}  // extern "C"
