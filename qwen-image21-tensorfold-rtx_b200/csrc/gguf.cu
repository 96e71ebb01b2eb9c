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
// Work split: a CTA of 256 threads decodes a tile of 4096 values (16 super-blocks, or 128 Q8_0 blocks). The tile's
// raw bytes (a multiple of 16 for every type) are staged in shared memory with 16-byte loads; each thread then
// decodes 16 consecutive values -- they share one block scale (and min), so the scale unpacking is paid once per
// 16 -- and writes them with two 16-byte (f16/bf16) or four (f32) stores. Codes become floats with one byte
// permute + one exact FP32 add each (2^23 + code), no conversion instructions. Grid-stride over tiles, up to 4 CTAs
// per SM, each with the raw bytes of its next two tiles in flight (register prefetch) while it decodes the current
// one. The 8-values-per-thread version was bound by instruction issue (~22 instructions per value). Per value the kernel
// moves the block bytes / values (1.06 / 0.56 / 0.69 / 0.82 B for Q8_0 / Q4_K / Q5_K / Q6_K) plus the output.
#include "tfb_common.cuh"

#include <cuda_fp16.h>

namespace tfb {
namespace {

constexpr int kThreads = 256;
constexpr int kVpt = 16;                       // values per thread: one block scale (and min) serves all 16
constexpr int kTileValues = kThreads * kVpt;   // 4096 values per CTA tile

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
  const unsigned short b = *reinterpret_cast<const unsigned short*>(p);     // 2-byte aligned in every format
  return __half2float(__ushort_as_half(b));
}

// Byte k of w as a float, exactly, with one byte permute and one FP32 add: the permute builds 0x4B0000bb = 2^23 + b
// and subtracting `bias` (2^23 plus an offset) is exact for these small integers.
template <int K>
__device__ __forceinline__ float byte_f(uint32_t w, float bias) {
  return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | K)), bias);
}

// Six-bit scale and min number `j` (0-7) of a K-quant block from its 12 packed bytes (ggml get_scale_min_k4).
__device__ __forceinline__ void scale_min_k4(const uint8_t* s, int j, float& sc, float& m) {
  uint32_t a, b;
  if (j < 4) {
    a = s[j] & 63;
    b = s[j + 4] & 63;
  } else {
    a = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    b = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
  sc = __fsub_rn(__uint_as_float(0x4B000000u | a), 8388608.0f);
  m = __fsub_rn(__uint_as_float(0x4B000000u | b), 8388608.0f);
}

// 16 bytes at a 2-byte aligned shared-memory address, as 4 little-endian words.
__device__ __forceinline__ void words16_a2(const uint8_t* p, uint32_t* w) {
  const unsigned short* h = reinterpret_cast<const unsigned short*>(p);
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = __byte_perm(h[2 * k], h[2 * k + 1], 0x5410);
}

// Values o .. o+15 (o a multiple of 16) of one block staged at `blk`: y[i] for value o + i.
template <int TYPE>
__device__ __forceinline__ void decode16(const uint8_t* blk, int o, float* y) {
  uint32_t q[4];                 // the 16 integer codes, one per byte, value i = byte i % 4 of word i / 4
  float mul, sub = 0.0f, bias = 8388608.0f;
  bool affine = false;           // K-quants with a min: y = ds * q - dm
  if constexpr (TYPE == TFB_GGUF_Q8_0) {
    words16_a2(blk + 2 + o, q);
#pragma unroll
    for (int k = 0; k < 4; ++k) q[k] ^= 0x80808080u;   // signed byte b -> b + 128
    mul = f16_at(blk);
    bias = 8388736.0f;                                // 2^23 + 128
  } else if constexpr (TYPE == TFB_GGUF_Q4_K || TYPE == TFB_GGUF_Q5_K) {
    const int j = o >> 6, hi = (o >> 5) & 1, p = o & 31, sb = 2 * j + hi;
    float sc, m;
    scale_min_k4(blk + 4, sb, sc, m);
    mul = __fmul_rn(f16_at(blk), sc);
    sub = __fmul_rn(f16_at(blk + 2), m);
    affine = true;
    constexpr int kQs = TYPE == TFB_GGUF_Q4_K ? 16 : 48;
    const uint4 w = *reinterpret_cast<const uint4*>(blk + kQs + 32 * j + p);   // 16-byte aligned (144 / 176-byte blocks)
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) q[k] = (hi ? ws[k] >> 4 : ws[k]) & 0x0F0F0F0Fu;
    if constexpr (TYPE == TFB_GGUF_Q5_K) {
      const uint4 h = *reinterpret_cast<const uint4*>(blk + 16 + p);          // bit sb of qh[p + i]
      const uint32_t hs[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] |= ((hs[k] >> sb) & 0x01010101u) << 4;
    }
  } else {  // Q6_K: half h, run r of 32 values, position p within the run; q - 32 through the bias
    const int h = o >> 7, r = (o >> 5) & 3, p = o & 31;
    mul = __fmul_rn(f16_at(blk + 208),
                    __fsub_rn(__uint_as_float(0x4B000000u | ((blk[192 + 8 * h + 2 * r + (p >> 4)] ^ 0x80u) & 0xFFu)),
                              8388736.0f));
    uint32_t lo[4], hb[4];
    words16_a2(blk + 64 * h + 32 * (r & 1) + p, lo);
    words16_a2(blk + 128 + 32 * h + p, hb);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      q[k] = ((r < 2 ? lo[k] : lo[k] >> 4) & 0x0F0F0F0Fu) | (((hb[k] >> (2 * r)) & 0x03030303u) << 4);
    bias = 8388640.0f;                                // 2^23 + 32
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float f[4] = {byte_f<0>(q[k], bias), byte_f<1>(q[k], bias), byte_f<2>(q[k], bias), byte_f<3>(q[k], bias)};
#pragma unroll
    for (int b = 0; b < 4; ++b) y[4 * k + b] = affine ? __fsub_rn(__fmul_rn(mul, f[b]), sub) : __fmul_rn(mul, f[b]);
  }
}

template <int OUT>
__device__ __forceinline__ void store16(void* out, int64_t idx, const float* y) {
  if constexpr (OUT == TFB_DT_F32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + idx);
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if constexpr (OUT == TFB_DT_BF16) {
        w[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
      } else {
        __half2 hv = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&hv);
      }
    }
    uint4* p = reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + idx);
    p[0] = make_uint4(w[0], w[1], w[2], w[3]);
    p[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

template <int TYPE, int OUT>
__global__ void __launch_bounds__(kThreads, 4) gguf_kernel(const uint8_t* __restrict__ raw, int64_t n_blocks,
                                                             void* __restrict__ out) {
  using F = Fmt<TYPE>;
  constexpr int kBlocksPerTile = kTileValues / F::kValues;
  constexpr int kTileBytes = kBlocksPerTile * F::kBytes;
  constexpr int kVecs = kTileBytes / 16;                      // 16-byte pieces of a full tile
  constexpr int kLpt = (kVecs + kThreads - 1) / kThreads;     // of them per thread (1, or 2 for Q8_0)
  static_assert(kTileBytes % 16 == 0, "a full tile stages with 16-byte loads");
  __shared__ __align__(16) uint8_t stage[kTileBytes];
  pdl_trigger();
  pdl_wait();
  const int t = threadIdx.x;
  const int v0 = kVpt * t;              // this thread's first value within the tile
  const int blk = v0 / F::kValues;
  const int64_t step = gridDim.x;
  // The raw bytes of the next two tiles of this CTA are loaded into registers while the current tile decodes
  // (two tiles in flight per CTA), so the HBM reads of a CTA overlap its decode and stores.
  auto prefetch = [&](int64_t tile, uint4* r) {
    if ((tile + 1) * kBlocksPerTile <= n_blocks) {
      const uint4* src = reinterpret_cast<const uint4*>(raw + tile * kBlocksPerTile * F::kBytes);
#pragma unroll
      for (int l = 0; l < kLpt; ++l)
        if (t + l * kThreads < kVecs) r[l] = __ldg(src + t + l * kThreads);
    }
  };
  auto body = [&](int64_t tile, uint4* r) {
    const int64_t b0 = tile * kBlocksPerTile;
    const int nb = n_blocks - b0 < kBlocksPerTile ? static_cast<int>(n_blocks - b0) : kBlocksPerTile;
    if (nb == kBlocksPerTile) {
#pragma unroll
      for (int l = 0; l < kLpt; ++l)
        if (t + l * kThreads < kVecs) reinterpret_cast<uint4*>(stage)[t + l * kThreads] = r[l];
    } else {                            // the ragged last tile: byte loads, no prefetch
      const uint8_t* src = raw + b0 * F::kBytes;
      for (int i = t; i < nb * F::kBytes; i += kThreads) stage[i] = __ldg(src + i);
    }
    __syncthreads();
    prefetch(tile + 2 * step, r);
    if (blk < nb) {
      float y[kVpt];
      decode16<TYPE>(stage + blk * F::kBytes, v0 % F::kValues, y);
      store16<OUT>(out, b0 * F::kValues + v0, y);
    }
    __syncthreads();
  };
  uint4 r0[kLpt], r1[kLpt];
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
  const int cap = di->sm_count * 4;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (type) {
    case TFB_GGUF_Q8_0: return launch_type<TFB_GGUF_Q8_0>(raw, n_values, out, out_dtype, cap, s);
    case TFB_GGUF_Q4_K: return launch_type<TFB_GGUF_Q4_K>(raw, n_values, out, out_dtype, cap, s);
    case TFB_GGUF_Q5_K: return launch_type<TFB_GGUF_Q5_K>(raw, n_values, out, out_dtype, cap, s);
    default: return launch_type<TFB_GGUF_Q6_K>(raw, n_values, out, out_dtype, cap, s);
  }
}

}  // extern "C"
