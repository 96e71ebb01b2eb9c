/*
 * libtfb -- sm_100a (B200) kernels behind tfimage's quantized-linear API, as a plain C ABI.
 *
 * Conventions (every entry point):
 *   - all buffers are caller-owned device pointers; nothing here allocates device memory;
 *   - work is enqueued on the caller's stream (`stream` is a cudaStream_t passed as void*; NULL = legacy default);
 *   - no entry point synchronizes except tfb_device_status();
 *   - the return value is a tfb_status; on failure tfb_last_error() (thread-local) explains it;
 *   - shapes/alignments are validated before any launch (TFB_BAD_SHAPE / TFB_BAD_ALIGN), the device must be
 *     compute capability 10.0 (TFB_BAD_ARCH);
 *   - GEMM kernels bound every pipeline wait; a wait that runs out records a code that tfb_device_status()
 *     returns (TFB_DEVICE_TIMEOUT) instead of hanging the GPU.
 *
 * Formats:
 *   bf16       -- raw 16-bit bfloat16 bit patterns;
 *   NVFP4      -- codes: uint8 [rows, K/2], two E2M1 values per byte, even element in the low nibble;
 *                 scales: one E4M3 byte per 16 K-elements, either row-major [rows, K/16] (TFB_SF_ROWS) or the
 *                 GEMM layout TFB_SF_TILED: 512-byte chunks [ceil(rows/128)][K/64][512] where row r, scale j of a
 *                 chunk sits at (r%32)*16 + ((r%128)/32)*4 + (j%4); rows past the end are zero;
 *                 global: an fp32 per-tensor scale g, value = lut[code] * e4m3(scale) * g.
 *   FP8        -- E4M3 bytes [rows, K].
 */
#ifndef TFB_H
#define TFB_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  TFB_OK = 0,
  TFB_BAD_SHAPE = 1,
  TFB_BAD_ALIGN = 2,
  TFB_BAD_ARCH = 3,
  TFB_DEVICE_TIMEOUT = 4,
  TFB_CUDA_ERR = 5,
  TFB_BAD_ARG = 6
} tfb_status;

enum { TFB_SF_ROWS = 0, TFB_SF_TILED = 1 };

/* Library version (major*10000 + minor*100 + patch). */
int tfb_version(void);

/* Message for the last failing call on this host thread ("" if none). */
const char* tfb_last_error(void);

/* Bytes of a TFB_SF_TILED scale buffer for `rows` x `k` elements. */
int64_t tfb_sf_tiled_bytes(int64_t rows, int64_t k);

/* Synchronizes the current device and reads (and, if reset != 0, clears) the device-side error word set by a
 * kernel whose bounded wait ran out: *code = 0 when clean. Returns TFB_DEVICE_TIMEOUT when *code != 0. */
tfb_status tfb_device_status(int* code, int reset);

/* amax = max |x| over n bf16 values, written to *amax_dev (fp32, device).
 * Replaces the device half of `float(x.abs().amax())` in Nvfp4Linear.__call__ (tfimage/linear.py:127). */
tfb_status tfb_absmax_bf16(const void* x, int64_t n, float* amax_dev, void* stream);

/* Dynamic FP8 activation scale on the device: *a_dev = max(amax(x) / 448, 1e-12) (fp32).
 * Replaces Fp8Linear._act (tfimage/linear.py:84-89). */
tfb_status tfb_fp8_act_scale(const void* x, int64_t n, float* a_dev, void* stream);

/* NVFP4 row quantizer: x bf16 [M, K] (row stride ldx elements) under global g -> codes [M, K/2] + scales.
 * Replaces TensorFold checkpoint.quant4 (called at tfimage/linear.py:36 and tools/gemm_tf.py:17,45).
 * K % 64 == 0 (K % 16 == 0 for TFB_SF_ROWS). */
tfb_status tfb_quant_nvfp4(const void* x, int64_t M, int64_t K, int64_t ldx, float global, uint8_t* codes,
                           uint8_t* sf, int sf_layout, void* stream);

/* FP8 activation quantizer: q[m, k] = e4m3(clamp(x / *a_dev, -448, 448)) (tfimage/linear.py:95). q is [M, K]. */
tfb_status tfb_quant_fp8(const void* x, int64_t M, int64_t K, int64_t ldx, const float* a_dev, uint8_t* q,
                         void* stream);

/* W4A4 NVFP4 GEMM on tcgen05 block-scaled FP4 MMA: y[M, N] = bf16(alpha * sum_k deq(a)[m,k] * deq(b)[n,k])
 * with deq() excluding the globals (alpha = g_a * g_b). Scales in TFB_SF_TILED layout.
 * Replaces TensorFold checkpoint.prompt(A4, ...) after quantization (tfimage/linear.py:130). K % 128 == 0,
 * N % 32 == 0, ldy % 8 == 0. */
tfb_status tfb_gemm_nvfp4(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes, const uint8_t* b_sf,
                          int64_t M, int64_t N, int64_t K, float alpha, void* y, int64_t ldy, void* stream);

/* W8A8 FP8 GEMM on tcgen05 kind::f8f6f4: y[M, N] = bf16(sum_k a[m,k] b[n,k] * a_scale * b_scale[n or 0]).
 * Scales are device fp32 (a_scale: one value; b_scale: N values if b_per_channel else one). Replaces
 * torch._scaled_mm in Fp8Linear.__call__ (tfimage/linear.py:98); M is ragged (no padding). K % 16 == 0,
 * N % 16 == 0 (the reference's FP8 envelope, tfimage/linear.py:159), ldy % 8 == 0. */
tfb_status tfb_gemm_fp8(const uint8_t* a, const uint8_t* b, int64_t M, int64_t N, int64_t K, const float* a_scale,
                        const float* b_scale, int b_per_channel, void* y, int64_t ldy, void* stream);

/* NVFP4 GEMM fused with the block's gated residual: x[m, n] = bf16(fma(bf16(alpha * acc[m, n]),
 * gate[m / rows_per_gate, n], x[m, n])) in place, i.e. x.addcmul_(linear(a), gate) of the reference block
 * (tfimage/qwen_image21.py:213-215, torch computes addcmul as one fused multiply-add in fp32). x bf16 [M, N] with
 * row stride ldx (elements, % 8 == 0); gate bf16 rows of N with stride ld_gate (% 8 == 0, 16-byte aligned), one row
 * per rows_per_gate rows of x (the batch's tokens). Operand formats as tfb_gemm_nvfp4. */
tfb_status tfb_gemm_nvfp4_resid(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes,
                                const uint8_t* b_sf, int64_t M, int64_t N, int64_t K, float alpha, void* x,
                                int64_t ldx, const void* gate, int64_t ld_gate, int64_t rows_per_gate, void* stream);

/* The attention input projection with the block's q / k RMSNorm + RoPE and the v copy in the epilogue: for rows
 * m = b * ntok + n of a_codes [B * ntok, K/2] and W_qkv codes [3 * H * 128, K/2], the GEMM output (bf16(alpha * acc),
 * the reference's qkv tensor) of q and k heads is normalised and rotated with the arithmetic of tfb_rms_rope_qkv
 * (weights wq / wk fp32 [128], cos / sin fp32 [ntok, 64] of the image tokens) and v is copied; each part goes to
 * its destination + b * *_sb + n * *_sn + h * 128 (element strides; k and v typically behind a kept prefix).
 * Replaces the reference block's qkv linear + two rms_rope calls + the v copy (tfimage/qwen_image21.py:176-191);
 * bit-equal to tfb_gemm_nvfp4 followed by tfb_rms_rope_qkv. ntok % 32 == 0, K % 128 == 0. */
tfb_status tfb_gemm_nvfp4_qkv(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes,
                              const uint8_t* b_sf, int64_t B, int64_t ntok, int64_t H, int64_t K, float alpha,
                              const float* wq, const float* wk, const float* cos, const float* sin, float eps, void* q,
                              int64_t q_sb, int64_t q_sn, void* k, int64_t k_sb, int64_t k_sn, void* v, int64_t v_sb,
                              int64_t v_sn, void* stream);

/* Gate/up NVFP4 GEMM with a SwiGLU epilogue that writes NVFP4: W_gu = [gate; up] codes [2F, K].
 * h = bf16(bf16(silu(gate)) * up) with gate/up = bf16(alpha * acc), quantized under h_global into
 * h_codes [M, F/2] and h_sf (TFB_SF_TILED, rows = M, K = F). gu_out and h_out (both nullable) receive the
 * bf16 gate/up [M, 2F] and the bf16 h [M, F] for testing. Replaces the first half of TensorFold
 * checkpoint.mlp_prompt (tfimage/linear.py:150). F % 128 == 0, K % 128 == 0. */
tfb_status tfb_gemm_nvfp4_swiglu(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* gu_codes,
                                 const uint8_t* gu_sf, int64_t M, int64_t F, int64_t K, float alpha, float h_global,
                                 uint8_t* h_codes, uint8_t* h_sf, void* gu_out, void* h_out, void* stream);

/* Whole fused MLP pair (tfimage/linear.py:136-150, swiglu_mlp): quantize x [M, K] under act_x, gate/up GEMM with
 * the SwiGLU->NVFP4 epilogue under act_h, down GEMM -> y [M, K] bf16. The four ws_* buffers are caller-owned
 * scratch: ws_xc [M, K/2], ws_xsf tfb_sf_tiled_bytes(M, K), ws_hc [M, F/2], ws_hsf tfb_sf_tiled_bytes(M, F). */
tfb_status tfb_mlp_nvfp4(const void* x, int64_t M, int64_t K, int64_t F, float act_x, const uint8_t* gu_codes,
                         const uint8_t* gu_sf, float g_gu, const uint8_t* down_codes, const uint8_t* down_sf,
                         float g_down, float act_h, void* y, uint8_t* ws_xc, uint8_t* ws_xsf, uint8_t* ws_hc,
                         uint8_t* ws_hsf, void* stream);

/* Size of the device array that tfb_mlp_nvfp4_static uses as scratch: 32 MiB, one array per device. */
#define TFB_MLP_STATIC_SCRATCH_BYTES (32ll << 20)

/* The fused MLP pair of tfb_mlp_nvfp4 without a workspace argument and without allocating device memory: the
 * x codes/scales and hidden codes/scales live in a device array inside the library (TFB_MLP_STATIC_SCRATCH_BYTES
 * per device). This entry point has no counterpart in the reference, whose fused MLP gets its intermediates from
 * torch's allocator.
 * It is meant for callers that cannot allocate: a host that reaches the library only through this C interface
 * and holds nothing but the device pointers its engine handed over (no device allocator of its own); an engine
 * whose device memory is a fixed budget managed by its own pool, where an allocation behind the pool's back could
 * fail or upset its accounting; and latency-critical loops, where cudaMalloc / cudaFree can block the calling
 * thread or wait for the device to go idle.
 * Rules:
 *  - Limit: the call needs round256(M*K/2) + round256(tfb_sf_tiled_bytes(M, K)) + round256(M*F/2) +
 *    tfb_sf_tiled_bytes(M, F) bytes (round256 = up to a multiple of 256). More than TFB_MLP_STATIC_SCRATCH_BYTES
 *    returns TFB_BAD_SHAPE with a message naming both figures; nothing is launched. Example: M = 4352, K = 3072,
 *    F = 8192 needs 27.6 MB and fits; larger M must be split across calls or go through tfb_mlp_nvfp4.
 *  - Set-up: the first call on a device looks up that device's copy of the array (cudaGetSymbolAddress, with the
 *    device current) together with the library's other one-time per-device work (device query, kernel
 *    attributes). Make the first call on each device before beginning any stream capture.
 *  - One array per device: two calls that can be in flight at the same time on the same device (different
 *    streams, or different host threads without ordering) race on it and corrupt each other's outputs. Issue
 *    them on one stream or otherwise serialise them. Calls on one stream are ordered and safe.
 *  - Nothing in the array has to start at zero and the library never clears it: every byte a call reads from it
 *    was written earlier in the same call.
 * Arguments, shape rules and results are those of tfb_mlp_nvfp4. */
tfb_status tfb_mlp_nvfp4_static(const void* x, int64_t M, int64_t K, int64_t F, float act_x, const uint8_t* gu_codes,
                                const uint8_t* gu_sf, float g_gu, const uint8_t* down_codes, const uint8_t* down_sf,
                                float g_down, float act_h, void* y, void* stream);

/* AdaLN modulate: per row of x [B*N, D] (batch b = row / N): y = LN(x) * (1 + scale[b]) (+ shift[b]), fp32
 * inside, eps inside the rsqrt; scale/shift are fp32 [B, D] (shift nullable). Outputs (each nullable, at least
 * one): out bf16 [B*N, D]; NVFP4 codes [B*N, D/2] + tiled scales of the bf16-rounded result under q_global.
 * Replaces the Triton _adaln_kernel (tfimage/kernels.py:14-37). D % 256 == 0, D <= 8192. */
tfb_status tfb_adaln(const void* x, int64_t B, int64_t N, int64_t D, const float* scale, const float* shift,
                     float eps, void* out, float q_global, uint8_t* codes, uint8_t* sf, void* stream);

/* RMSNorm over the head dim (weight w, fp32 [D]) then RoPE on interleaved pairs with cos/sin fp32 [N, D/2], per
 * (b, n, h): src element (b, n, h, d) at src + b*src_sb + n*src_sn + src_off + h*D + d; dst at
 * dst + b*dst_sb + n*dst_sn + h*D + d (element strides; dst may be a row slice of a larger buffer).
 * Replaces the Triton _rms_rope_kernel (tfimage/kernels.py:40-70). D == 128. */
tfb_status tfb_rms_rope(const void* src, int64_t B, int64_t N, int64_t H, int64_t D, int64_t src_sb, int64_t src_sn,
                        int64_t src_off, const float* w, const float* cos, const float* sin, float eps, void* dst,
                        int64_t dst_sb, int64_t dst_sn, void* stream);

/* The attention inputs of one block in one pass: src = qkv rows [B, N, 3, H, D] (element strides src_sb, src_sn;
 * q, k, v at column offsets 0, H*D, 2*H*D) -> q = rms_rope(q part, wq), k = rms_rope(k part, wk), v = v part, each
 * to its own strided destination (element strides *_sb, *_sn; dst + b*sb + n*sn + h*D + d). Same arithmetic as
 * tfb_rms_rope per part. Replaces the reference block's two rms_rope calls plus the v copy into the kept-prefix
 * buffer (tfimage/qwen_image21.py:180-191). D == 128. */
tfb_status tfb_rms_rope_qkv(const void* src, int64_t B, int64_t N, int64_t H, int64_t D, int64_t src_sb,
                            int64_t src_sn, const float* wq, const float* wk, const float* cos, const float* sin,
                            float eps, void* q, int64_t q_sb, int64_t q_sn, void* k, int64_t k_sb, int64_t k_sn,
                            void* v, int64_t v_sb, int64_t v_sn, void* stream);

/* Standalone SwiGLU: gu bf16 [M, 2F] = [gate | up] -> out bf16 [M, F] = bf16(bf16(silu(gate)) * up), silu rounded
 * correctly to bf16 (the round-to-nearest-even bf16 of the exact value).
 * Replaces the Triton _swiglu_kernel (tfimage/kernels.py:73-92). F % 8 == 0. */
tfb_status tfb_swiglu(const void* gu, int64_t M, int64_t F, void* out, void* stream);

/* ---- Tensor-parallel MLP down projection with the cross-GPU reduction fused into the GEMM (no counterpart in the
 * reference, which runs on one GPU; it replaces the NCCL all-reduce + addcmul_ of the K-split down projection of
 * tfimage/tp.py, the reference's linear.py:136-150 MLP split over ranks). One process per GPU, all on one node. */
#define TFB_TP_MAX_WORLD 8

/* Every rank's communication buffer as mapped in this process (base[rank] = its own; the others through
 * tfb_ipc_open), and the shape it was laid out for. */
typedef struct {
  int world, rank;
  void* base[TFB_TP_MAX_WORLD];
  int64_t max_rows, n_cols;
} tfb_tp_comm;

/* Bytes of one rank's communication buffer for `world` ranks and up to max_rows x n_cols bf16 rows, and (nullable)
 * offsets[5] of its regions: x (the replicated residual stream [max_rows, n_cols] bf16, row stride n_cols), the
 * receive slots, the partial counters, the x counters, the device epoch word. The buffer must be zero before its
 * first use, on every rank before any rank's first call; it serves one (M, N) shape until it is zeroed again. -1 on
 * bad arguments. */
int64_t tfb_tp_layout(int world, int64_t max_rows, int64_t n_cols, int64_t* offsets);

/* x += gate * (sum over ranks of bf16(alpha * a_r @ b_r^T)), x = the comm's x region [M, N] on every rank: this
 * rank's K-slice (a_codes [M, K/2], b_codes [N, K/2], tiled scales) is multiplied on tcgen05; the M rows are cut into
 * one chunk per rank; tiles of other ranks' chunks are sent to their owners over NVLink as they finish, tiles of
 * this rank's chunk add the received partials (bf16 sum in rank order, fp32) and the gated residual
 * (bf16(fma(y, gate, x)), the arithmetic of tfb_gemm_nvfp4_resid) and are stored into every rank's x. Every rank
 * calls it with the same M, N, K, gate and epoch (1, 2, 3, ... per call on this buffer). x rows of other ranks'
 * chunks are complete only after tfb_tp_wait. Waits are bounded (TFB_DEVICE_TIMEOUT via tfb_device_status).
 * epoch = 0 takes the epoch from this rank's device epoch word instead (advanced by tfb_tp_advance on the same
 * stream before each call), so that a captured CUDA graph of the calls can be replayed. */
tfb_status tfb_gemm_nvfp4_tp(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes, const uint8_t* b_sf,
                             int64_t M, int64_t N, int64_t K, float alpha, const void* gate, int64_t ld_gate,
                             int64_t rows_per_gate, const tfb_tp_comm* comm, uint32_t epoch, void* stream);

/* Enqueues a wait (bounded) until every other rank's x rows of call `epoch` (0: the device epoch word) are in
 * this rank's x. */
tfb_status tfb_tp_wait(const tfb_tp_comm* comm, int64_t M, int64_t N, uint32_t epoch, void* stream);

/* Enqueues this rank's device epoch word += 1 (for the epoch = 0 form of the two calls above). */
tfb_status tfb_tp_advance(const tfb_tp_comm* comm, void* stream);

/* CUDA IPC between the processes of one node: the 64-byte handle of the device allocation holding `ptr`, and ptr's
 * offset inside it; tfb_ipc_open maps another process's allocation here (*ptr = its base + offset); tfb_ipc_close
 * unmaps it (ptr as returned by tfb_ipc_open, with the same offset). */
tfb_status tfb_ipc_handle(const void* ptr, uint8_t* handle, int64_t* offset);
tfb_status tfb_ipc_open(const uint8_t* handle, int64_t offset, void** ptr);
tfb_status tfb_ipc_close(void* ptr, int64_t offset);

/* GGUF quantized block types decoded on the device (ggml type ids) and output element types. */
enum { TFB_GGUF_Q8_0 = 8, TFB_GGUF_Q4_K = 12, TFB_GGUF_Q5_K = 13, TFB_GGUF_Q6_K = 14 };
enum { TFB_DT_F32 = 0, TFB_DT_F16 = 1, TFB_DT_BF16 = 2 };

/* Bytes per block of a TFB_GGUF_* type (-1 for any other type); *values_per_block (nullable) receives 32 or 256. */
int64_t tfb_gguf_block_bytes(int type, int64_t* values_per_block);

/* GGUF block decode: raw = n_values / values_per_block consecutive blocks of `type` (device, 16-byte aligned) ->
 * out (device, 16-byte aligned) n_values elements of out_dtype, in block order (the tensor's row-major order).
 * Arithmetic: one fp32 rounding per operation in the reference's order, then round to nearest even to out_dtype.
 * Replaces the torch decoders _q8_0 / _q6_k / _q4_k / _q5_k and the .to(dtype) of dequantize
 * (tfimage/gguf_load.py:21-86). n_values % values_per_block == 0. */
tfb_status tfb_gguf_dequant(int type, const uint8_t* raw, int64_t n_values, void* out, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TFB_H */
