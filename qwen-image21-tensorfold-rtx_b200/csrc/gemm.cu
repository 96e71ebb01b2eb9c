// tcgen05 GEMMs for sm_100a: NVFP4 W4A4 (kind::mxf4nvf4, E4M3 block scales per 16), FP8 W8A8 (kind::f8f6f4), and
// the NVFP4 gate/up GEMM whose epilogue applies SwiGLU and writes NVFP4 rows + scales for the down projection.
//
// Persistent kernel, one CTA per SM. For M > 128 the CTAs work in pairs (a 2-CTA cluster, tcgen05 cta_group::2):
// the pair owns a 256 x 256 output tile, each CTA holds 128 A rows and half of the tile's 256 B rows in its shared
// memory, and the leader (rank 0) issues M=256 MMAs that run on both SMs' tensor cores, each accumulating its own
// 128 rows x 256 columns in its own TMEM. Per SM that halves the B bytes TMA must deliver per MMA (the single-CTA
// kernel was bound by it). M <= 128 uses single CTAs on 128 x 256 tiles. Warp roles (448 threads, 14 warps):
//   warp 0 lane 0 : TMA producer -- per stage its A tile [128 rows x 128 B] and B rows [128 (pair) or 256 x 128 B],
//                   128-byte swizzle, plus the stage's scale chunks (NVFP4). In a pair the tile loads of both CTAs
//                   complete on the leader's `full` barrier (cta_group::2 tensor loads), so the MMA thread waits
//                   on one local barrier for both halves.
//   warp 1        : allocates TMEM (512 columns); lane 0 of the leader issues tcgen05.mma (N=256, K=64 fp4 / 32
//                   fp8) into a 256-column fp32 accumulator. Its waits poll with mbarrier.test_wait: a blocking
//                   try_wait on the issue path costs ~128 cycles per stage, a quarter of the stage's MMA time.
//   warps 2..5    : scale writers (NVFP4 modes) -- copy the stage's scales from shared memory into this CTA's TMEM
//                   with tcgen05.st (one warp per TMEM lane quadrant) and arrive on the leader's `full` barrier, so
//                   that one barrier per stage tells the MMA thread both the tiles and the scales are in place.
//                   tcgen05.cp of the same bytes serialises with the MMAs and costs ~40% of the tensor time;
//                   tcgen05.st from four warps runs alongside them.
//   warps 6..13   : epilogue, two warps per TMEM lane quadrant (warp w reads lanes 32*(w%4)..+31, one output row
//                   per thread, each warp half of the columns). They drain the accumulator into registers, release
//                   it to the MMA thread, then scale / convert / store while the next tile's MMAs run. bf16 outputs
//                   go through a 128-byte-swizzled smem box per warp and TMA tensor stores: per-row 16-byte global
//                   stores crowd the memory-instruction path the MMA issue shares and stalled it ~4500 cycles/tile.
//                   FP8 keeps no scales in TMEM, so its accumulator is double-buffered (tile t in columns
//                   256 * (t % 2)) and the next tile's MMAs do not wait for the drain.
// Every mbarrier wait is bounded (kWaitLimitNs); a wait that runs out records a code in the device error word,
// the other roles see it and leave their loops, in-flight copies/MMAs are drained (bounded) and TMEM is freed.
// Each CTA issues its own tile loads from this GPU's memory; no load is broadcast across the cluster.
#include <stdlib.h>

#include <atomic>
#include <mutex>

#include "tfb_common.cuh"

namespace tfb {
namespace {

constexpr int BM = 128, BN = 256, BKB = 128;  // tile rows, tile cols, K bytes per stage (and swizzle span)

constexpr int A_BYTES = BM * BKB;             // 16 KB
constexpr int SFA_BYTES = 4 * 512;            // 4 scale chunks (64 K-elements each) of 128 rows
constexpr int SFB_BYTES = 2 * 4 * 512;        // two 128-row groups
constexpr int OUT_WARP_BYTES = 32 * 128;      // epilogue staging per warp: 32 rows x 128 B (one TMA store box)
constexpr int OUT_BYTES = 8 * OUT_WARP_BYTES; // 8 epilogue warps
constexpr int THREADS = 448;
// MODE_FP4_TP adds warp 14: it turns the epilogue's finished tiles into cross-GPU signals (a system-scope fence
// and a counter add on the peer per tile), so the epilogue warps never stall on a fence; kSigSlots tiles in flight.
constexpr int SIG_WARP = 14, kSigSlots = 4;
template <int MODE>
constexpr int kThreads = MODE == 4 ? THREADS + 32 : THREADS;
constexpr int EPI_WARP0 = 6;   // warps 2..5 write scales, 6..13 drain the accumulator
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_COL = 0;               // accumulator: columns [0, 256)
constexpr uint32_t SF_COL = 256;              // scales: one 48-column buffer per stage (SFA 4 x 4, SFB 4 x 8)
constexpr uint32_t SF_STAGE_COLS = 48;

// MODE_FP4_RESID: NVFP4 GEMM whose epilogue adds the gated result into a bf16 residual stream in place,
// y = bf16(fma(bf16(alpha * acc), gate[row / rows_per_gate, col], y)) -- torch's x.addcmul_(linear(a), gate).
// MODE_FP4_TP: the K-split (tensor-parallel) down projection with the cross-GPU reduction fused into the
// epilogue. The M rows are cut into one chunk per rank; rank r computes its bf16 partial of every tile, sends
// the tiles of other ranks' chunks to their owners over NVLink (peer stores into the owner's receive slot, then a
// per-tile counter on the owner), and for the tiles of its own chunk adds the received partials,
// x = bf16(fma(bf16(sum over ranks of the partials), gate, x)), and stores the new x rows locally and into every
// other rank's x (again with a per-tile counter). Tiles of other ranks' chunks go first, so by the time a rank
// reaches its own chunk the partials for it have been sent a wave of tiles earlier.
// MODE_FP4_QKV: the attention input projection with the reference block's RMSNorm + RoPE of q and k (and the v
// copy behind the kept prefix) in the epilogue: every 128-column half of a 256-column tile is one head of one of
// q / k / v (H * 128 columns each), one epilogue thread holds one head row, so the row's norm needs no exchange.
enum Mode { MODE_FP4 = 0, MODE_FP8 = 1, MODE_FP4_SWIGLU = 2, MODE_FP4_RESID = 3, MODE_FP4_TP = 4, MODE_FP4_QKV = 5 };

struct Params {
  int M, N;              // output rows / cols (swiglu: N = F, the hidden width)
  int num_m, num_n, num_tiles;
  int num_ks;            // pipeline stages along K
  int kb_total;          // MMA k-blocks along K
  int b_rows;            // rows of the B operand (N, or 2F for swiglu)
  const uint8_t* sfa;    // tiled scales (fp4 modes)
  const uint8_t* sfb;
  int sf_chunks;         // K / 64
  int sfb_groups;        // ceil(b_rows / 128)
  int sfa_groups;        // ceil(M / 128): scale groups (and tiled-scale rows / 128) of A and of the h output
  void* y;
  int64_t ldy;
  float alpha;           // fp4: g_a * g_b
  const float* a_scale;  // fp8
  const float* b_scale;
  int b_per_channel;
  float h_g;             // swiglu: global of the NVFP4 output
  uint8_t* h_codes;      // [M, F/2]
  uint8_t* h_sf;         // tiled, K = F
  __nv_bfloat16* gu_out; // optional [M, 2F]
  __nv_bfloat16* h_out;  // optional [M, F]
  const __nv_bfloat16* gate;   // resid: [rows / rows_per_gate, N] with row stride ld_gate
  int64_t ld_gate;
  int64_t rows_per_gate;
  int* err;
  // MODE_FP4_TP
  int tp_world, tp_rank;
  int tp_chunk_mb;       // M blocks (BM * CG rows) per rank's chunk
  int tp_chunk_rows;
  int tp_tiles_chunk;    // flag slots per (sender or owner, chunk): tp_chunk_mb * num_n
  uint32_t tp_target;    // a tile's counter value once both CTAs of its group signalled this launch: CG * epoch
  const uint32_t* tp_epoch_dev;   // non-null: the epoch is this rank's device epoch word (tfb_tp_advance)
  uint8_t* tp_base[TFB_TP_MAX_WORLD];   // every rank's communication buffer as mapped here (this rank's included)
  int64_t tp_r_off, tp_fp_off, tp_fx_off;
  // MODE_FP4_QKV: rows m = b * qk_ntok + n; outputs part p in {q, k, v} at dst[p] + b * sb[p] + n * sn[p] + h * 128
  int qk_heads, qk_ntok;
  __nv_bfloat16* qk_dst[3];
  int64_t qk_sb[3], qk_sn[3];
  const float* qk_w[2];          // RMSNorm weights of q and k, fp32 [128]
  const float* qk_cos;           // fp32 [qk_ntok, 64]
  const float* qk_sin;
  float qk_eps;
};

// ----------------------------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Blocking probe (the thread may be suspended for a while inside it): for waits off the MMA issue path.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe: returns at once (used where a wake-up delay would idle the tensor core).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false if the limit ran out (code recorded) or another role already aborted. The first probe is
// inlined; only a miss calls the out-of-line loop (a call on the MMA issue path costs ~270 cycles, and the
// tensor core's instruction queue is only ~2 MMAs deep, so every stall of the issuing thread idles it).
template <bool POLL>
__device__ __noinline__ bool mbar_wait_slow(uint32_t a, uint32_t parity, int* err, int code) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (POLL ? mbar_test(a, parity) : mbar_try(a, parity)) return true;
    if ((it & 1023) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if ((long long)(globaltimer() - t0) > kWaitLimitNs) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}
template <bool POLL>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t a = smem_u32(bar);
  if (POLL ? mbar_test(a, parity) : mbar_try(a, parity)) return true;
  return mbar_wait_slow<POLL>(a, parity, err, code);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// CTA-pair form: the transaction bytes land on the mbarrier at `bar` (a shared::cluster address, here the leader
// CTA's), while the data goes to this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows 128 B apart, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_sw128(const void* p) {
  const uint64_t a = smem_u32(p);
  return ((a & 0x3FFFFull) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptors (M = 128 per CTA of the group, N = 256, both operands K-major, fp32 accumulate).
//   block-scaled mxf4nvf4: A/B format E2M1 (1) at bits 7-9 / 10-12, scale format UE4M3 (0) at bit 23;
//   f8f6f4: D format F32 (1) at bits 4-5, A/B format E4M3 (0). M is encoded >> 4 at bits 24-28, N >> 3 at 17-22.
template <int CG>
struct Idesc {
  static constexpr uint32_t fp4 = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM * CG >> 4) << 24);
  static constexpr uint32_t fp8 = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM * CG >> 4) << 24);
};

template <int CG>
__device__ __forceinline__ void mma_fp4(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb, uint32_t acc) {
  if (CG == 2)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(Idesc<2>::fp4), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(Idesc<1>::fp4), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}
template <int CG>
__device__ __forceinline__ void mma_fp8(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
  if (CG == 2)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(Idesc<2>::fp8), "r"(acc)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(Idesc<1>::fp8), "r"(acc)
        : "memory");
}
// Commit of every tcgen05 op issued so far to an mbarrier at the same smem offset in each CTA of the group
// (tcgen05.commit multicast to the CTA pair: a signal, not a data load).
template <int CG>
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  if (CG == 2)
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t)3)
        : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Commit to this CTA's barrier only.
template <int CG>
__device__ __forceinline__ void tc_commit_local(uint32_t bar) {
  if (CG == 2)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Arrive on the leader CTA's mbarrier (a shared::cluster address) from the follower CTA of a pair. Relaxed: what
// the leader consumes after the wait is never ordinary memory published by this arrive -- it is this CTA's TMEM,
// whose tcgen05.st / tcgen05.ld traffic has completed (tcgen05.wait::st / ::ld) before the arrive and is ordered
// around it by tcgen05.fence::before_thread_sync here and ::after_thread_sync on the leader. A release at cluster
// scope made each arrive take ~0.7 us, which starved the MMA issue of the pair by ~40%.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

// fence::after_thread_sync + 4 MMAs + the commit that frees the stage's smem slot(s), as one asm statement.
template <int CG>
__device__ __forceinline__ void stage4_fp4(uint32_t d, uint64_t da, uint64_t db, uint32_t sf, uint32_t acc0,
                                           uint32_t empty_bar) {
  if (CG == 2)
    asm volatile(
        "{\n\t.reg .pred pa;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t.reg .b32 s1, s2, s3, t0, t1, t2, t3;\n\t"
        "setp.ne.b32 pa, %5, 0;\n\t"
        "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\t"
        "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\t"
        "add.u32 s1, %3, 4;\n\tadd.u32 s2, %3, 8;\n\tadd.u32 s3, %3, 12;\n\t"
        "add.u32 t0, %3, 16;\n\tadd.u32 t1, %3, 24;\n\tadd.u32 t2, %3, 32;\n\tadd.u32 t3, %3, 40;\n\t"
        "tcgen05.fence::after_thread_sync;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %6, [%3], [t0], pa;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], a1, b1, %6, [s1], [t1], 1;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], a2, b2, %6, [s2], [t2], 1;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], a3, b3, %6, [s3], [t3], 1;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%4], %7;\n\t}"
        ::"r"(d), "l"(da), "l"(db), "r"(sf), "r"(empty_bar), "r"(acc0), "r"(Idesc<2>::fp4), "h"((uint16_t)3)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred pa;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t.reg .b32 s1, s2, s3, t0, t1, t2, t3;\n\t"
        "setp.ne.b32 pa, %5, 0;\n\t"
        "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\t"
        "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\t"
        "add.u32 s1, %3, 4;\n\tadd.u32 s2, %3, 8;\n\tadd.u32 s3, %3, 12;\n\t"
        "add.u32 t0, %3, 16;\n\tadd.u32 t1, %3, 24;\n\tadd.u32 t2, %3, 32;\n\tadd.u32 t3, %3, 40;\n\t"
        "tcgen05.fence::after_thread_sync;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %6, [%3], [t0], pa;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], a1, b1, %6, [s1], [t1], 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], a2, b2, %6, [s2], [t2], 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], a3, b3, %6, [s3], [t3], 1;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%4];\n\t}"
        ::"r"(d), "l"(da), "l"(db), "r"(sf), "r"(empty_bar), "r"(acc0), "r"(Idesc<1>::fp4)
        : "memory");
}
template <int CG>
__device__ __forceinline__ void stage4_fp8(uint32_t d, uint64_t da, uint64_t db, uint32_t acc0, uint32_t empty_bar) {
  if (CG == 2)
    asm volatile(
        "{\n\t.reg .pred pa;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
        "setp.ne.b32 pa, %4, 0;\n\t"
        "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\t"
        "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\t"
        "tcgen05.fence::after_thread_sync;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %5, pa;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], a1, b1, %5, 1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], a2, b2, %5, 1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], a3, b3, %5, 1;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%3], %6;\n\t}"
        ::"r"(d), "l"(da), "l"(db), "r"(empty_bar), "r"(acc0), "r"(Idesc<2>::fp8), "h"((uint16_t)3)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred pa;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
        "setp.ne.b32 pa, %4, 0;\n\t"
        "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\t"
        "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\t"
        "tcgen05.fence::after_thread_sync;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %5, pa;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], a1, b1, %5, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], a2, b2, %5, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], a3, b3, %5, 1;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%3];\n\t}"
        ::"r"(d), "l"(da), "l"(db), "r"(empty_bar), "r"(acc0), "r"(Idesc<1>::fp8)
        : "memory");
}

// Warp-collective TMEM stores of this warp's 32 lanes: 4 and 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint4 v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, uint4 a, uint4 b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(a.x),
               "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

// Two 16-column pieces of this thread's TMEM lane (at taddr_a and taddr_b) with one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t taddr_a, uint32_t taddr_b, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr_a), "r"(taddr_b)
      : "memory");
}

// TMA tensor store of a 2-D box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// silu(g) = g / (1 + e^-g) with the hardware exp2 and reciprocal approximations (used by the SwiGLU GEMM epilogue;
// the caller rounds the result to bf16).
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }


// Output tile -> (M block, N block). Tiles go in bands of kBandM M blocks; inside a band the M block changes fastest,
// so the ~74-148 tiles in flight at once share a few B column blocks and all of the band's A rows. A band's A
// (16 x 256 rows) stays in L2 while the band walks every N block and B is read once per band; with the plain
// M-fastest order A was re-read from HBM once per N block when it did not fit in L2 (M = 131072: 13 GB per
// gate/up launch).
constexpr int kBandM = 16;
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int band_tiles = kBandM * num_n;
  const int band = tile / band_tiles;
  const int first = band * kBandM;
  const int gm = min(kBandM, num_m - first);
  const int idx = tile - band * band_tiles;
  mb = first + idx % gm;
  nb = idx / gm;
}

// MODE_FP4_TP: the chunks in the order rank+1, rank+2, ..., rank (this rank's own chunk last), each in the banded
// order above over its own M blocks. Every role of the kernel maps tiles through here.
template <int MODE>
__device__ __forceinline__ void map_tile(const Params& p, int tile, int& mb, int& nb) {
  if constexpr (MODE == MODE_FP4_TP) {
    int li = tile;
    for (int i = 1; i <= p.tp_world; ++i) {
      const int c = (p.tp_rank + i) % p.tp_world;
      const int mbc = max(0, min(p.tp_chunk_mb, p.num_m - c * p.tp_chunk_mb));
      if (li < mbc * p.num_n) {
        tile_coords(li, mbc, p.num_n, mb, nb);
        mb += c * p.tp_chunk_mb;
        return;
      }
      li -= mbc * p.num_n;
    }
    mb = nb = 0;   // not reached for tile < num_tiles
  } else {
    tile_coords(tile, p.num_m, p.num_n, mb, nb);
  }
}

// Cross-GPU counters (MODE_FP4_TP): system-scope acquire / release on a 32-bit counter in this GPU's or a peer's
// memory, and a bounded wait for a counter to reach `target` (modulo 2^32).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* a, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __noinline__ bool wait_counter(const uint32_t* a, uint32_t target, int* err, int code) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if ((int32_t)(ld_acquire_sys(a) - target) >= 0) return true;
    if ((it & 63) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if ((long long)(globaltimer() - t0) > kWaitLimitNs) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
    __nanosleep(100);
  }
}

// --------------------------------------------------------------------------------------------------- the kernel
// Pipeline depth per (mode, CTA group): an NVFP4 stage holds A 16 KB + B 16 KB per CTA of the group's B half
// (1 CTA: the whole 32 KB B tile) + 6 KB of scales; FP8 stages have no scales. All fit beside the 32 KB epilogue
// staging in the 227 KB of shared memory.
template <int MODE, int CG>
struct Cfg {
  static constexpr int B_BYTES_CTA = CG == 2 ? 128 * BKB : BN * BKB;
  static constexpr int SF_BYTES = MODE == 1 ? 0 : SFA_BYTES + SFB_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES_CTA + SF_BYTES;
  static constexpr int STAGES = CG == 2 ? 5 : 3;
  // FP8: each epilogue warp stages its 128 per-channel weight scales (512 B) before the accumulator is ready
  // QKV: the q and k RMSNorm weights (2 x 128 floats), staged once per launch
  static constexpr int SC_BYTES = MODE == 1 ? 8 * 128 * 4 : MODE == 5 ? 2 * 128 * 4 : 0;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + OUT_BYTES + SC_BYTES + 512;
};

template <int MODE, int CG>
__global__ void __launch_bounds__(kThreads<MODE>, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmY, const Params p) {
  using C = Cfg<MODE, CG>;
  constexpr bool FP4 = MODE != MODE_FP8;
  constexpr int STAGES = C::STAGES;
  constexpr int B_BYTES_CTA = C::B_BYTES_CTA;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES_CTA;
  uint8_t* sSFB = sSFA + (FP4 ? STAGES * SFA_BYTES : 0);
  uint8_t* sOut = sSFB + (FP4 ? STAGES * SFB_BYTES : 0);
  // full: the stage's loads landed -- one CTA: all of them; a pair: the leader's copy counts both CTAs' operand
  // tiles (each CTA's tensor loads complete on it), the follower's is unused
  float* sSC = reinterpret_cast<float*>(sOut + OUT_BYTES);   // FP8: output scales, 128 per epilogue warp;
                                                             // QKV: the q and k norm weights
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + OUT_BYTES + C::SC_BYTES);
  uint64_t* empty = full + STAGES;          // the stage's MMAs completed (commit from the group's MMA thread)
  uint64_t* sff = empty + STAGES;           // NVFP4: this CTA's scale bytes landed (its scale warps wait here)
  // FP8 has no scales in TMEM, so its accumulator is double-buffered (columns [0, 256) and [256, 512), tile t in
  // buffer t % 2): the next tile's MMAs run while the epilogue drains the previous tile
  constexpr int NACC = MODE == MODE_FP8 ? 2 : 1;
  uint64_t* acc_full = sff + STAGES;        // per accumulator buffer
  uint64_t* acc_empty = acc_full + 2;       // leader: every epilogue warp of the group drained the buffer
  uint64_t* drain = acc_empty + 2;
  uint64_t* xbar = drain + 1;               // resid: per epilogue warp, its residual box landed in its staging
  uint64_t* sigbar = xbar + 8;              // TP: every epilogue warp finished the tile's stores (ring of slots)
  uint64_t* ackbar = sigbar + kSigSlots;    // TP: the signal warp has signalled that slot's tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ackbar + kSigSlots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t rank = 0;                        // CTA rank inside the MMA group (0 = leader, issues the MMAs)
  if (CG == 2) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int grp = blockIdx.x / CG, ngrp = gridDim.x / CG;
  if (threadIdx.x == 0) {
    // the operand maps are kernel parameters, not outputs of the previous kernel: fetch them before pdl_wait
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    for (int s = 0; s < STAGES; ++s) {
      // leader: its producer's arrive (with the tile bytes of the group) + every scale warp of the group
      mbar_init(full + s, 1 + (FP4 ? 4 * CG : 0));
      mbar_init(empty + s, 1);
      mbar_init(sff + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 8 * CG);
    }
    mbar_init(drain, 1);
    for (int w = 0; w < 8; ++w) mbar_init(xbar + w, 1);
    for (int k = 0; k < kSigSlots; ++k) {
      mbar_init(sigbar + k, 8);
      mbar_init(ackbar + k, 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (CG == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if (CG == 2) {
    // barriers of both CTAs are initialised before either CTA signals the other
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  } else {
    __syncthreads();
  }
  tc_fence_after();
  // everything above (barriers, TMEM) overlapped the previous kernel's tail; its outputs are read only below
  pdl_trigger();
  pdl_wait();
  const uint32_t tmem = *tmem_slot;
  // the leader's copies of `full` and `acc_empty`, as shared::cluster addresses
  uint32_t acc_empty_l = smem_u32(acc_empty), full_l = smem_u32(full);
  if (CG == 2 && rank != 0) {
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(acc_empty_l) : "r"(acc_empty_l));
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(full_l) : "r"(full_l));
  }

  if (warp == 0) {
    if (lane == 0) {
      // ----------------------------------------------------------------------------------------- producer
      int stage = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;     // bit s: stage s was armed at least once
      uint32_t last_ph = 0;    // bit s: parity of its last arming
      bool ok = true;
      for (int tile = grp; ok && tile < p.num_tiles; tile += ngrp) {
        int mb, nb;
        map_tile<MODE>(p, tile, mb, nb);
        const int arow = mb * (BM * CG) + (int)rank * BM;             // this CTA's A rows
        int rb0, rb1;                                                  // the tile's two 128-row B groups
        if (MODE == MODE_FP4_SWIGLU) {
          rb0 = nb * 128;
          rb1 = p.N + nb * 128;
        } else {
          rb0 = nb * BN;
          rb1 = nb * BN + 128;
        }
        const int g0 = rb0 >> 7, g1 = rb1 >> 7, ga = arow >> 7;
        for (int ks = 0; ks < p.num_ks; ++ks) {
          if (!mbar_wait<false>(empty + stage, ph ^ 1, p.err, 0x101)) {
            ok = false;
            break;
          }
          uint32_t sf_bytes = 0, sf_tx = 0;
          if (FP4) {
            sf_bytes = min(4, p.kb_total - ks * 4) * 512;
            sf_tx = sf_bytes * ((ga < p.sfa_groups) + (g0 < p.sfb_groups) + (g1 < p.sfb_groups));
          }
          // scale copies complete on this CTA's `sff` (its scale warps wait there, then arrive on `full`)
          uint64_t* sf_bar = sff + stage;
          if (FP4) mbar_expect_tx(sff + stage, sf_tx);
          if (CG == 2) {
            // both CTAs' operand tiles complete on the leader's `full`, which the leader alone arms (tile loads
            // always count their whole box, rows past the tensor's end included)
            if (rank == 0) mbar_expect_tx(full + stage, 2 * (A_BYTES + B_BYTES_CTA));
            tma_load_2d_pair(sA + stage * A_BYTES, &tmA, full_l + stage * 8, ks * BKB, arow);
            tma_load_2d_pair(sB + stage * B_BYTES_CTA, &tmB, full_l + stage * 8, ks * BKB, rank == 0 ? rb0 : rb1);
          } else {
            mbar_expect_tx(full + stage, A_BYTES + B_BYTES_CTA);
            tma_load_2d(sA + stage * A_BYTES, &tmA, full + stage, ks * BKB, arow);
            tma_load_2d(sB + stage * B_BYTES_CTA, &tmB, full + stage, ks * BKB, rb0);
            tma_load_2d(sB + stage * B_BYTES_CTA + 128 * BKB, &tmB, full + stage, ks * BKB, rb1);
          }
          if (FP4) {
            const size_t chunk = (size_t)ks * 4;
            if (ga < p.sfa_groups)
              bulk_load(sSFA + stage * SFA_BYTES, p.sfa + ((size_t)ga * p.sf_chunks + chunk) * 512, sf_bytes, sf_bar);
            if (g0 < p.sfb_groups)
              bulk_load(sSFB + stage * SFB_BYTES, p.sfb + ((size_t)g0 * p.sf_chunks + chunk) * 512, sf_bytes, sf_bar);
            if (g1 < p.sfb_groups)
              bulk_load(sSFB + stage * SFB_BYTES + 2048, p.sfb + ((size_t)g1 * p.sf_chunks + chunk) * 512, sf_bytes,
                        sf_bar);
          }
          issued |= 1u << stage;
          last_ph = (last_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {  // let every copy already in flight land before the CTA exits
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            // `sff`: this CTA's scale copies; `full`: the tiles (of both CTAs in a pair; the follower cannot wait on
            // the leader's barrier and pauses instead, below). A `full` phase may also miss scale-warp arrivals
            // after an abort: its wait then runs to the limit.
            for (int b = 0; b < 2; ++b) {
              const uint64_t* bar = b == 0 ? full + s : sff + s;
              if ((b == 0 && CG == 2 && rank != 0) || (b == 1 && !FP4)) continue;
              const uint32_t a = smem_u32(bar);
              const unsigned long long t0 = globaltimer();
              while (!mbar_try(a, (last_ph >> s) & 1) && (long long)(globaltimer() - t0) < kWaitLimitNs) {
              }
            }
          }
        // a pair: tiles this CTA issued for a stage the leader never armed complete on no barrier either CTA
        // can wait for; a tile load lands within microseconds, so both CTAs stay for 100 us before leaving
        if (CG == 2) {
          const unsigned long long t0 = globaltimer();
          while ((long long)(globaltimer() - t0) < 100000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // --------------------------------------------------------------------------------------------- MMA
      // Lean on purpose: the tensor core's MMA queue is ~2 instructions deep, so every cycle the issuing thread
      // spends between stages is at risk of idling it. Descriptors advance arithmetically (start address >> 4).
      const uint64_t dA0 = desc_sw128(sA), dB0 = desc_sw128(sB);
      const uint32_t full0 = smem_u32(full), empty0 = smem_u32(empty);
      int stage = 0, acc_t = 0;                    // acc_t: this CTA's tiles so far
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = grp; ok && tile < p.num_tiles; tile += ngrp, ++acc_t) {
        const int ab = acc_t % NACC;
        const uint32_t acc_ph = (uint32_t)(acc_t / NACC) & 1;
        const uint32_t dacc = tmem + ACC_COL + ab * 256;
        if (!mbar_wait<true>(acc_empty + ab, acc_ph ^ 1, p.err, 0x201)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ks = 0; ks < p.num_ks; ++ks) {
          // one barrier: the stage's tiles (both CTAs' in a pair) and, NVFP4, every scale warp's TMEM writes
          const uint32_t fbar = full0 + stage * 8;
          if (!mbar_test(fbar, ph)) {
            if (!mbar_wait_slow<true>(fbar, ph, p.err, 0x202)) {
              ok = false;
              break;
            }
          }
          const uint64_t da = dA0 + (uint64_t)(stage * (A_BYTES >> 4));
          const uint64_t db = dB0 + (uint64_t)(stage * (B_BYTES_CTA >> 4));
          const uint32_t sft = tmem + SF_COL + stage * SF_STAGE_COLS;
          const int kb_here = min(4, p.kb_total - ks * 4);
          if (kb_here == 4) {
            if (FP4) stage4_fp4<CG>(dacc, da, db, sft, ks != 0, empty0 + stage * 8);
            else stage4_fp8<CG>(dacc, da, db, ks != 0, empty0 + stage * 8);
          } else {
            tc_fence_after();
            for (int kb = 0; kb < kb_here; ++kb) {
              const uint32_t acc = (ks | kb) != 0;
              if (FP4)
                mma_fp4<CG>(dacc, da + 2 * kb, db + 2 * kb, sft + kb * 4, sft + 16 + kb * 8, acc);
              else
                mma_fp8<CG>(dacc, da + 2 * kb, db + 2 * kb, acc);
            }
            tc_commit<CG>(empty0 + stage * 8);
          }
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit<CG>(smem_u32(acc_full + ab));
      }
      // drain: the commit arrives once every tcgen05 op this thread issued has completed
      tc_commit_local<CG>(smem_u32(drain));
      const uint32_t a = smem_u32(drain);
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(a, 0) && (long long)(globaltimer() - t0) < kWaitLimitNs) {
      }
    }
  } else if (warp < EPI_WARP0) {
    // ------------------------------------------------------------------------------------------ scale writers
    // Lane r of quadrant q writes TMEM lane 32q + r: for SFA the 16 bytes at r * 16 of each 512-byte chunk (rows
    // r, r+32, r+64, r+96 x 4 scales), for SFB the same from the tile's two 128-row B groups (8 columns). Every
    // quadrant holds the same values: the block-scaled MMA reads the copy of its own lane quadrant. With a CTA
    // pair each CTA writes its own A rows' scales and all 256 B columns' scales into its own TMEM. Then the warp
    // tells the group's MMA thread (on the leader) that this CTA's part of the stage is in place.
    const uint32_t q = warp & 3;
    const uint32_t tq = tmem + ((q * 32) << 16);
    int stage = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int tile = grp; FP4 && ok && tile < p.num_tiles; tile += ngrp) {
      for (int ks = 0; ks < p.num_ks; ++ks) {
        // the stage's scales landed; its TMEM scale buffer is free too: the producer re-armed the stage only after
        // the MMAs of its previous use completed
        if (!mbar_wait<false>(sff + stage, ph, p.err, 0x401)) {
          ok = false;
          break;
        }
        if (FP4) {
          const int kb_here = min(4, p.kb_total - ks * 4);
          const uint4* a4 = reinterpret_cast<const uint4*>(sSFA + stage * SFA_BYTES) + lane;
          const uint4* b4 = reinterpret_cast<const uint4*>(sSFB + stage * SFB_BYTES) + lane;
          // all shared-memory reads first: the TMEM stores below are asm with a memory clobber, and a read placed
          // after one of them would wait out its own latency before the next store
          uint4 va[4], vb0[4], vb1[4];
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            va[kb] = a4[kb * 32];
            vb0[kb] = b4[kb * 32];
            vb1[kb] = b4[128 + kb * 32];
          }
          const uint32_t col = SF_COL + stage * SF_STAGE_COLS;
          tc_fence_after();
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            if (kb < kb_here) {
              tmem_st4(tq + col + kb * 4, va[kb]);
              tmem_st8(tq + col + 16 + kb * 8, vb0[kb], vb1[kb]);
            }
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) {
          if (CG == 2 && rank != 0) mbar_arrive_cluster(full_l + stage * 8);   // the leader's barrier
          else mbar_arrive(full + stage);
        }
        if (++stage == STAGES) {
          stage = 0;
          ph ^= 1;
        }
      }
    }
  } else if (MODE == MODE_FP4_TP && warp == SIG_WARP) {
    // ------------------------------------------------------------------------------------------ signal (TP)
    // Per tile of this CTA, in the epilogue's order: wait until its 8 warps have issued every peer store of the
    // tile (their CTA-scope arrive orders those stores before this thread's system-scope release, which is
    // cumulative), then add 1 to the tile's counter on the receiving rank(s): the owner's partial counter for a
    // tile of another rank's chunk, every other rank's x counter for a tile of this rank's chunk.
    if (lane == 0) {
      int seq = 0;
      for (int tile = grp; tile < p.num_tiles; tile += ngrp, ++seq) {
        int mb, nb;
        map_tile<MODE>(p, tile, mb, nb);
        const int owner = mb / p.tp_chunk_mb;
        const int tc = (mb - owner * p.tp_chunk_mb) * p.num_n + nb;
        if (!mbar_wait<false>(sigbar + seq % kSigSlots, (seq / kSigSlots) & 1, p.err, 0x305)) break;
        // the release add is cumulative: the peer stores the epilogue warps issued before their arrive are visible
        // to whoever acquires the counter (a separate fence.sc.sys here cost ~10 us per launch)
        if (owner != p.tp_rank) {
          const int slot = (p.tp_rank - owner - 1 + p.tp_world) % p.tp_world;
          red_release_sys_add(reinterpret_cast<uint32_t*>(p.tp_base[owner] + p.tp_fp_off) +
                                  (int64_t)slot * p.tp_tiles_chunk + tc, 1u);
        } else {
          for (int qr = 1; qr < p.tp_world; ++qr)
            red_release_sys_add(reinterpret_cast<uint32_t*>(p.tp_base[(p.tp_rank + qr) % p.tp_world] + p.tp_fx_off) +
                                    (int64_t)p.tp_rank * p.tp_tiles_chunk + tc, 1u);
        }
        mbar_arrive(ackbar + seq % kSigSlots);
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - EPI_WARP0) >> 2;      // which half of the tile's columns this warp drains
    const int r = q * 32 + lane;                   // row inside this CTA's 128 rows == TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    uint8_t* stg = sOut + (warp - EPI_WARP0) * OUT_WARP_BYTES;   // this warp's 32 x 128-byte staging box
    int acc_t = 0;                                // this CTA's tiles so far (accumulator buffer and phase)
    uint64_t* xb = xbar + (warp - EPI_WARP0);
    uint32_t x_ph = 0, x_pending = 0;             // resid: parity of the next load; a load not yet waited for
    constexpr bool kResidMode = MODE == MODE_FP4_RESID || MODE == MODE_FP4_TP;
    // TP: the counter value this launch's tiles reach (the device epoch word was written by the previous kernel
    // of the stream, which completed before pdl_wait returned)
    const uint32_t tp_target = MODE == MODE_FP4_TP && p.tp_epoch_dev
                                   ? (uint32_t)CG * *reinterpret_cast<const volatile uint32_t*>(p.tp_epoch_dev)
                                   : p.tp_target;
    int sig_seq = 0;                              // TP: tiles handed to the signal warp so far
    // FP8: the activation scale (and a per-tensor weight scale) for the whole launch, written by earlier kernels
    const float fp8_scale =
        MODE == MODE_FP8 ? __ldg(p.a_scale) * (p.b_per_channel ? 1.0f : __ldg(p.b_scale)) : 0.0f;
    (void)fp8_scale;
    if constexpr (MODE == MODE_FP4_QKV) {
      // the q and k norm weights for every tile of the launch (the 8 epilogue warps fill them; named barrier 1)
      const int et = threadIdx.x - EPI_WARP0 * 32;
      sSC[et] = __ldg(p.qk_w[et >> 7] + (et & 127));
      asm volatile("bar.sync 1, 256;" ::: "memory");
    }
    auto sig_hand_off = [&]() {
      // slot reuse: the signal warp has finished the tile kSigSlots back
      if (sig_seq >= kSigSlots && lane == 0)
        mbar_wait<false>(ackbar + sig_seq % kSigSlots, (sig_seq / kSigSlots - 1) & 1, p.err, 0x306);
      __syncwarp();                               // every lane's peer stores before lane 0's arrive
      if (lane == 0) mbar_arrive(sigbar + sig_seq % kSigSlots);
      ++sig_seq;
    };
    for (int tile = grp; tile < p.num_tiles; tile += ngrp) {
      int mb, nb;
      map_tile<MODE>(p, tile, mb, nb);
      const int row0 = mb * (BM * CG) + (int)rank * BM;            // this CTA's first output row
      const int64_t m = (int64_t)row0 + r;
      const bool rows_live = row0 + q * 32 < p.M;
      // MODE_FP4_TP: the rank owning the tile's rows (its chunk) and the tile's index inside that chunk
      const int owner = MODE == MODE_FP4_TP ? mb / p.tp_chunk_mb : 0;
      const int tc = MODE == MODE_FP4_TP ? (mb - owner * p.tp_chunk_mb) * p.num_n + nb : 0;
      const bool resid_tile = MODE == MODE_FP4_RESID || (MODE == MODE_FP4_TP && owner == p.tp_rank);
      if (kResidMode && resid_tile && lane == 0 && rows_live && nb * BN + half * 128 < p.N) {
        // the first residual box does not depend on the accumulator: fetch it while the tile's MMAs run (the
        // staging box is free once the previous tile's last store has read it)
        tma_store_wait_read();
        mbar_expect_tx(xb, OUT_WARP_BYTES);
        tma_load_2d(stg, &tmY, xb, nb * BN + half * 128, row0 + q * 32);
        x_pending = 1;
      }
      float* wsc = sSC + (warp - EPI_WARP0) * 128;
      if constexpr (MODE == MODE_FP8) {
        // this tile's output scale of each of this warp's 128 columns, a * ws[n] (per-channel weight scales) or a * ws,
        // written while the MMAs run (zero past N); a per-element global load inside the drain held the accumulator
        // ~6 us per tile
        const int nc = nb * BN + half * 128 + lane * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          wsc[lane * 4 + k] = nc + k < p.N ? (p.b_per_channel ? fp8_scale * __ldg(p.b_scale + nc + k) : fp8_scale) : 0.0f;
        __syncwarp();
      }
      const int ab = acc_t % NACC;                 // this tile's accumulator buffer
      if (!mbar_wait<false>(acc_full + ab, (uint32_t)(acc_t / NACC) & 1, p.err, 0x301)) break;
      tc_fence_after();
      if (MODE == MODE_FP4_SWIGLU) {
        // this warp: hidden columns [half*64, half*64 + 64) of the tile = gate and up accumulator columns
        const int F = p.N;
        const int64_t col0 = (int64_t)nb * 128 + half * 64;
        // drain first, release, then compute: the accumulator goes to bf16 pairs (gate and up, 64 registers) and is
        // handed back to the MMA thread before the SwiGLU math, so the next tile's MMAs start after the TMEM reads
        // alone (the math, ~2 us of a tile, overlaps them)
        uint32_t hp[32], upk[32];                  // gate pairs, then h pairs in place; up pairs
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t raw[32];                        // [0, 16): gate, [16, 32): up -- 16 hidden columns
          tmem_ld16x2(trow + ACC_COL + half * 64 + c * 16, trow + ACC_COL + 128 + half * 64 + c * 16, raw);
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            // every bf16 rounding goes through the paired converter (one cvt.rn.bf16x2 per two values): single-
            // value conversions made this loop ~13 % of the whole GEMM's time, as much as the silu itself
            hp[c * 8 + j / 2] = pack_bf16x2(__uint_as_float(raw[j]) * p.alpha, __uint_as_float(raw[j + 1]) * p.alpha);
            upk[c * 8 + j / 2] =
                pack_bf16x2(__uint_as_float(raw[16 + j]) * p.alpha, __uint_as_float(raw[16 + j + 1]) * p.alpha);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {                           // drained: the next tile's MMAs may start
          if (CG == 2 && rank != 0) mbar_arrive_cluster(acc_empty_l + ab * 8);
          else mbar_arrive(acc_empty + ab);
        }
        if (p.gu_out && m < p.M) {                 // test-only output: the bf16 gate/up values the math used
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            __nv_bfloat16* dg = p.gu_out + m * 2 * F + col0 + 2 * i;
            *reinterpret_cast<uint32_t*>(dg) = hp[i];
            *reinterpret_cast<uint32_t*>(dg + F) = upk[i];
          }
        }
        // h = bf16(bf16(silu(g)) * u) with the hardware exp2 / reciprocal approximations for silu. Correct rounding
        // of silu (the standalone kernel's silu_for_bf16) was measured here at 1.25-1.5x the time of the whole
        // gate/up GEMM: this epilogue sits just under the mainloop's per-tile time, and with 2048 values per warp and
        // tile most warp-tiles meet a value near a bf16 midpoint whose fp64 recomputation then stalls the warp.
        // The fast form equals the correctly rounded silu except within a few fp32 ulp of a bf16 rounding midpoint:
        // none of the 35.7 M values of configs[1] differs (tests/test_gemm_gpu.py counts them).
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t gp = hp[i], up = upk[i];
          const uint32_t sp = pack_bf16x2(silu_fast(__uint_as_float(gp << 16)), silu_fast(__uint_as_float(gp & 0xFFFF0000u)));
          hp[i] = pack_bf16x2(__uint_as_float(sp << 16) * __uint_as_float(up << 16),
                              __uint_as_float(sp & 0xFFFF0000u) * __uint_as_float(up & 0xFFFF0000u));
        }
        if (lane == 0) tma_store_wait_read();      // the staging box is free once the previous store read it
        __syncwarp();
        if (m < p.M) {
          if (p.h_out) {
            uint4* dh = reinterpret_cast<uint4*>(p.h_out + m * F + col0);
#pragma unroll
            for (int v = 0; v < 8; ++v) dh[v] = make_uint4(hp[4 * v], hp[4 * v + 1], hp[4 * v + 2], hp[4 * v + 3]);
          }
          const Nvfp4Enc enc = nvfp4_enc(p.h_g);
          uint32_t cw[8], sfw = 0;
#pragma unroll
          for (int blk = 0; blk < 4; ++blk) {
            float h[16];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              h[2 * j] = __uint_as_float(hp[blk * 8 + j] << 16);
              h[2 * j + 1] = __uint_as_float(hp[blk * 8 + j] & 0xFFFF0000u);
            }
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(h[j]));
            const uint32_t sf = nvfp4_scale(amax, enc);
            const float inv = nvfp4_inv(sf, enc);
            cw[2 * blk] = nvfp4_codes8(h, inv);
            cw[2 * blk + 1] = nvfp4_codes8(h + 8, inv);
            sfw |= sf << (8 * blk);
          }
          uint4* dc = reinterpret_cast<uint4*>(stg + lane * 32);
          dc[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
          dc[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
          *reinterpret_cast<uint32_t*>(p.h_sf + sf_tiled_offset(m, col0 / 16, F / 64)) = sfw;
        } else if (m < (int64_t)p.sfa_groups * 128) {
          *reinterpret_cast<uint32_t*>(p.h_sf + sf_tiled_offset(m, col0 / 16, F / 64)) = 0u;
        }
        // 32 rows x 32 bytes of codes for this warp (rows past M are clipped by the tensor map)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0 && row0 + q * 32 < p.M) tma_store_2d(&tmY, stg, (int)(col0 / 2), row0 + q * 32);
      } else if constexpr (MODE == MODE_FP8) {
        // this warp: output columns [half*128, half*128 + 128) of the tile: all 128 drained to bf16 pairs (scaled
        // per tensor, or per channel from the scales staged above) and the accumulator released before the two
        // 64-column boxes go through the staging box to TMA stores
        const int n_base = nb * BN + half * 128;
        uint32_t pk[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t raw[32];
          const uint32_t t0 = trow + ACC_COL + ab * 256 + half * 128 + c * 32;
          tmem_ld16x2(t0, t0 + 16, raw);
          const float2* w = reinterpret_cast<const float2*>(wsc) + c * 16;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 w2 = w[j];
            pk[c * 16 + j] = pack_bf16x2(__uint_as_float(raw[2 * j]) * w2.x, __uint_as_float(raw[2 * j + 1]) * w2.y);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {                           // drained: the next tile's MMAs may start
          if (CG == 2 && rank != 0) mbar_arrive_cluster(acc_empty_l + ab * 8);
          else mbar_arrive(acc_empty + ab);
        }
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          if (lane == 0) tma_store_wait_read();    // the staging box is free once the previous store read it
          __syncwarp();
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                make_uint4(pk[bx * 32 + 4 * ch], pk[bx * 32 + 4 * ch + 1], pk[bx * 32 + 4 * ch + 2],
                           pk[bx * 32 + 4 * ch + 3]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0 && rows_live && n_base + bx * 64 < p.N) tma_store_2d(&tmY, stg, n_base + bx * 64, row0 + q * 32);
        }
      } else {
        // this warp: output columns [half*128, half*128 + 128) of the tile, drained 32 at a time
        const float scale = p.alpha;
        const int n_base = nb * BN + half * 128;
        uint32_t pk[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t raw[32];
          tmem_ld16x2(trow + ACC_COL + half * 128 + c * 32, trow + ACC_COL + half * 128 + c * 32 + 16, raw);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            pk[c * 16 + j] = pack_bf16x2(__uint_as_float(raw[2 * j]) * scale, __uint_as_float(raw[2 * j + 1]) * scale);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {                           // drained: the next tile's MMAs may start
          if (CG == 2 && rank != 0) mbar_arrive_cluster(acc_empty_l + ab * 8);
          else mbar_arrive(acc_empty + ab);
        }
        if constexpr (MODE == MODE_FP4_QKV) {
          // this warp's 128 columns are head `head` of part q / k / v; thread = one row of it
          const int HD = p.qk_heads * 128;
          const int part = n_base / HD, head = (n_base - part * HD) >> 7;
          const int grow0 = row0 + q * 32;                   // qk_ntok % 32 == 0: the 32 rows share a batch
          const int bb = grow0 / p.qk_ntok, n0 = grow0 - bb * p.qk_ntok;
          const bool norm = part < 2 && m < p.M;
          float rr = 0.0f;
          if (norm) {
            // RMSNorm statistics over the head row from the bf16 GEMM outputs (the reference's qkv tensor): 16
            // partial sums of 8, added in the butterfly order of the standalone kernel's 16-lane reduction
            float a8[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float x[8], y[8];
              unpack_bf16x8(make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]), x);
              unpack_bf16x8(make_uint4(pk[32 + 4 * j], pk[33 + 4 * j], pk[34 + 4 * j], pk[35 + 4 * j]), y);
              a8[j] = __fadd_rn(sumsq8(x), sumsq8(y));
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) a8[j] = __fadd_rn(a8[j], a8[j + 4]);
#pragma unroll
            for (int j = 0; j < 2; ++j) a8[j] = __fadd_rn(a8[j], a8[j + 2]);
            rr = rms_rr(__fadd_rn(a8[0], a8[1]), p.qk_eps);
          }
          __nv_bfloat16* dst = p.qk_dst[part] + (int64_t)bb * p.qk_sb[part] + (int64_t)head * 128;
          const float* w = sSC + (part == 1 ? 128 : 0);
          const int ck = lane & 7;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int jj = c * 8 + ck;             // this lane's 8 columns of the head: RoPE pairs jj*4 .. jj*4+3
            __syncwarp();
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                  make_uint4(pk[c * 32 + 4 * ch], pk[c * 32 + 4 * ch + 1], pk[c * 32 + 4 * ch + 2],
                             pk[c * 32 + 4 * ch + 3]);
            __syncwarp();
            // 4 rows x 128 B per pass: lane (r % 4) * 8 + ck takes chunk ck (8 values) of row r, so the row's cos /
            // sin (fp32, 64 per token) and the stores into the part's destination rows are both contiguous per 8
            // lanes; the row's RMS factor comes from the lane that summed it. The cos / sin of four passes are
            // loaded together, ahead of their math: token n0 + r < qk_ntok for every row of the warp, live or past
            // M (M = B * qk_ntok and qk_ntok % 32 == 0), so the loads need no row guard
#pragma unroll
            for (int g4 = 0; g4 < 2; ++g4) {
              float4 cq[4], sq[4];
              if (part < 2) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int64_t t = (int64_t)(n0 + (g4 * 4 + u) * 4 + (lane >> 3)) * 64 + jj * 4;
                  cq[u] = __ldg(reinterpret_cast<const float4*>(p.qk_cos + t));
                  sq[u] = __ldg(reinterpret_cast<const float4*>(p.qk_sin + t));
                }
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int r = (g4 * 4 + u) * 4 + (lane >> 3);
                const float rr_r = __shfl_sync(0xffffffffu, rr, r);
                const bool row_live = grow0 + r < p.M;
                uint4 o = *reinterpret_cast<const uint4*>(stg + r * 128 + ((ck ^ (r & 7)) << 4));
                if (part < 2 && row_live) {
                  float x[8];
                  unpack_bf16x8(o, x);
                  const float4 w0 = *reinterpret_cast<const float4*>(w + jj * 8);
                  const float4 w1 = *reinterpret_cast<const float4*>(w + jj * 8 + 4);
                  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                  const float cv[4] = {cq[u].x, cq[u].y, cq[u].z, cq[u].w};
                  const float sv[4] = {sq[u].x, sq[u].y, sq[u].z, sq[u].w};
                  o = norm_rope8(x, rr_r, wv, cv, sv);
                }
                if (row_live && n_base + c * 64 < p.N)
                  *reinterpret_cast<uint4*>(dst + (int64_t)(n0 + r) * p.qk_sn[part] + c * 64 + ck * 8) = o;
              }
            }
          }
          __syncwarp();
          ++acc_t;
          continue;
        }
        if constexpr (MODE == MODE_FP4_TP) {
          if (owner != p.tp_rank) {
            // another rank's rows: this rank's bf16 partial goes to the owner's receive slot for this sender,
            // through the staging box (swizzled like the TMA boxes) and coalesced 16-byte peer stores
            const int slot = (p.tp_rank - owner - 1 + p.tp_world) % p.tp_world;
            uint8_t* dst = p.tp_base[owner] + p.tp_r_off;
            const int64_t lrow = (int64_t)slot * p.tp_chunk_rows + (row0 + q * 32 - owner * p.tp_chunk_rows);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int col0 = n_base + c * 64;
              if (lane == 0) tma_store_wait_read();
              __syncwarp();
#pragma unroll
              for (int ch = 0; ch < 8; ++ch)
                *reinterpret_cast<uint4*>(stg + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                    make_uint4(pk[c * 32 + 4 * ch], pk[c * 32 + 4 * ch + 1], pk[c * 32 + 4 * ch + 2],
                               pk[c * 32 + 4 * ch + 3]);
              __syncwarp();
#pragma unroll
              for (int i = 0; i < 8; ++i) {          // 4 rows x 128 bytes per pass
                const int rr = i * 4 + (lane >> 3), ck = lane & 7;
                if (row0 + q * 32 + rr < p.M && col0 + ck * 8 < p.N)
                  *reinterpret_cast<uint4*>(dst + ((lrow + rr) * p.N + col0 + ck * 8) * 2) =
                      *reinterpret_cast<const uint4*>(stg + rr * 128 + ((ck ^ (rr & 7)) << 4));
              }
              // these generic reads of the box come before any later async-proxy write to it (a TMA load)
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              __syncwarp();
            }
            sig_hand_off();                        // the signal warp tells the owner
            ++acc_t;
            continue;
          }
          // this rank's rows: every other rank's partial of the tile has arrived in this rank's receive slots
          if (lane == 0)
            for (int s = 0; s + 1 < p.tp_world; ++s)
              wait_counter(reinterpret_cast<const uint32_t*>(p.tp_base[p.tp_rank] + p.tp_fp_off) +
                               (int64_t)s * p.tp_tiles_chunk + tc, tp_target, p.err, 0x303);
          __syncwarp();
        }
        // two 64-column boxes through the 128-byte-swizzled staging buffer and TMA stores (coalesced, async,
        // clipped at the M / N edges); the buffer is reused once the previous store has read it
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const bool live = n_base + c * 64 < p.N && rows_live;
          if (kResidMode) {
            if (!live) continue;
            if constexpr (MODE == MODE_FP4_TP) {
              // y = bf16(sum of every rank's bf16 partial of this row, in rank order, in fp32), into pk; the loads
              // of the whole box are independent of each other and of any store, so they are all in flight at once
              const int64_t lr0 = m - (int64_t)p.tp_rank * p.tp_chunk_rows;   // row inside this rank's chunk
              const uint8_t* rv = p.tp_base[p.tp_rank] + p.tp_r_off + (lr0 * p.N + n_base + c * 64) * 2;
              const int64_t slot_bytes = (int64_t)p.tp_chunk_rows * p.N * 2;
              if (p.tp_world == 2) {
                uint4 v[8];
#pragma unroll
                for (int ch = 0; ch < 8; ++ch)
                  v[ch] = m < p.M && n_base + c * 64 + ch * 8 < p.N
                              ? __ldcg(reinterpret_cast<const uint4*>(rv) + ch) : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                  const uint32_t pv[4] = {v[ch].x, v[ch].y, v[ch].z, v[ch].w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    uint32_t& own = pk[c * 32 + 4 * ch + j];
                    const float o_lo = __uint_as_float(own << 16), o_hi = __uint_as_float(own & 0xFFFF0000u);
                    const float r_lo = __uint_as_float(pv[j] << 16), r_hi = __uint_as_float(pv[j] & 0xFFFF0000u);
                    own = p.tp_rank == 0 ? pack_bf16x2(o_lo + r_lo, o_hi + r_hi) : pack_bf16x2(r_lo + o_lo, r_hi + o_hi);
                  }
                }
              } else {
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                  float lo[4] = {0.f, 0.f, 0.f, 0.f}, hi[4] = {0.f, 0.f, 0.f, 0.f};
                  for (int qr = 0; qr < p.tp_world; ++qr) {
                    uint4 v = make_uint4(pk[c * 32 + 4 * ch], pk[c * 32 + 4 * ch + 1], pk[c * 32 + 4 * ch + 2],
                                         pk[c * 32 + 4 * ch + 3]);
                    if (qr != p.tp_rank) {
                      const int sl = (qr - p.tp_rank - 1 + p.tp_world) % p.tp_world;
                      v = m < p.M && n_base + c * 64 + ch * 8 < p.N
                              ? __ldcg(reinterpret_cast<const uint4*>(rv + sl * slot_bytes) + ch)
                              : make_uint4(0, 0, 0, 0);
                    }
                    const uint32_t vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                      lo[j] += __uint_as_float(vs[j] << 16);
                      hi[j] += __uint_as_float(vs[j] & 0xFFFF0000u);
                    }
                  }
#pragma unroll
                  for (int j = 0; j < 4; ++j) pk[c * 32 + 4 * ch + j] = pack_bf16x2(lo[j], hi[j]);
                }
              }
            }
            if (c == 1 && lane == 0) {               // second box: after the first one's store has read the box
              tma_store_wait_read();
              mbar_expect_tx(xb, OUT_WARP_BYTES);
              tma_load_2d(stg, &tmY, xb, n_base + 64, row0 + q * 32);
            }
            __syncwarp();
            // the load always lands (in-bounds tensor map); a wait that still runs out records its code
            mbar_wait<false>(xb, x_ph, p.err, 0x302);
            x_ph ^= 1;
            x_pending = 0;
            const int64_t grow = m < p.M ? m / p.rows_per_gate : 0;
            const uint4* gp = reinterpret_cast<const uint4*>(p.gate + grow * p.ld_gate + n_base + c * 64);
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              uint4* px = reinterpret_cast<uint4*>(stg + lane * 128 + ((ch ^ (lane & 7)) << 4));
              const uint4 xv = *px, gv = __ldg(gp + ch);
              const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, gs[4] = {gv.x, gv.y, gv.z, gv.w};
              uint32_t o[4];
              uint32_t y2[4] = {pk[c * 32 + 4 * ch], pk[c * 32 + 4 * ch + 1], pk[c * 32 + 4 * ch + 2],
                                pk[c * 32 + 4 * ch + 3]};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t a2 = y2[j];
                const float lo = fmaf(__uint_as_float(a2 << 16), __uint_as_float(gs[j] << 16),
                                      __uint_as_float(xs[j] << 16));
                const float hi = fmaf(__uint_as_float(a2 & 0xFFFF0000u), __uint_as_float(gs[j] & 0xFFFF0000u),
                                      __uint_as_float(xs[j] & 0xFFFF0000u));
                o[j] = pack_bf16x2(lo, hi);
              }
              *px = make_uint4(o[0], o[1], o[2], o[3]);
            }
          } else {
            if (lane == 0) tma_store_wait_read();
            __syncwarp();
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                  make_uint4(pk[c * 32 + 4 * ch], pk[c * 32 + 4 * ch + 1], pk[c * 32 + 4 * ch + 2],
                             pk[c * 32 + 4 * ch + 3]);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0 && live) tma_store_2d(&tmY, stg, n_base + c * 64, row0 + q * 32);
          if constexpr (MODE == MODE_FP4_TP) {
            // the new x rows also go to every other rank's copy of x (coalesced 16-byte peer stores from the box;
            // the TMA store above only reads it too)
            const int col0 = n_base + c * 64;
            for (int qr = 1; qr < p.tp_world; ++qr) {
              uint8_t* dst = p.tp_base[(p.tp_rank + qr) % p.tp_world];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int rr = i * 4 + (lane >> 3), ck = lane & 7;
                if (row0 + q * 32 + rr < p.M && col0 + ck * 8 < p.N)
                  *reinterpret_cast<uint4*>(dst + ((int64_t)(row0 + q * 32 + rr) * p.N + col0 + ck * 8) * 2) =
                      *reinterpret_cast<const uint4*>(stg + rr * 128 + ((ck ^ (rr & 7)) << 4));
              }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
          }
        }
        if constexpr (MODE == MODE_FP4_TP) sig_hand_off();   // own tile: the signal warp tells every other rank
      }
      ++acc_t;
    }
    if (kResidMode && x_pending) {     // left the loop with a residual box still in flight
      const uint32_t a = smem_u32(xb);
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(a, x_ph) && (long long)(globaltimer() - t0) < kWaitLimitNs) {
      }
    }
    if (lane == 0) tma_store_wait_all();
  }

  tc_fence_before();
  if (CG == 2) {
    // neither CTA releases TMEM or exits while the other may still signal it
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

template <int MODE, int CG>
tfb_status launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ty, const Params& p,
                  cudaStream_t s) {
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads<MODE>);
  cfg.dynamicSmemBytes = Cfg<MODE, CG>::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // pdl_trigger / pdl_wait in the kernel
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = CG;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = CG == 2 ? 2 : 1;
  // Persistent grid: as many groups as can be resident at once. A CTA pair must sit inside one GPC, so on parts
  // whose GPCs hold an odd number of usable SMs fewer than sm_count / 2 pairs fit; a larger grid would run its
  // extra pairs as a second wave after the first ones finished all their tiles.
  // (set-up calls from several host threads may race; they store the same value)
  static std::atomic<int> resident[64];
  int res = resident[di->device].load(std::memory_order_acquire);
  if (!res) {
    TFB_CUDA(cudaFuncSetAttribute(gemm_kernel<MODE, CG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Cfg<MODE, CG>::SMEM));
    int n = di->sm_count;
    if (CG == 2) {
      cfg.gridDim = dim3(di->sm_count);
      TFB_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_kernel<MODE, CG>, &cfg));
      if (n <= 0) return fail(TFB_CUDA_ERR, "gemm: no CTA pair of this kernel fits on the device");
    }
    res = min(n, di->sm_count / CG);
    resident[di->device].store(res, std::memory_order_release);
  }
  const int groups = min(p.num_tiles, res);
  if (groups == 0) return TFB_OK;
  cfg.gridDim = dim3(groups * CG);
  TFB_CUDA(cudaLaunchKernelEx(&cfg, gemm_kernel<MODE, CG>, ta, tb, ty, p));
  return TFB_OK;
}

tfb_status check_common(int64_t M, int64_t N, int64_t K, const char* who) {
  if (M < 0 || N <= 0 || K <= 0 || K % 128 || N % 32)
    return fail(TFB_BAD_SHAPE, "%s: need K %% 128 == 0 and N %% 32 == 0 (M=%lld N=%lld K=%lld)", who, (long long)M,
                (long long)N, (long long)K);
  if (M > (int64_t)1 << 30 || N > (int64_t)1 << 30 || K > (int64_t)1 << 30)
    return fail(TFB_BAD_SHAPE, "%s: dimension too large", who);
  return TFB_OK;
}

// CTAs per MMA group: pairs (cta_group::2, 256-row tiles) unless M fits one 128-row tile or TFB_CTA_GROUP=1.
int cta_group(int64_t M) {
  static const int forced = [] {   // read once (a function-local static is initialised thread-safely)
    const char* e = getenv("TFB_CTA_GROUP");
    return e ? atoi(e) : 0;
  }();
  return (forced == 1 || M <= BM) ? 1 : 2;
}

void fill_tiles(Params& p, int cg, int64_t M, int64_t ncols_per_tile, int64_t N) {
  p.num_m = (int)((M + BM * cg - 1) / (BM * cg));
  p.num_n = (int)((N + ncols_per_tile - 1) / ncols_per_tile);
  p.num_tiles = p.num_m * p.num_n;
  p.sfa_groups = (int)((M + BM - 1) / BM);
}

template <int MODE>
tfb_status dispatch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ty, Params& p, int64_t M,
                    int64_t ncols_per_tile, int64_t N, cudaStream_t s) {
  const int cg = cta_group(M);
  fill_tiles(p, cg, M, ncols_per_tile, N);
  return cg == 2 ? launch<MODE, 2>(ta, tb, ty, p, s) : launch<MODE, 1>(ta, tb, ty, p, s);
}

}  // namespace

tfb_status gemm_nvfp4(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, int64_t M,
                      int64_t N, int64_t K, float alpha, void* y, int64_t ldy, cudaStream_t s) {
  tfb_status st = check_common(M, N, K, "gemm_nvfp4");
  if (st != TFB_OK) return st;
  if (ldy < N || ldy % 8 || !aligned(y, 16) || !aligned(a_sf, 16) || !aligned(b_sf, 16))
    return fail(TFB_BAD_ALIGN, "gemm_nvfp4: y/ldy need 16-byte alignment, scales 16-byte aligned");
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  if (M == 0) return TFB_OK;
  CUtensorMap ta, tb;
  if ((st = make_tmap_u8(&ta, a, K / 2, M, K / 2, BKB, BM)) != TFB_OK) return st;
  if ((st = make_tmap_u8(&tb, b, K / 2, N, K / 2, BKB, 128)) != TFB_OK) return st;
  CUtensorMap ty;
  if ((st = make_tmap_2d(&ty, y, 2, N, M, ldy * 2, 64, 32, true)) != TFB_OK) return st;
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.num_ks = (int)(K / 256 + (K % 256 ? 1 : 0));
  p.kb_total = (int)(K / 64);
  p.b_rows = (int)N;
  p.sfa = a_sf;
  p.sfb = b_sf;
  p.sf_chunks = (int)(K / 64);
  p.sfb_groups = (int)((N + 127) / 128);
  p.y = y;
  p.ldy = ldy;
  p.alpha = alpha;
  p.err = di->err_word;
  return dispatch<MODE_FP4>(ta, tb, ty, p, M, BN, N, s);
}

tfb_status gemm_nvfp4_resid(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, int64_t M,
                            int64_t N, int64_t K, float alpha, void* x, int64_t ldx, const void* gate,
                            int64_t ld_gate, int64_t rows_per_gate, cudaStream_t s) {
  tfb_status st = check_common(M, N, K, "gemm_nvfp4_resid");
  if (st != TFB_OK) return st;
  if (ldx < N || ldx % 8 || !aligned(x, 16) || !aligned(a_sf, 16) || !aligned(b_sf, 16))
    return fail(TFB_BAD_ALIGN, "gemm_nvfp4_resid: x/ldx need 16-byte alignment, scales 16-byte aligned");
  if (!gate || !aligned(gate, 16) || ld_gate < N || ld_gate % 8 || rows_per_gate < 1)
    return fail(TFB_BAD_ARG, "gemm_nvfp4_resid: gate must be 16-byte aligned bf16 rows (ld_gate >= N, %% 8 == 0) "
                "and rows_per_gate >= 1");
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  if (M == 0) return TFB_OK;
  CUtensorMap ta, tb, ty;
  if ((st = make_tmap_u8(&ta, a, K / 2, M, K / 2, BKB, BM)) != TFB_OK) return st;
  if ((st = make_tmap_u8(&tb, b, K / 2, N, K / 2, BKB, 128)) != TFB_OK) return st;
  if ((st = make_tmap_2d(&ty, x, 2, N, M, ldx * 2, 64, 32, true)) != TFB_OK) return st;
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.num_ks = (int)(K / 256 + (K % 256 ? 1 : 0));
  p.kb_total = (int)(K / 64);
  p.b_rows = (int)N;
  p.sfa = a_sf;
  p.sfb = b_sf;
  p.sf_chunks = (int)(K / 64);
  p.sfb_groups = (int)((N + 127) / 128);
  p.y = x;
  p.ldy = ldx;
  p.alpha = alpha;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.ld_gate = ld_gate;
  p.rows_per_gate = rows_per_gate;
  p.err = di->err_word;
  return dispatch<MODE_FP4_RESID>(ta, tb, ty, p, M, BN, N, s);
}

// ------------------------------------------------------------------- tensor-parallel down projection (MODE_FP4_TP)
namespace {

int64_t tp_round256(int64_t v) { return (v + 255) / 256 * 256; }

// Rows of each rank's chunk: M / world rounded up to whole 256-row pair tiles, so no tile straddles two owners.
int64_t tp_chunk_rows(int world, int64_t rows) { return ((rows + world - 1) / world + 255) / 256 * 256; }

struct TpLayout {
  int64_t chunk_rows, tiles_chunk, x, recv, fp, fx, epoch, bytes;
};

// One rank's communication buffer: x [max_rows, n_cols] bf16 (the replicated residual stream), world-1 receive
// slots [chunk_rows, n_cols] bf16, then the per-tile counters: partials received [world-1][tiles_chunk] and x rows
// received [world][tiles_chunk] (u32). Counter slots per chunk cover the 128-row single-CTA tiling too.
TpLayout tp_layout(int world, int64_t max_rows, int64_t n_cols) {
  TpLayout L{};
  L.chunk_rows = tp_chunk_rows(world, max_rows);
  L.tiles_chunk = (L.chunk_rows / BM) * ((n_cols + BN - 1) / BN);
  L.x = 0;   // the kernel addresses every rank's x at its buffer's base
  L.recv = tp_round256(max_rows * n_cols * 2);
  L.fp = L.recv + tp_round256((int64_t)(world - 1) * L.chunk_rows * n_cols * 2);
  L.fx = L.fp + tp_round256((int64_t)(world - 1) * L.tiles_chunk * 4);
  L.epoch = L.fx + tp_round256((int64_t)world * L.tiles_chunk * 4);   // this rank's device epoch word
  L.bytes = L.epoch + 256;
  return L;
}

tfb_status tp_check(const tfb_tp_comm* c, int64_t M, int64_t N, uint32_t epoch, const char* who) {
  if (!c || c->world < 2 || c->world > TFB_TP_MAX_WORLD || c->rank < 0 || c->rank >= c->world)
    return fail(TFB_BAD_ARG, "%s: communicator needs 2 <= world <= %d and 0 <= rank < world", who, TFB_TP_MAX_WORLD);
  for (int q = 0; q < c->world; ++q)
    if (!c->base[q] || !aligned(c->base[q], 256))
      return fail(TFB_BAD_ARG, "%s: rank %d's buffer is missing or not 256-byte aligned", who, q);
  if (M <= 0 || M > c->max_rows || N != c->n_cols)
    return fail(TFB_BAD_SHAPE, "%s: M=%lld N=%lld outside the buffer's %lld x %lld", who, (long long)M, (long long)N,
                (long long)c->max_rows, (long long)c->n_cols);
  if (epoch >= (1u << 27)) return fail(TFB_BAD_ARG, "%s: epoch must be 0 (device epoch) or in [1, 2^27)", who);
  return TFB_OK;
}

// Waits (bounded) until every tile of every other rank's chunk has its x rows in this rank's x.
__global__ void __launch_bounds__(256) tp_wait_kernel(const uint32_t* fx, int world, int rank, int chunk_mb,
                                                      int num_m, int num_n, int tiles_chunk, uint32_t target,
                                                      const uint32_t* epoch_dev, uint32_t cg, int* err) {
  pdl_trigger();
  pdl_wait();
  if (epoch_dev) target = cg * *reinterpret_cast<const volatile uint32_t*>(epoch_dev);
  for (int c = 0; c < world; ++c) {
    if (c == rank) continue;
    const int mbc = max(0, min(chunk_mb, num_m - c * chunk_mb));
    for (int t = threadIdx.x; t < mbc * num_n; t += blockDim.x)
      if (!wait_counter(fx + (int64_t)c * tiles_chunk + t, target, err, 0x304)) return;
  }
}

// One thread: this rank's device epoch word += 1 (after the previous kernel of the stream completed).
__global__ void tp_advance_kernel(uint32_t* epoch) {
  pdl_trigger();
  pdl_wait();
  *epoch += 1u;
}

}  // namespace

tfb_status tp_advance(const tfb_tp_comm* comm, cudaStream_t s) {
  if (!comm || comm->world < 2 || comm->world > TFB_TP_MAX_WORLD || comm->rank < 0 || comm->rank >= comm->world ||
      !comm->base[comm->rank])
    return fail(TFB_BAD_ARG, "tp_advance: bad communicator");
  const TpLayout L = tp_layout(comm->world, comm->max_rows, comm->n_cols);
  TFB_LAUNCH(tp_advance_kernel, 1, 1, s, reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(comm->base[comm->rank]) + L.epoch));
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

tfb_status gemm_nvfp4_tp(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, int64_t M,
                         int64_t N, int64_t K, float alpha, const void* gate, int64_t ld_gate, int64_t rows_per_gate,
                         const tfb_tp_comm* comm, uint32_t epoch, cudaStream_t s) {
  tfb_status st = check_common(M, N, K, "gemm_nvfp4_tp");
  if (st != TFB_OK) return st;
  if ((st = tp_check(comm, M, N, epoch, "gemm_nvfp4_tp")) != TFB_OK) return st;
  if (N % 8 || !aligned(a_sf, 16) || !aligned(b_sf, 16))
    return fail(TFB_BAD_ALIGN, "gemm_nvfp4_tp: N %% 8 == 0 and 16-byte aligned scales needed");
  if (!gate || !aligned(gate, 16) || ld_gate < N || ld_gate % 8 || rows_per_gate < 1)
    return fail(TFB_BAD_ARG, "gemm_nvfp4_tp: gate must be 16-byte aligned bf16 rows (ld_gate >= N, %% 8 == 0) "
                "and rows_per_gate >= 1");
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  const TpLayout L = tp_layout(comm->world, comm->max_rows, comm->n_cols);
  uint8_t* x = static_cast<uint8_t*>(comm->base[comm->rank]) + L.x;
  CUtensorMap ta, tb, ty;
  if ((st = make_tmap_u8(&ta, a, K / 2, M, K / 2, BKB, BM)) != TFB_OK) return st;
  if ((st = make_tmap_u8(&tb, b, K / 2, N, K / 2, BKB, 128)) != TFB_OK) return st;
  if ((st = make_tmap_2d(&ty, x, 2, N, M, N * 2, 64, 32, true)) != TFB_OK) return st;
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.num_ks = (int)(K / 256 + (K % 256 ? 1 : 0));
  p.kb_total = (int)(K / 64);
  p.b_rows = (int)N;
  p.sfa = a_sf;
  p.sfb = b_sf;
  p.sf_chunks = (int)(K / 64);
  p.sfb_groups = (int)((N + 127) / 128);
  p.y = x;
  p.ldy = N;
  p.alpha = alpha;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.ld_gate = ld_gate;
  p.rows_per_gate = rows_per_gate;
  p.err = di->err_word;
  const int cg = cta_group(M);
  p.tp_world = comm->world;
  p.tp_rank = comm->rank;
  p.tp_chunk_rows = (int)tp_chunk_rows(comm->world, M);
  p.tp_chunk_mb = p.tp_chunk_rows / (BM * cg);
  p.tp_tiles_chunk = (int)L.tiles_chunk;
  p.tp_target = (uint32_t)cg * epoch;   // one add per CTA of the tile's group
  p.tp_epoch_dev = epoch == 0 ? reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(comm->base[comm->rank]) + L.epoch)
                              : nullptr;
  for (int q = 0; q < comm->world; ++q) p.tp_base[q] = static_cast<uint8_t*>(comm->base[q]);
  p.tp_r_off = L.recv;
  p.tp_fp_off = L.fp;
  p.tp_fx_off = L.fx;
  return dispatch<MODE_FP4_TP>(ta, tb, ty, p, M, BN, N, s);
}

tfb_status tp_wait(const tfb_tp_comm* comm, int64_t M, int64_t N, uint32_t epoch, cudaStream_t s) {
  tfb_status st = tp_check(comm, M, N, epoch, "tp_wait");
  if (st != TFB_OK) return st;
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  const TpLayout L = tp_layout(comm->world, comm->max_rows, comm->n_cols);
  const int cg = cta_group(M);
  const int chunk_mb = (int)(tp_chunk_rows(comm->world, M) / (BM * cg));
  const int num_m = (int)((M + BM * cg - 1) / (BM * cg)), num_n = (int)((N + BN - 1) / BN);
  const uint32_t* fx = reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(comm->base[comm->rank]) + L.fx);
  const uint32_t* ep =
      epoch == 0 ? reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(comm->base[comm->rank]) + L.epoch) : nullptr;
  TFB_LAUNCH(tp_wait_kernel, 1, 256, s, fx, comm->world, comm->rank, chunk_mb, num_m, num_n, (int)L.tiles_chunk,
             (uint32_t)cg * epoch, ep, (uint32_t)cg, di->err_word);
  TFB_CUDA(cudaGetLastError());
  return TFB_OK;
}

tfb_status gemm_nvfp4_qkv(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, int64_t B,
                          int64_t ntok, int64_t H, int64_t K, float alpha, const float* wq, const float* wk,
                          const float* cosp, const float* sinp, float eps, void* const dst[3], const int64_t sb[3],
                          const int64_t sn[3], cudaStream_t s) {
  const int64_t M = B * ntok, N = 3 * H * 128;
  tfb_status st = check_common(M, N, K, "gemm_nvfp4_qkv");
  if (st != TFB_OK) return st;
  if (B < 0 || ntok <= 0 || ntok % 32 || H <= 0)
    return fail(TFB_BAD_SHAPE, "gemm_nvfp4_qkv: need ntok %% 32 == 0 and H > 0 (B=%lld ntok=%lld H=%lld)",
                (long long)B, (long long)ntok, (long long)H);
  if (!wq || !wk || !cosp || !sinp || !aligned(wq, 16) || !aligned(wk, 16) || !aligned(cosp, 16) || !aligned(sinp, 16) ||
      !aligned(a_sf, 16) || !aligned(b_sf, 16))
    return fail(TFB_BAD_ALIGN, "gemm_nvfp4_qkv: weights, cos/sin tables and scales must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (!dst[i] || !aligned(dst[i], 16) || sb[i] % 8 || sn[i] % 8 || sn[i] < H * 128)
      return fail(TFB_BAD_ALIGN, "gemm_nvfp4_qkv: destination %d needs 16-byte alignment, strides %% 8 == 0 and a row "
                  "stride >= H * 128", i);
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  if (M == 0) return TFB_OK;
  CUtensorMap ta, tb, ty;
  if ((st = make_tmap_u8(&ta, a, K / 2, M, K / 2, BKB, BM)) != TFB_OK) return st;
  if ((st = make_tmap_u8(&tb, b, K / 2, N, K / 2, BKB, 128)) != TFB_OK) return st;
  // (the epilogue stores through its own row addressing; this map is a placeholder over the q destination)
  if ((st = make_tmap_2d(&ty, dst[0], 2, H * 128, ntok, sn[0] * 2, 64, 32, true)) != TFB_OK) return st;
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.num_ks = (int)(K / 256 + (K % 256 ? 1 : 0));
  p.kb_total = (int)(K / 64);
  p.b_rows = (int)N;
  p.sfa = a_sf;
  p.sfb = b_sf;
  p.sf_chunks = (int)(K / 64);
  p.sfb_groups = (int)((N + 127) / 128);
  p.alpha = alpha;
  p.err = di->err_word;
  p.qk_heads = (int)H;
  p.qk_ntok = (int)ntok;
  for (int i = 0; i < 3; ++i) {
    p.qk_dst[i] = static_cast<__nv_bfloat16*>(dst[i]);
    p.qk_sb[i] = sb[i];
    p.qk_sn[i] = sn[i];
  }
  p.qk_w[0] = wq;
  p.qk_w[1] = wk;
  p.qk_cos = cosp;
  p.qk_sin = sinp;
  p.qk_eps = eps;
  return dispatch<MODE_FP4_QKV>(ta, tb, ty, p, M, BN, N, s);
}

tfb_status gemm_nvfp4_swiglu(const uint8_t* a, const uint8_t* a_sf, const uint8_t* gu, const uint8_t* gu_sf, int64_t M,
                             int64_t F, int64_t K, float alpha, float h_g, uint8_t* h_codes, uint8_t* h_sf,
                             void* gu_out, void* h_out, cudaStream_t s) {
  tfb_status st = check_common(M, F, K, "gemm_nvfp4_swiglu");
  if (st != TFB_OK) return st;
  if (F % 128) return fail(TFB_BAD_SHAPE, "gemm_nvfp4_swiglu: F=%lld must be a multiple of 128", (long long)F);
  if (!(h_g > 0.0f) || !isfinite(h_g)) return fail(TFB_BAD_ARG, "gemm_nvfp4_swiglu: h_global must be positive");
  if (!aligned(h_codes, 16) || !aligned(h_sf, 16) || !aligned(a_sf, 16) || !aligned(gu_sf, 16) ||
      (gu_out && !aligned(gu_out, 16)) || (h_out && !aligned(h_out, 16)))
    return fail(TFB_BAD_ALIGN, "gemm_nvfp4_swiglu: outputs and scales must be 16-byte aligned");
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  if (M == 0) return TFB_OK;
  CUtensorMap ta, tb;
  if ((st = make_tmap_u8(&ta, a, K / 2, M, K / 2, BKB, BM)) != TFB_OK) return st;
  if ((st = make_tmap_u8(&tb, gu, K / 2, 2 * F, K / 2, BKB, 128)) != TFB_OK) return st;
  Params p{};
  p.M = (int)M;
  p.N = (int)F;
  p.num_ks = (int)(K / 256 + (K % 256 ? 1 : 0));
  p.kb_total = (int)(K / 64);
  p.b_rows = (int)(2 * F);
  p.sfa = a_sf;
  p.sfb = gu_sf;
  p.sf_chunks = (int)(K / 64);
  p.sfb_groups = (int)((2 * F + 127) / 128);
  p.alpha = alpha;
  p.h_g = h_g;
  p.h_codes = h_codes;
  p.h_sf = h_sf;
  p.gu_out = static_cast<__nv_bfloat16*>(gu_out);
  p.h_out = static_cast<__nv_bfloat16*>(h_out);
  p.err = di->err_word;
  CUtensorMap th;                                      // h codes: 32-byte x 32-row boxes, one per epilogue warp
  if ((st = make_tmap_2d(&th, h_codes, 1, F / 2, M, F / 2, 32, 32, false)) != TFB_OK) return st;
  return dispatch<MODE_FP4_SWIGLU>(ta, tb, th, p, M, 128, F, s);
}

// FP8 takes the reference's FP8 envelope (tfimage/linear.py:159: K % 16 == 0, N % 16 == 0): the last K stage and
// the last MMA k-block may be partly past K, and the last tile's B rows past N; TMA fills both with zeros, which add
// nothing to the accumulator, and the output tensor map clips the stores at N.
tfb_status gemm_fp8(const uint8_t* a, const uint8_t* b, int64_t M, int64_t N, int64_t K, const float* a_scale,
                    const float* b_scale, int per_channel, void* y, int64_t ldy, cudaStream_t s) {
  if (M < 0 || N <= 0 || K <= 0 || K % 16 || N % 16)
    return fail(TFB_BAD_SHAPE, "gemm_fp8: need K %% 16 == 0 and N %% 16 == 0 (M=%lld N=%lld K=%lld)", (long long)M,
                (long long)N, (long long)K);
  if (M > (int64_t)1 << 30 || N > (int64_t)1 << 30 || K > (int64_t)1 << 30)
    return fail(TFB_BAD_SHAPE, "gemm_fp8: dimension too large");
  tfb_status st = TFB_OK;
  if (ldy < N || ldy % 8 || !aligned(y, 16) || !aligned(a_scale, 4) || !aligned(b_scale, 4))
    return fail(TFB_BAD_ALIGN, "gemm_fp8: y/ldy need 16-byte alignment");
  const DeviceInfo* di;
  if ((st = device_info(&di)) != TFB_OK) return st;
  if (M == 0) return TFB_OK;
  CUtensorMap ta, tb;
  if ((st = make_tmap_u8(&ta, a, K, M, K, BKB, BM)) != TFB_OK) return st;
  if ((st = make_tmap_u8(&tb, b, K, N, K, BKB, 128)) != TFB_OK) return st;
  CUtensorMap ty;
  if ((st = make_tmap_2d(&ty, y, 2, N, M, ldy * 2, 64, 32, true)) != TFB_OK) return st;
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.num_ks = (int)((K + 127) / 128);
  p.kb_total = (int)((K + 31) / 32);
  p.b_rows = (int)N;
  p.y = y;
  p.ldy = ldy;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.b_per_channel = per_channel;
  p.err = di->err_word;
  return dispatch<MODE_FP8>(ta, tb, ty, p, M, BN, N, s);
}

}  // namespace tfb

extern "C" {

tfb_status tfb_gemm_nvfp4(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes, const uint8_t* b_sf,
                          int64_t M, int64_t N, int64_t K, float alpha, void* y, int64_t ldy, void* stream) {
  return tfb::gemm_nvfp4(a_codes, a_sf, b_codes, b_sf, M, N, K, alpha, y, ldy, static_cast<cudaStream_t>(stream));
}

tfb_status tfb_gemm_nvfp4_resid(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes,
                                const uint8_t* b_sf, int64_t M, int64_t N, int64_t K, float alpha, void* x,
                                int64_t ldx, const void* gate, int64_t ld_gate, int64_t rows_per_gate, void* stream) {
  return tfb::gemm_nvfp4_resid(a_codes, a_sf, b_codes, b_sf, M, N, K, alpha, x, ldx, gate, ld_gate, rows_per_gate,
                               static_cast<cudaStream_t>(stream));
}

int64_t tfb_tp_layout(int world, int64_t max_rows, int64_t n_cols, int64_t* offsets) {
  if (world < 2 || world > TFB_TP_MAX_WORLD || max_rows <= 0 || n_cols <= 0 || n_cols % 32) return -1;
  const tfb::TpLayout L = tfb::tp_layout(world, max_rows, n_cols);
  if (offsets) {
    offsets[0] = L.x;
    offsets[1] = L.recv;
    offsets[2] = L.fp;
    offsets[3] = L.fx;
    offsets[4] = L.epoch;
  }
  return L.bytes;
}

tfb_status tfb_tp_advance(const tfb_tp_comm* comm, void* stream) {
  return tfb::tp_advance(comm, static_cast<cudaStream_t>(stream));
}

tfb_status tfb_gemm_nvfp4_tp(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes, const uint8_t* b_sf,
                             int64_t M, int64_t N, int64_t K, float alpha, const void* gate, int64_t ld_gate,
                             int64_t rows_per_gate, const tfb_tp_comm* comm, uint32_t epoch, void* stream) {
  return tfb::gemm_nvfp4_tp(a_codes, a_sf, b_codes, b_sf, M, N, K, alpha, gate, ld_gate, rows_per_gate, comm, epoch,
                            static_cast<cudaStream_t>(stream));
}

tfb_status tfb_tp_wait(const tfb_tp_comm* comm, int64_t M, int64_t N, uint32_t epoch, void* stream) {
  return tfb::tp_wait(comm, M, N, epoch, static_cast<cudaStream_t>(stream));
}

tfb_status tfb_gemm_nvfp4_qkv(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* b_codes,
                              const uint8_t* b_sf, int64_t B, int64_t ntok, int64_t H, int64_t K, float alpha,
                              const float* wq, const float* wk, const float* cos, const float* sin, float eps, void* q,
                              int64_t q_sb, int64_t q_sn, void* k, int64_t k_sb, int64_t k_sn, void* v, int64_t v_sb,
                              int64_t v_sn, void* stream) {
  void* const dst[3] = {q, k, v};
  const int64_t sb[3] = {q_sb, k_sb, v_sb}, sn[3] = {q_sn, k_sn, v_sn};
  return tfb::gemm_nvfp4_qkv(a_codes, a_sf, b_codes, b_sf, B, ntok, H, K, alpha, wq, wk, cos, sin, eps, dst, sb, sn,
                             static_cast<cudaStream_t>(stream));
}

tfb_status tfb_gemm_fp8(const uint8_t* a, const uint8_t* b, int64_t M, int64_t N, int64_t K, const float* a_scale,
                        const float* b_scale, int b_per_channel, void* y, int64_t ldy, void* stream) {
  return tfb::gemm_fp8(a, b, M, N, K, a_scale, b_scale, b_per_channel, y, ldy, static_cast<cudaStream_t>(stream));
}

tfb_status tfb_gemm_nvfp4_swiglu(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* gu_codes,
                                 const uint8_t* gu_sf, int64_t M, int64_t F, int64_t K, float alpha, float h_global,
                                 uint8_t* h_codes, uint8_t* h_sf, void* gu_out, void* h_out, void* stream) {
  return tfb::gemm_nvfp4_swiglu(a_codes, a_sf, gu_codes, gu_sf, M, F, K, alpha, h_global, h_codes, h_sf, gu_out, h_out,
                                static_cast<cudaStream_t>(stream));
}

tfb_status tfb_mlp_nvfp4(const void* x, int64_t M, int64_t K, int64_t F, float act_x, const uint8_t* gu_codes,
                         const uint8_t* gu_sf, float g_gu, const uint8_t* down_codes, const uint8_t* down_sf,
                         float g_down, float act_h, void* y, uint8_t* ws_xc, uint8_t* ws_xsf, uint8_t* ws_hc,
                         uint8_t* ws_hsf, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  tfb_status st = tfb::quant_nvfp4(x, M, K, K, act_x, ws_xc, ws_xsf, TFB_SF_TILED, s);
  if (st != TFB_OK) return st;
  st = tfb::gemm_nvfp4_swiglu(ws_xc, ws_xsf, gu_codes, gu_sf, M, F, K, (float)((double)act_x * g_gu), act_h, ws_hc,
                              ws_hsf, nullptr, nullptr, s);
  if (st != TFB_OK) return st;
  return tfb::gemm_nvfp4(ws_hc, ws_hsf, down_codes, down_sf, M, K, F, (float)((double)act_h * g_down), y, K, s);
}

}  // extern "C"

// ------------------------------------------------------------------------ fused MLP pair on static device scratch
// tfb_mlp_nvfp4_static's scratch: one array per device (every context that loads the library gets its own copy),
// carved per call into x codes | x scales | h codes | h scales at 256-byte boundaries.
static __device__ __align__(256) uint8_t g_mlp_static_scratch[TFB_MLP_STATIC_SCRATCH_BYTES];

namespace tfb {
namespace {

std::atomic<uint8_t*> g_mlp_scratch_addr[64];
std::mutex g_mlp_scratch_mu;

// The device address of the current device's copy of the array, looked up once per device (with that device
// current, as cudaGetSymbolAddress requires) and cached.
tfb_status mlp_static_scratch(uint8_t** out) {
  const DeviceInfo* di;
  tfb_status st = device_info(&di);
  if (st != TFB_OK) return st;
  uint8_t* p = g_mlp_scratch_addr[di->device].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(g_mlp_scratch_mu);
    p = g_mlp_scratch_addr[di->device].load(std::memory_order_relaxed);
    if (!p) {
      void* a = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&a, g_mlp_static_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (tfb_mlp_nvfp4_static scratch)");
      if (!a || !aligned(a, 256)) return fail(TFB_CUDA_ERR, "tfb_mlp_nvfp4_static: scratch address unusable");
      p = static_cast<uint8_t*>(a);
      g_mlp_scratch_addr[di->device].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return TFB_OK;
}

constexpr int64_t round256(int64_t n) { return (n + 255) / 256 * 256; }

}  // namespace
}  // namespace tfb

extern "C" tfb_status tfb_mlp_nvfp4_static(const void* x, int64_t M, int64_t K, int64_t F, float act_x,
                                           const uint8_t* gu_codes, const uint8_t* gu_sf, float g_gu,
                                           const uint8_t* down_codes, const uint8_t* down_sf, float g_down,
                                           float act_h, void* y, void* stream) {
  constexpr int64_t kDimMax = (int64_t)1 << 30;
  if (M < 0 || K <= 0 || F <= 0 || K % 64 || F % 64 || M > kDimMax || K > kDimMax || F > kDimMax)
    return tfb::fail(TFB_BAD_SHAPE, "tfb_mlp_nvfp4_static: bad shape M=%lld K=%lld F=%lld", (long long)M,
                     (long long)K, (long long)F);
  const int64_t o_xsf = tfb::round256(M * (K / 2));
  const int64_t o_hc = o_xsf + tfb::round256(tfb_sf_tiled_bytes(M, K));
  const int64_t o_hsf = o_hc + tfb::round256(M * (F / 2));
  const int64_t need = o_hsf + tfb_sf_tiled_bytes(M, F);
  if (need > TFB_MLP_STATIC_SCRATCH_BYTES)
    return tfb::fail(TFB_BAD_SHAPE,
                     "tfb_mlp_nvfp4_static: M=%lld K=%lld F=%lld needs %lld bytes of scratch, more than the "
                     "%lld-byte static array; split M across calls or use tfb_mlp_nvfp4 with a workspace",
                     (long long)M, (long long)K, (long long)F, (long long)need, (long long)TFB_MLP_STATIC_SCRATCH_BYTES);
  uint8_t* base = nullptr;
  const tfb_status st = tfb::mlp_static_scratch(&base);
  if (st != TFB_OK) return st;
  return tfb_mlp_nvfp4(x, M, K, F, act_x, gu_codes, gu_sf, g_gu, down_codes, down_sf, g_down, act_h, y, base,
                       base + o_xsf, base + o_hc, base + o_hsf, stream);
}
