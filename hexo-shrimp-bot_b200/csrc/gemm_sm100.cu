// Fused row GEMM on the 5th-generation tensor cores (sm_100a tcgen05):
//
//     out = epilogue( prologue(x) @ W^T + bias )
//
//   prologue: LN      - fp32 rows -> LayerNorm (fp32 statistics) -> bf16
//             COPY    - bf16 rows used as they are
//             TMA     - bf16 rows loaded by the tensor memory accelerator, one
//                       128-row x 64-column K-block per copy, already in the
//                       MMA's swizzled layout, into a ring of K-block slots
//             HEXMEAN - mean of the bf16 rows of a node's present hex
//                       neighbours (six-slot int32 table, -1 = absent; fp32
//                       sum, zero when none is present) -> bf16
//   epilogue: STORE    - bf16 rows (optionally ReLU, optionally plus an fp32
//                        addend row)
//             RESIDUAL - x_res[row] += result (fp32, in place)
//             ADD_X    - out[row] = x[row] + result (bf16), the fused
//                        message-passing update y = x + W mean(x[nbr]) + b
//             RESID_LN - RESIDUAL, then up to three LayerNorms of each
//                        updated row (bf16 outputs), from the same launch
//             HEAD     - a decoder head's last two layers: per row
//                        out[j] = b_out[j] + w_out[j] . relu(result +
//                        tok[tok_idx[row]]), up to four outputs (fp32)
//
// K = 256 or 512 (the A tile is held whole in shared memory), N any multiple
// of 128: a tile's N blocks (256 columns, the last one 128 when N is an odd
// multiple of 128) run back to back on the same A tile; M any.
// The op is HBM-bound (about 1.5-4 KB of row traffic per 131 kFLOP), so the
// design is about keeping row bytes in flight and accesses coalesced.
//
// Persistent, warp-specialised CTA (one per SM, 16 warps = 4 per SM
// sub-partition, so every thread may hold 128 registers):
//   warp 0      lane 0 streams pre-swizzled 64-wide K-blocks of W (32 KB,
//               L2-resident) through a 1- or 2-stage ring with cp.async.bulk
//               and issues the tcgen05.mma stream (M=128, N=256 or 128, K=16,
//               bf16 x bf16 -> fp32) into a double-buffered TMEM accumulator
//               (one buffer per (tile, N block) work item), signalling with
//               tcgen05.commit.
//   warps 1-7   A producers (11 for the neighbour gather), three variants:
//               staged (LayerNorm of contiguous fp32 rows): lane 1 of warp 0
//                 bulk-copies 32-row groups (32 KB) into a 3-deep ring; warps
//                 1-7 normalise rows out of shared memory into the A tile;
//               copy (bf16 rows): every lane cp.asyncs its 16-byte chunk of
//                 each of its warp's rows straight into the swizzled slot, so
//                 the whole 64 KB tile is in flight at once;
//               direct (strided fp32 rows, neighbour means): 16-byte vector
//                 loads, several rows in flight per warp.
//               The A tile is bf16 in the 128-byte-swizzled K-major layout the
//               UMMA descriptor reads.
//   warps 8-15  epilogue: two warps per TMEM lane quadrant, one per 128-column
//               half; tcgen05.ld 32 columns at a time (thread = row). A bf16
//               result is stored directly. The residual variants stream the
//               residual rows through a per-warp cp.async ring of 32 x 32
//               boxes and write back whole row segments; the LayerNorm variant
//               keeps the updated rows in TMEM for its statistics and output
//               passes (see the epilogue).
//
// Every mbarrier wait is bounded by a clock deadline; on expiry the CTA
// records a device error, stops issuing work, and still frees its TMEM.
#include <cuda.h>  // CUtensorMap and its encoding enums (the encoder is fetched through the runtime)

#include "common.cuh"

namespace mb {
namespace sm100 {

constexpr int BM = 128, BN = 256, BK = 64, KDIM = 256;
constexpr int A_KB_BYTES = BM * BK * 2;            // 16 KB per K-block
constexpr int W_KB_BYTES = BN * BK * 2;            // 32 KB per K-block
constexpr int XG_ROWS = 32;                        // rows per staged group
constexpr int XG_BYTES = XG_ROWS * KDIM * 4;       // 32 KB of fp32 rows
constexpr int X_STAGES = 3;
constexpr int TMEM_COLS = 512;                     // 2 accumulators of 256 columns
constexpr int EPILOGUE = 8;
constexpr int THREADS = 32 * 16;
constexpr int RB = 8;                              // rows in flight per direct producer warp
constexpr int BOX_FLOATS = 32 * 32;
constexpr int OUT_BOX_BYTES = 32 * 32 * 2;          // 32 rows x 32 bf16 LayerNorm outputs
constexpr int BAR_BYTES = 512;
constexpr int A_RING = 8;                          // A K-block slots of the tensor-map prologue
constexpr long long kWaitCycles = 4000000000LL;   // ~2 s at 1.9 GHz

enum Prologue { PRO_LN = 0, PRO_COPY = 1, PRO_HEXMEAN = 2, PRO_TMA = 3 };
enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_ADD_X = 2, EPI_RESID_LN = 3, EPI_HEAD = 4 };
constexpr int MAX_LN = 3;
constexpr int MAX_HEAD_OUT = 4;
constexpr int HEX_SLOTS = 6;

constexpr uint32_t ERR_TIMEOUT = 4;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and a recorded device error) when the deadline passes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      report(ERR_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Tensor-map load of one (64-column, 128-row) box of a 2-D bf16 tensor into
// shared memory (128-byte swizzle), completing on `bar`. Rows past the
// tensor's end read as zero. x (the column) is a multiple of 64.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 16-byte cp.async (L2 only) that zero-fills the destination when `live` is
// false, and the group commit / wait that orders a warp's boxes.
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool live) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(live ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Tensor-map store of one 32-column x 32-row bf16 box (64-byte swizzle) from
// shared memory; rows past the tensor's end are not written.
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor: K-major operand, 128-byte swizzle, 8-row
// core-matrix groups 1024 bytes apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t make_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.st of 32 consecutive columns of this thread's TMEM lane (the
// counterpart of tmem_ld32), and the wait that orders it before later loads.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

struct alignas(64) Params {
  CUtensorMap tmap_x;   // PRO_TMA: the (m, K) bf16 input rows, 64 x 128 boxes, 128-byte swizzle
  CUtensorMap tmap_out; // EPI_STORE: the (m, N) bf16 output rows, 32 x 32 boxes, 64-byte swizzle
  const void* x;        // prologue input rows (fp32 for LN, bf16 for COPY)
  int64_t ldx;
  const float* gamma;   // LN
  const float* beta;
  float eps;
  const __nv_bfloat16* w_img;  // pre-swizzled weight image, KBLOCKS x (BN x 128 B)
  const float* bias;    // may be null
  int64_t m;
  int relu;
  __nv_bfloat16* out;   // EPI_STORE
  int64_t ldo;
  float* res;           // EPI_RESIDUAL
  int64_t ldr;
  const int32_t* nbr;   // PRO_HEXMEAN: (m, 6) neighbour rows of x, -1 = absent
  // EPI_RESID_LN: up to three LayerNorms of the updated residual row
  int n_ln;
  float ln_eps;
  const float* ln_g[MAX_LN];
  const float* ln_b[MAX_LN];
  void* ln_out[MAX_LN];
  int ln_dtype[MAX_LN];
  int64_t ln_ld[MAX_LN];
  // N blocks per tile (256 columns each, 128 for the K = 512 weight-
  // stationary plan; the last one n_last = 128 or 256)
  int n_blocks;
  int n_last;
  // the weight image's own 256-row blocks (w_blocks, the last w_last rows)
  int w_blocks;
  int w_last;
  // EPI_STORE: optional fp32 addend rows (add + row * ld_add + column)
  const float* add;
  int64_t ld_add;
  // EPI_HEAD: per-row second operand tok[tok_idx[row]] (bf16 rows), the
  // output layer w_out (n_out x N fp32, row-major), b_out, fp32 outputs
  const __nv_bfloat16* tok;
  int64_t ld_tok;
  int64_t n_tok;
  const int64_t* tok_idx;
  const float* w_out;
  const float* b_out;
  int n_out;
  float* head_out;
  int64_t ld_head;
};

// Shared-memory plan of one variant (all region offsets 1024-byte aligned).
template <int PRO, int EPI, bool XS, int KB, bool WS>
struct Plan {
  // The residual epilogues stream the residual through a shared-memory ring,
  // which takes the second A buffer's space (the epilogue, not the MMA,
  // bounds these variants). A K = 512 tile (128 KB) is single-buffered.
  static constexpr bool RESID = EPI == EPI_RESIDUAL || EPI == EPI_RESID_LN;
  static_assert(KB == 4 || KB == 8, "K must be 256 or 512");
  static_assert(KB == 4 || ((PRO == PRO_COPY || PRO == PRO_TMA) && EPI != EPI_RESID_LN), "K = 512 takes bf16 rows");
  static constexpr int A_BYTES = BM * BK * 2 * KB;
  // Weight-stationary plan (WS): the CTA holds one whole N block of W (K =
  // 256: 128 KB) and runs every one of its row tiles against it before the
  // next N block, so W crosses from L2 once per CTA and N block instead of
  // once per tile; its A tiles are re-read for each N block.
  static_assert(!WS || (!RESID && !XS && (PRO == PRO_TMA || (PRO == PRO_LN && KB == 4))),
                "the weight-stationary plan serves bf16-output launches");
  // K = 512 keeps a 128-column N block stationary (128 KB of W) and streams
  // its A K-blocks through a four-slot ring.
  static constexpr bool HALF = WS && KB == 8;
  static constexpr int BNB = HALF ? 128 : BN;       // columns per N block
  static constexpr int WKB = BNB * BK * 2;          // bytes per stationary W K-block
  // The neighbour-mean prologue keeps one tile and one W stage so that the
  // L1 cache keeps most of the SM's 256 KB: a tile's neighbour rows (its own
  // rows +- 64) are then gathered from L1 after their first touch.
  static constexpr bool L1_HEAVY = PRO == PRO_HEXMEAN;
  static constexpr int A_BUFS = (XS || RESID || KB > 4 || WS || L1_HEAVY) ? 1 : 2;
  // PRO_TMA keeps K-block slots in a ring instead of whole tiles: a slot is
  // refilled as soon as the MMAs that read it finish.
  static constexpr bool RING_A = PRO == PRO_TMA;
  static constexpr int A_SLOTS = RING_A ? (RESID ? KB : (WS ? (HALF ? 4 : KB) : A_RING)) : 0;
  static_assert(!RING_A || A_SLOTS >= KB || HALF, "a tile's K-blocks must fit the ring");
  static constexpr int A_SPACE = RING_A ? A_SLOTS * A_KB_BYTES : A_BUFS * A_BYTES;
  // bf16-output epilogues stage 32 x 32 boxes for whole-segment stores
  static constexpr bool OUT_BOXES = EPI == EPI_RESID_LN || EPI == EPI_STORE || EPI == EPI_ADD_X;
  // W K-blocks in flight. The residual epilogues are long enough to hide a
  // one-stage W stream; the freed 32 KB hold the output staging boxes.
  static constexpr int W_STAGES = (RESID || L1_HEAVY) ? 1 : 2;
  // Residual boxes (32 rows x 32 fp32 columns, 4 KB) per epilogue warp.
  static constexpr int RING = KB > 4 ? 1 : 3;
  // Warps writing the A tile (1..PRODUCERS) and draining TMEM (the rest).
  // The neighbour-gather prologue is latency-bound, so it gets more warps and
  // the epilogue four (one per TMEM lane quadrant, all 256 columns each).
  static constexpr int PRODUCERS = PRO == PRO_HEXMEAN ? 11 : 7;  // idle under PRO_TMA
  static constexpr int EPI_WARPS = 16 - 1 - PRODUCERS;
  static constexpr int A_OFF = 0;
  static constexpr int W_OFF = A_OFF + A_SPACE;
  static constexpr int X_OFF = W_OFF + (WS ? KB * WKB : W_STAGES * W_KB_BYTES);
  // staged LayerNorm rows: 32-row groups in flight (two when the output boxes
  // need the space)
  static constexpr int XSTAGES = OUT_BOXES ? 2 : X_STAGES;
  static constexpr int E_OFF = X_OFF + (XS ? XSTAGES * XG_BYTES : 0);
  static constexpr int OUT_OFF = E_OFF + (RESID ? EPILOGUE * RING * BOX_FLOATS * 4 : 0);
  // bias and the LayerNorms' gamma / beta, copied once per CTA (uniform
  // reads in the epilogue, kept out of the busy L1 miss path)
  // EPI_STORE writes its boxes with tensor-map stores: two boxes per warp
  // where they fit, so a box is refilled while the other one's store reads it
  static constexpr int OUT_NBOX =
      (EPI == EPI_STORE && OUT_OFF + 2 * EPILOGUE * OUT_BOX_BYTES + BAR_BYTES + 1024 <= 232448) ? 2 : 1;
  static constexpr int PAR_OFF = OUT_OFF + (OUT_BOXES ? EPILOGUE * OUT_BOX_BYTES * OUT_NBOX : 0);
  static constexpr int RED_OFF = PAR_OFF + (RESID ? (1 + 2 * MAX_LN) * BN * 4 : 0);
  static constexpr int BAR_OFF = RED_OFF + (EPI == EPI_RESID_LN ? 4 * 64 * 4 : 0) +
                                 (EPI == EPI_HEAD ? 4 * MAX_HEAD_OUT * 32 * 4 : 0);
  static constexpr int SMEM = BAR_OFF + BAR_BYTES + 1024 /*alignment slack*/;
  static_assert(SMEM <= 232448, "shared memory plan exceeds 227 KB");
  static_assert(PRO != PRO_TMA || EPI != EPI_RESID_LN, "the LayerNorm epilogue keeps its cp.async producers");
};

template <int PRO, int EPI, bool XS, int KB = 4, bool WS = false>
__global__ void __launch_bounds__(THREADS, 1) rowgemm_kernel(const __grid_constant__ Params p) {
  using L = Plan<PRO, EPI, XS, KB, WS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_smem = smem + L::A_OFF;
  uint8_t* w_smem = smem + L::W_OFF;
  uint8_t* x_smem = smem + L::X_OFF;
  float* e_smem = reinterpret_cast<float*>(smem + L::E_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* a_full = bars;            // [A_RING]: tiles (2) or K-block slots
  uint64_t* a_empty = bars + 8;       // [A_RING]
  uint64_t* w_full = bars + 16;       // [2]
  uint64_t* w_empty = bars + 18;      // [2]
  uint64_t* t_full = bars + 20;       // [2]
  uint64_t* t_empty = bars + 22;      // [2]
  uint64_t* x_full = bars + 24;       // [3]
  uint64_t* x_empty = bars + 27;      // [3]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 30);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 31);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_tiles = (p.m + BM - 1) / BM;
  const int nbn = p.n_blocks;
  // Tile groups: without WS a CTA takes tiles blockIdx.x + k * gridDim.x and
  // runs all N blocks of each. With WS the grid is n_blocks CTAs per group:
  // CTA b holds N block b % n_blocks of W and takes the tiles of group
  // b / n_blocks, so the CTAs of one group read the same A tiles at about
  // the same time and every A tile but the first read of it comes from L2.
  const int64_t grp = WS ? blockIdx.x / nbn : blockIdx.x;
  const int64_t gstride = WS ? gridDim.x / nbn : gridDim.x;
  const int ws_nb = WS ? (int)(blockIdx.x % nbn) : 0;
  const int64_t my_tiles = n_tiles > grp ? (n_tiles - 1 - grp) / gstride + 1 : 0;
  // A units: the A tiles the producers write, in MMA order: one per tile
  // (shared by its N blocks without WS: work items t * n_blocks + nb).
  const int64_t n_units = my_tiles;
  auto unit_tile = [&](int64_t u) -> int64_t { return u; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < A_RING; ++i) {
      mbar_init(smem_u32(&a_full[i]), L::RING_A ? 1 : L::PRODUCERS);
      mbar_init(smem_u32(&a_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&w_full[i]), 1);
      mbar_init(smem_u32(&w_empty[i]), 1);
      mbar_init(smem_u32(&t_full[i]), 1);
      mbar_init(smem_u32(&t_empty[i]), L::EPI_WARPS);
    }
    for (int i = 0; i < L::XSTAGES; ++i) {
      mbar_init(smem_u32(&x_full[i]), 1);
      mbar_init(smem_u32(&x_empty[i]), L::PRODUCERS);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  float* par = reinterpret_cast<float*>(smem + L::PAR_OFF);  // [bias | g0 b0 | g1 b1 | g2 b2] x BN
  if constexpr (L::RESID) {
    if (threadIdx.x < BN) {
      const int c = threadIdx.x;
      par[c] = p.bias ? p.bias[c] : 0.f;
#pragma unroll
      for (int o = 0; o < MAX_LN; ++o) {
        par[(1 + 2 * o) * BN + c] = o < p.n_ln ? p.ln_g[o][c] : 0.f;
        par[(2 + 2 * o) * BN + c] = o < p.n_ln ? p.ln_b[o][c] : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------- W stream + MMA issuer (1 lane)
    if (lane == 0) {
      const int64_t total_kb = WS ? 0 : (int64_t)my_tiles * nbn * KB;
      const uint8_t* wimg = reinterpret_cast<const uint8_t*>(p.w_img);
      uint64_t issued = 0;
      auto issue_w = [&](uint64_t upto) -> bool {
        for (; (int64_t)issued < total_kb && issued < upto; ++issued) {
          const uint32_t s = issued % L::W_STAGES, ph = (issued / L::W_STAGES) & 1;
          if (!mbar_wait(smem_u32(&w_empty[s]), ph ^ 1, abort)) return false;
          const int nb = (int)((issued / KB) % nbn), kb = (int)(issued % KB);
          const uint32_t bytes = (uint32_t)(nb == nbn - 1 ? p.n_last : BN) * 128u;
          mbar_expect_tx(smem_u32(&w_full[s]), bytes);
          bulk_g2s(smem_u32(w_smem + s * W_KB_BYTES), wimg + (size_t)nb * BN * KB * 128 + (size_t)kb * bytes, bytes,
                   smem_u32(&w_full[s]));
        }
        return true;
      };
      // WS: the CTA's N block nb into shared memory, once (each CTA of a tile
      // group holds one N block for all its tiles)
      auto load_block = [&](int nb) -> bool {
        const uint32_t kb_bytes = (uint32_t)(nb == nbn - 1 ? p.n_last : L::BNB) * 128u;
        // block nb in the image: 256-row image block wb, rows from h * BNB
        const int wb = L::HALF ? nb >> 1 : nb, h = L::HALF ? nb & 1 : 0;
        const size_t wrows = (size_t)(wb == p.w_blocks - 1 ? p.w_last : BN);
        mbar_expect_tx(smem_u32(&w_full[0]), kb_bytes * KB);
        for (int kb = 0; kb < KB; ++kb)
          bulk_g2s(smem_u32(w_smem + kb * kb_bytes),
                   wimg + (size_t)wb * BN * KB * 128 + (size_t)kb * wrows * 128 + (size_t)h * L::BNB * 128, kb_bytes,
                   smem_u32(&w_full[0]));
        if (!mbar_wait(smem_u32(&w_full[0]), 0, abort)) return false;
        tc_fence_after();
        return true;
      };
      bool ok = WS ? true : issue_w(L::W_STAGES);
      uint64_t used = 0;
      for (int64_t u = 0; ok && u < n_units && !*abort; ++u) {
        const int64_t t = unit_tile(u);
        const uint32_t ab = u % L::A_BUFS, aph = (u / L::A_BUFS) & 1;
        const int nb0 = WS ? ws_nb : 0, nb1 = WS ? nb0 + 1 : nbn;
        if constexpr (WS) {
          if (t == 0 && !load_block(nb0)) break;
        }
        if constexpr (!L::RING_A) {
          if (!mbar_wait(smem_u32(&a_full[ab]), aph, abort)) break;
          tc_fence_after();
        }
        for (int nb = nb0; ok && nb < nb1; ++nb) {
          const int64_t item = WS ? u : t * nbn + nb;
          const uint32_t tb = item & 1, tph = (item >> 1) & 1;
          if (!mbar_wait(smem_u32(&t_empty[tb]), tph ^ 1, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem_base + tb * BN;
          const int rows = nb == nbn - 1 ? p.n_last : L::BNB;
          const uint32_t idesc = make_idesc(rows);
          for (int kb = 0; kb < KB; ++kb, ++used) {
            const uint32_t s = used % L::W_STAGES, ph = (used / L::W_STAGES) & 1;
            uint32_t a0;
            uint64_t aseq = 0;
            if constexpr (L::RING_A) {
              aseq = (uint64_t)u * KB + kb;  // this K-block's slot in the ring
              if (nb == nb0 && !mbar_wait(smem_u32(&a_full[aseq % L::A_SLOTS]), (aseq / L::A_SLOTS) & 1, abort)) {
                ok = false;
                break;
              }
              a0 = smem_u32(a_smem + (aseq % L::A_SLOTS) * A_KB_BYTES);
            } else {
              a0 = smem_u32(a_smem + ab * L::A_BYTES + kb * A_KB_BYTES);
            }
            uint32_t b0;
            if constexpr (WS) {
              tc_fence_after();
              b0 = smem_u32(w_smem + kb * rows * 128);
            } else {
              if (!mbar_wait(smem_u32(&w_full[s]), ph, abort)) { ok = false; break; }
              tc_fence_after();
              b0 = smem_u32(w_smem + s * W_KB_BYTES);
            }
#pragma unroll
            for (int j = 0; j < BK / 16; ++j)
              umma(d, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), idesc, (kb | j) != 0);
            if constexpr (!WS) umma_commit(smem_u32(&w_empty[s]));  // frees the W stage once these MMAs finish
            if constexpr (L::RING_A) {
              if (nb == nb1 - 1) umma_commit(smem_u32(&a_empty[aseq % L::A_SLOTS]));  // the slot may be refilled
            }
            // request block used + 1: with two stages it refills the stage the
            // previous block used (its MMAs are older, so the wait rarely
            // blocks); with one stage it waits for these MMAs
            if (!WS && !issue_w(used + 2)) { ok = false; break; }
          }
          if (!ok) break;
          umma_commit(smem_u32(&t_full[tb]));
        }
        if (!ok) break;
        if constexpr (!L::RING_A) umma_commit(smem_u32(&a_empty[ab]));  // the A tile may be rewritten
      }
    }
  }
  if (L::RING_A && warp == 0) {
    // ------------------------ tensor-map A loads: K-blocks into the ring (lane 1)
    if (lane == 1) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmap_x)) : "memory");
      for (int64_t u = 0; u < n_units && !*abort; ++u) {
        const int64_t tile = grp + unit_tile(u) * gstride;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          const uint64_t aseq = (uint64_t)u * KB + kb;
          constexpr uint32_t kSlots = L::A_SLOTS > 0 ? L::A_SLOTS : 1;  // (RING_A plans only)
          const uint32_t slot = aseq % kSlots;
          if (!mbar_wait(smem_u32(&a_empty[slot]), ((aseq / kSlots) & 1) ^ 1, abort)) { ok = false; break; }
          mbar_expect_tx(smem_u32(&a_full[slot]), A_KB_BYTES);
          tma_load_2d(smem_u32(a_smem + slot * A_KB_BYTES), &p.tmap_x, kb * BK, (int)(tile * BM),
                      smem_u32(&a_full[slot]));
        }
        if (!ok) break;
      }
    }
  } else if (XS && warp == 0) {
    // ----------------------- staged rows: bulk-copy loader (warp 0, lane 1)
    if (lane == 1) {
      const float* x = reinterpret_cast<const float*>(p.x);
      for (int64_t t = 0; t < my_tiles && !*abort; ++t) {
        const int64_t tile = grp + t * gstride;
        bool ok = true;
        for (int grp = 0; grp < BM / XG_ROWS; ++grp) {
          const uint64_t seq = (uint64_t)t * (BM / XG_ROWS) + grp;
          const uint32_t s = seq % L::XSTAGES, ph = (seq / L::XSTAGES) & 1;
          if (!mbar_wait(smem_u32(&x_empty[s]), ph ^ 1, abort)) { ok = false; break; }
          const int64_t row0 = tile * BM + grp * XG_ROWS;
          int64_t rows = p.m - row0;
          rows = rows < 0 ? 0 : (rows > XG_ROWS ? XG_ROWS : rows);
          mbar_expect_tx(smem_u32(&x_full[s]), (uint32_t)(rows * KDIM * 4));
          if (rows > 0)
            bulk_g2s(smem_u32(x_smem + s * XG_BYTES), x + row0 * KDIM, (uint32_t)(rows * KDIM * 4),
                     smem_u32(&x_full[s]));
        }
        if (!ok) break;
      }
    }
  } else if (!L::RING_A && warp >= 1 && warp < 1 + L::PRODUCERS) {
    // ------------------------------------------------------ A producers
    const int kb = lane >> 3, chunk = lane & 7;  // lane owns columns [8*lane, 8*lane+8)
    // LayerNorm of NR rows at once: the NR warp reductions are interleaved so
    // their shuffle latencies overlap.
    auto layer_norm = [&](auto& v) {
      constexpr int NR = sizeof(v) / sizeof(v[0]);
      float s[NR], sq[NR];
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        s[u] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s[u] += v[u][i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < NR; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        s[u] *= (1.f / KDIM);
        sq[u] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) { const float d = v[u][i] - s[u]; sq[u] += d * d; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < NR; ++u) sq[u] += __shfl_xor_sync(0xffffffffu, sq[u], o);
      float g[8], bta[8];  // L1-resident; re-read to keep registers for rows in flight
      load_vec<8>(p.gamma + lane * 8, g);
      load_vec<8>(p.beta + lane * 8, bta);
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        const float rstd = rsqrtf(sq[u] * (1.f / KDIM) + p.eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[u][i] = (v[u][i] - s[u]) * rstd * g[i] + bta[i];
      }
    };
    auto put = [&](uint8_t* abuf, int r, const float* v) {
      uint8_t* dst = abuf + kb * A_KB_BYTES + r * 128 + ((chunk ^ (r & 7)) << 4);
      store_vec<8>(reinterpret_cast<__nv_bfloat16*>(dst), v);
    };
    if constexpr (XS) {
      const int pw = warp - 1;  // 0..6: rows pw, pw + 7, ... of each 32-row group
      for (int64_t t = 0; t < my_tiles && !*abort; ++t) {
        const int64_t tile = grp + t * gstride;
        uint8_t* abuf = a_smem;
        bool ok = true;
        for (int grp = 0; grp < BM / XG_ROWS; ++grp) {
          const uint64_t seq = (uint64_t)t * (BM / XG_ROWS) + grp;
          const uint32_t s = seq % L::XSTAGES, ph = (seq / L::XSTAGES) & 1;
          if (!mbar_wait(smem_u32(&x_full[s]), ph, abort)) { ok = false; break; }
          if (grp == 0 && !mbar_wait(smem_u32(&a_empty[0]), (t & 1) ^ 1, abort)) { ok = false; break; }
          const float* stage = reinterpret_cast<const float*>(x_smem + s * XG_BYTES);
          constexpr int NR = (XG_ROWS + L::PRODUCERS - 1) / L::PRODUCERS;  // 5
          float v[NR][8];
#pragma unroll
          for (int u = 0; u < NR; ++u) {
            const int rl = pw + u * L::PRODUCERS;
            if (rl < XG_ROWS && tile * BM + grp * XG_ROWS + rl < p.m) {
              const float4* src = reinterpret_cast<const float4*>(stage + rl * KDIM + lane * 8);
              const float4 a0 = src[0], a1 = src[1];
              v[u][0] = a0.x; v[u][1] = a0.y; v[u][2] = a0.z; v[u][3] = a0.w;
              v[u][4] = a1.x; v[u][5] = a1.y; v[u][6] = a1.z; v[u][7] = a1.w;
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
            }
          }
          layer_norm(v);
#pragma unroll
          for (int u = 0; u < NR; ++u) {
            const int rl = pw + u * L::PRODUCERS;
            if (rl < XG_ROWS) put(abuf, grp * XG_ROWS + rl, v[u]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&x_empty[s]));
        }
        if (!ok) break;
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&a_full[0]));
      }
    } else {
      const int pw = warp - 1;  // rows pw, pw + PRODUCERS, ... of each tile
      for (int64_t u = 0; u < n_units && !*abort; ++u) {
        const int64_t tile = grp + unit_tile(u) * gstride;
        const uint32_t ab = u % L::A_BUFS, aph = (u / L::A_BUFS) & 1;
        uint8_t* abuf = a_smem + ab * L::A_BYTES;
        if constexpr (PRO == PRO_COPY) {
          // bf16 rows need no arithmetic: each lane cp.asyncs its 16-byte
          // chunk of every row of the warp straight into the swizzled slot
          // (zero-filled past m), so the whole tile is in flight at once with
          // no register cost; the warp then waits for its own copies and
          // fences them for the tensor core's (async-proxy) reads.
          if (!mbar_wait(smem_u32(&a_empty[ab]), aph ^ 1, abort)) break;
          const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(p.x);
          for (int r = pw; r < BM; r += L::PRODUCERS) {
            const int64_t row = tile * BM + r;
            const bool live = row < p.m;
#pragma unroll
            for (int i = 0; i < KB / 4; ++i)  // K-blocks kb, kb + 4: 64-column strips of the row
              cp_async16_zfill(smem_u32(abuf + (kb + 4 * i) * A_KB_BYTES + r * 128 + ((chunk ^ (r & 7)) << 4)),
                               xb + (live ? row : 0) * p.ldx + (kb + 4 * i) * BK + chunk * 8, live);
          }
          cp_async_commit();
          cp_async_wait<0>();
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&a_full[ab]));
          continue;
        }
        bool ok = true;
        constexpr int NRB = PRO == PRO_HEXMEAN ? 3 : RB;  // rows in flight (6 gathers each for HEXMEAN)
        // HEXMEAN: lanes 0-5 hold the six neighbour slots of each row of a
        // batch; the next batch's slots are requested before this batch's
        // gathers, so the table read overlaps the row gathers.
        constexpr int NHX = PRO == PRO_HEXMEAN ? NRB : 1;
        int hx_cur[NHX], hx_next[NHX];
        auto fetch_slots = [&](int rb, int* out) {
#pragma unroll
          for (int u = 0; u < NHX; ++u) {
            const int rr = (rb + u) * L::PRODUCERS + pw;
            const int64_t row = tile * BM + rr;
            out[u] = (rr < BM && row < p.m && lane < HEX_SLOTS) ? __ldg(p.nbr + row * HEX_SLOTS + lane) : -1;
          }
        };
        if constexpr (PRO == PRO_HEXMEAN) fetch_slots(0, hx_cur);
        for (int r0 = 0; r0 * L::PRODUCERS + pw < BM; r0 += NRB) {
          float v[NRB][8];
#pragma unroll
          for (int u = 0; u < NRB; ++u) {
            const int r = (r0 + u) * L::PRODUCERS + pw;
            const int64_t row = tile * BM + r;
            if (r < BM && row < p.m) {
              if constexpr (PRO == PRO_LN) {
                load_vec<8>(reinterpret_cast<const float*>(p.x) + row * p.ldx + lane * 8, v[u]);
              } else if constexpr (PRO == PRO_HEXMEAN) {
                // gathered below, all rows' neighbour loads in flight together
              } else {
                load_vec<8>(reinterpret_cast<const __nv_bfloat16*>(p.x) + row * p.ldx + lane * 8, v[u]);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
            }
          }
          if constexpr (PRO == PRO_HEXMEAN) {
            // lanes 0-5 fetch a row's six slots; every lane then gathers its
            // 16-byte column chunk of each present neighbour row, all NRB rows'
            // gathers issued before the first is summed
            const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(p.x);
            fetch_slots(r0 + NRB, hx_next);
            const int* my = hx_cur;
            uint4 raw[NRB][HEX_SLOTS];
            int present[NRB];
#pragma unroll
            for (int u = 0; u < NRB; ++u) {
              present[u] = 0;
#pragma unroll
              for (int j = 0; j < HEX_SLOTS; ++j) {
                const int nb = __shfl_sync(0xffffffffu, my[u], j);
                raw[u][j] = make_uint4(0, 0, 0, 0);
                if (nb >= p.m) report(ERR_INDEX);
                if (nb >= 0 && nb < p.m) {
                  raw[u][j] = __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)nb * p.ldx) + lane);
                  ++present[u];
                }
              }
            }
#pragma unroll
            for (int u = 0; u < NRB; ++u) {
              float acc[8] = {};
#pragma unroll
              for (int j = 0; j < HEX_SLOTS; ++j) {
                const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&raw[u][j]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 f = __bfloat1622float2(hh[i]);
                  acc[2 * i] += f.x;
                  acc[2 * i + 1] += f.y;
                }
              }
              const float inv = present[u] ? 1.f / (float)present[u] : 0.f;
#pragma unroll
              for (int i = 0; i < 8; ++i) v[u][i] = acc[i] * inv;
            }
#pragma unroll
            for (int u = 0; u < NHX; ++u) hx_cur[u] = hx_next[u];
          }
          // the first batch is fetched before waiting for the buffer to drain
          if (r0 == 0 && !mbar_wait(smem_u32(&a_empty[ab]), aph ^ 1, abort)) { ok = false; break; }
          if constexpr (PRO == PRO_LN) layer_norm(v);
#pragma unroll
          for (int u = 0; u < NRB; ++u) {
            const int r = (r0 + u) * L::PRODUCERS + pw;
            if (r < BM) put(abuf, r, v[u]);
          }
        }
        if (!ok) break;
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&a_full[ab]));
      }
    }
  } else if (warp >= 1 + L::PRODUCERS) {
    // ------------------------------------------------------ epilogue
    const int ew = warp - 1 - L::PRODUCERS;  // 0..EPI_WARPS-1
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    constexpr int PARTS = L::EPI_WARPS / 4;  // column ranges per quadrant
    const int half = ew >> 2;                // this warp's column range
    uint32_t out_seq = 0;                    // EPI_STORE: boxes this warp has handed to the tensor store
    // Residual variants: the warp's residual rows arrive by cp.async in
    // boxes of 32 rows x 32 columns (one box per 32-column chunk of its
    // column range, the chunks of all its tiles in one sequence). A box is
    // requested as soon as its ring slot is free, RING boxes ahead, so the
    // next tile's boxes load during this tile's LayerNorm passes and MMA. A box row's eight 16-byte
    // pieces sit at piece j ^ (row & 7): reading a row (thread = row, TMEM
    // order) and reading a column across rows (lane = column, for coalesced
    // global stores) are both conflict-free.
    constexpr int CHUNKS = (BN / PARTS) / 32;
    constexpr int RING = L::RING;
    float* ring = e_smem + ew * (RING * BOX_FLOATS);
    const int64_t n_boxes = L::RESID ? my_tiles * CHUNKS : 0;
    auto issue_box = [&](int64_t k) {
      if (k < n_boxes) {
        const int64_t tile = grp + (k / CHUNKS) * gstride;
        const int col = half * (BN / PARTS) + (int)(k % CHUNKS) * 32 + (lane & 7) * 4;
        float* box = ring + (k % RING) * BOX_FLOATS;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = (lane >> 3) + 4 * i;
          const int64_t row = tile * BM + q * 32 + r;
          const bool live = row < p.m;
          cp_async16_zfill(smem_u32(box + r * 32 + (((lane & 7) ^ (r & 7)) << 2)),
                           p.res + (live ? row : 0) * p.ldr + col, live);
        }
      }
      cp_async_commit();  // an empty group past the end keeps the wait count uniform
    };
    if constexpr (L::RESID) {
      for (int64_t k = 0; k < RING; ++k) issue_box(k);
    }
    const int64_t n_items = WS ? my_tiles : my_tiles * nbn;  // nbn = 1 for the residual epilogues
    for (int64_t it = 0; it < n_items && !*abort; ++it) {
      const int64_t t = WS ? it : it / nbn;
      const int nb = WS ? ws_nb : (int)(it % nbn);
      const int64_t tile = grp + t * gstride;
      const uint32_t tb = it & 1, tph = (it >> 1) & 1;
      if (!mbar_wait(smem_u32(&t_full[tb]), tph, abort)) break;
      tc_fence_after();
      const int64_t row0 = tile * BM + q * 32;  // this warp's 32 rows
      const int64_t row = row0 + lane;
      if constexpr (L::RESID) {
        // Pass 1 (thread = row): x = residual + acc + bias per chunk; x goes
        // back into the box, from which the warp stores whole 128-byte row
        // segments (lane = column), and, for the LayerNorm variant, into this
        // tile's TMEM columns, summed per row. The two column halves of a row
        // meet in shared memory (a 64-thread named barrier per quadrant).
        // Passes 2 (squared deviations) and 3 (normalised outputs, thread =
        // row, a 64- or 128-byte run of its row per store) read TMEM only, so
        // the LayerNorm costs no further global reads. The TMEM buffer is
        // released after the last pass.
        constexpr bool LN = EPI == EPI_RESID_LN;
        const int cbeg = half * (BN / PARTS);
        const int nr = (int)(p.m - row0 < 32 ? (p.m - row0 < 0 ? 0 : p.m - row0) : 32);  // live rows of the warp
        const uint32_t tcol = tmem_base + ((uint32_t)(q * 32) << 16) + tb * BN;
        float s1 = 0.f;
#pragma unroll 1
        for (int c = 0; c < CHUNKS; ++c) {
          const int64_t k = t * CHUNKS + c;
          const int c0 = cbeg + c * 32;
          float v[32];
          tmem_ld32(tcol + c0, v);
          cp_async_wait<RING - 1>();
          __syncwarp();
          float* box = ring + (k % RING) * BOX_FLOATS;
          float4* br = reinterpret_cast<float4*>(box + lane * 32);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 b4 = reinterpret_cast<const float4*>(par + c0)[j];
            float* e = v + 4 * j;
            e[0] += b4.x; e[1] += b4.y; e[2] += b4.z; e[3] += b4.w;
            if (p.relu) {
              e[0] = fmaxf(e[0], 0.f); e[1] = fmaxf(e[1], 0.f); e[2] = fmaxf(e[2], 0.f); e[3] = fmaxf(e[3], 0.f);
            }
            float4 r4 = br[j ^ (lane & 7)];
            r4.x += e[0]; r4.y += e[1]; r4.z += e[2]; r4.w += e[3];
            e[0] = r4.x; e[1] = r4.y; e[2] = r4.z; e[3] = r4.w;
            br[j ^ (lane & 7)] = r4;
            if constexpr (LN) s1 += (r4.x + r4.y) + (r4.z + r4.w);
          }
          if constexpr (LN) tmem_st32(tcol + c0, v);
          __syncwarp();
          // lane = 16-byte piece: each store covers 4 whole 128-byte row segments
          float* dst = p.res + row0 * p.ldr + c0 + (lane & 7) * 4;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (lane >> 3);
            const float4 x4 = reinterpret_cast<const float4*>(box)[r * 8 + ((lane & 7) ^ (r & 7))];
            if (r < nr) *reinterpret_cast<float4*>(dst + r * p.ldr) = x4;
          }
          __syncwarp();
          issue_box(k + RING);  // into the slot just finished
        }
        if constexpr (LN) {
          float* red = reinterpret_cast<float*>(smem + L::RED_OFF) + q * 64;  // [half][32 rows]
          uint8_t* outbox = smem + L::OUT_OFF + ew * OUT_BOX_BYTES;
          tmem_st_wait();
          red[half * 32 + lane] = s1;
          asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
          const float mean = (red[lane] + red[32 + lane]) * (1.f / BN);
          asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");  // both halves have read the sums
          float s2 = 0.f;
#pragma unroll 1
          for (int c0 = cbeg; c0 < cbeg + BN / PARTS; c0 += 32) {
            float v[32];
            tmem_ld32(tcol + c0, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float d = v[i] - mean;
              s2 += d * d;
            }
          }
          red[half * 32 + lane] = s2;
          asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
          const float rstd = rsqrtf((red[lane] + red[32 + lane]) * (1.f / BN) + p.ln_eps);
          asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");  // both halves have read the squares
#pragma unroll 1
          for (int c0 = cbeg; c0 < cbeg + BN / PARTS; c0 += 32) {
            float v[32];
            tmem_ld32(tcol + c0, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = (v[i] - mean) * rstd;
#pragma unroll
            for (int o = 0; o < MAX_LN; ++o) {
              if (o >= p.n_ln) break;
              // Through the warp's staging box (32 rows of 64 bytes, 16-byte
              // piece j of row r at j ^ ((r >> 1) & 3); the row-wise writes and
              // the piece-wise reads are both conflict-free), so that each
              // store writes whole 64-byte row segments, 8 rows at a time.
              // Each 8-column piece is scaled, shifted and packed on its own,
              // so no second 32-value row is held in registers.
              __syncwarp();  // the previous output's reads of the box are done
              uint4* sb = reinterpret_cast<uint4*>(outbox);
              const float4* g4 = reinterpret_cast<const float4*>(par + (1 + 2 * o) * BN + c0);
              const float4* b4 = reinterpret_cast<const float4*>(par + (2 + 2 * o) * BN + c0);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 ga = g4[2 * j], gb = g4[2 * j + 1], ba = b4[2 * j], bb = b4[2 * j + 1];
                const float* x = v + 8 * j;
                uint4 w;
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
                h[0] = __floats2bfloat162_rn(x[0] * ga.x + ba.x, x[1] * ga.y + ba.y);
                h[1] = __floats2bfloat162_rn(x[2] * ga.z + ba.z, x[3] * ga.w + ba.w);
                h[2] = __floats2bfloat162_rn(x[4] * gb.x + bb.x, x[5] * gb.y + bb.y);
                h[3] = __floats2bfloat162_rn(x[6] * gb.z + bb.z, x[7] * gb.w + bb.w);
                sb[lane * 4 + (j ^ ((lane >> 1) & 3))] = w;
              }
              __syncwarp();
              __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.ln_out[o]) + row0 * p.ln_ld[o] + c0 + (lane & 3) * 8;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = 8 * i + (lane >> 2);
                const uint4 w = sb[r * 4 + ((lane & 3) ^ ((r >> 1) & 3))];
                if (r < nr) *reinterpret_cast<uint4*>(d + r * p.ln_ld[o]) = w;
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&t_empty[tb]));
      } else if constexpr (EPI == EPI_HEAD) {
        // One N block of width cols (128 or 256): each column half takes
        // cols / 2 columns of its rows, v = relu(acc + bias + tok[tok_idx[row]]),
        // and its partial dot products with the output layer's rows; the
        // halves meet in shared memory and half 0 writes the outputs.
        const int cols = p.n_last;
        const int span = cols / 2;
        const int cbeg = half * span;
        float part[MAX_HEAD_OUT] = {};
        int64_t trow = -1;
        if (row < p.m) {
          trow = p.tok_idx[row];
          if (trow < 0 || trow >= p.n_tok) {
            report(ERR_INDEX);
            trow = -1;
          }
        }
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + span; c0 += 32) {
          float v[32];
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + tb * BN + c0, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + c0) + i) : make_float4(0, 0, 0, 0);
            v[4 * i] += bb.x; v[4 * i + 1] += bb.y; v[4 * i + 2] += bb.z; v[4 * i + 3] += bb.w;
          }
          if (trow >= 0) {
            const __nv_bfloat16* tr = p.tok + trow * p.ld_tok + c0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float a[8];
              load_vec<8>(tr + 8 * i, a);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[8 * i + j] += a[j];
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
#pragma unroll
          for (int o = 0; o < MAX_HEAD_OUT; ++o) {
            if (o >= p.n_out) break;
            const float4* w4 = reinterpret_cast<const float4*>(p.w_out + (int64_t)o * cols + c0);
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 w = __ldg(w4 + i);
              acc += v[4 * i] * w.x + v[4 * i + 1] * w.y + v[4 * i + 2] * w.z + v[4 * i + 3] * w.w;
            }
            part[o] += acc;
          }
        }
        float* red = reinterpret_cast<float*>(smem + L::RED_OFF) + q * (MAX_HEAD_OUT * 32);
        if (half == 1) {
#pragma unroll
          for (int o = 0; o < MAX_HEAD_OUT; ++o) red[o * 32 + lane] = part[o];
        }
        asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
        if (half == 0 && row < p.m) {
#pragma unroll
          for (int o = 0; o < MAX_HEAD_OUT; ++o)
            if (o < p.n_out) p.head_out[row * p.ld_head + o] = part[o] + red[o * 32 + lane] + p.b_out[o];
        }
        asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");  // the partials are read before the next tile
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&t_empty[tb]));
      } else {
      const int cols = nb == nbn - 1 ? p.n_last : L::BNB;
      // column ranges of BNB / PARTS (a 128-column block gives each warp 64)
      constexpr int SPAN = L::BNB / PARTS;
      const int cend = (half + 1) * SPAN < cols ? (half + 1) * SPAN : cols;
      const int nr = (int)(p.m - row0 < 32 ? (p.m - row0 < 0 ? 0 : p.m - row0) : 32);  // live rows of the warp
      uint4* sb = reinterpret_cast<uint4*>(smem + L::OUT_OFF + ew * OUT_BOX_BYTES);
#pragma unroll 1
      for (int c0 = half * SPAN; c0 < cend; c0 += 32) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + tb * BN + c0, v);
        const int oc = nb * L::BNB + c0;  // output column
        if (p.bias) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(p.bias + oc) + i);
            v[4 * i] += bb.x; v[4 * i + 1] += bb.y; v[4 * i + 2] += bb.z; v[4 * i + 3] += bb.w;
          }
        }
        if constexpr (EPI == EPI_STORE) {
          if (p.add && row < p.m) {
            const float4* ar = reinterpret_cast<const float4*>(p.add + row * p.ld_add + oc);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 a4 = __ldg(ar + i);
              v[4 * i] += a4.x; v[4 * i + 1] += a4.y; v[4 * i + 2] += a4.z; v[4 * i + 3] += a4.w;
            }
          }
        }
        if (p.relu) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
        }
        if constexpr (EPI == EPI_STORE || EPI == EPI_ADD_X) {
          if constexpr (EPI == EPI_ADD_X) {
            if (row < p.m) {
              const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(p.x) + row * p.ldx + c0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float a[8];
                load_vec<8>(xr + 8 * i, a);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[8 * i + j] += a[j];
              }
            }
          }
          if constexpr (EPI == EPI_STORE) {
            // Into one of the warp's boxes in the tensor map's 64-byte swizzle
            // (16-byte piece j of row r at j ^ ((r >> 1) & 3): conflict-free
            // row-wise writes), then one tensor-map store of the 32 x 32 box
            // by lane 0. The box's previous store must have read it first.
            const uint32_t bi = out_seq % L::OUT_NBOX;
            uint4* ob = reinterpret_cast<uint4*>(smem + L::OUT_OFF + (bi * EPILOGUE + ew) * OUT_BOX_BYTES);
            if (lane == 0) bulk_wait_read<L::OUT_NBOX - 1>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float* x = v + 8 * j;
              uint4 w;
              __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
              for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
              ob[lane * 4 + (j ^ ((lane >> 1) & 3))] = w;
            }
            fence_proxy_async();  // generic-proxy writes -> the tensor store's reads
            __syncwarp();
            if (lane == 0 && nr > 0) {
              tma_store_2d(&p.tmap_out, smem_u32(ob), oc, (int)row0);
              bulk_commit();
            }
            ++out_seq;
            continue;
          }
          // Through the warp's staging box (32 rows of 64 bytes, 16-byte piece
          // j of row r at j ^ ((r >> 1) & 3): the row-wise writes and the
          // piece-wise reads are both conflict-free), so that each store
          // writes whole 64-byte row segments, 8 rows at a time.
          __syncwarp();  // the previous chunk's reads of the box are done
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float* x = v + 8 * j;
            uint4 w;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
            sb[lane * 4 + (j ^ ((lane >> 1) & 3))] = w;
          }
          __syncwarp();
          __nv_bfloat16* d = p.out + row0 * p.ldo + oc + (lane & 3) * 8;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 8 * i + (lane >> 2);
            const uint4 w = sb[r * 4 + ((lane & 3) ^ ((r >> 1) & 3))];
            if (r < nr) *reinterpret_cast<uint4*>(d + r * p.ldo) = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&t_empty[tb]));
      }
    }
    if constexpr (L::RESID) cp_async_wait<0>();  // no box load outlives the loop
    if constexpr (EPI == EPI_STORE) {
      if (lane == 0) bulk_wait_all();  // every tensor store has finished
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// Pre-swizzle W (N x K row-major bf16) into the image the kernel streams:
// N block nb (rows nb * 256 onwards, 256 of them or 128 for a short last
// block) holds its K-blocks one after another, K-block kb holding the
// block's rows, 128 bytes each, 16-byte chunk c of row r stored at chunk
// c ^ (r % 8).
__global__ void swizzle_weight_kernel(const __nv_bfloat16* __restrict__ w, int64_t n, int64_t k,
                                      __nv_bfloat16* __restrict__ img) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // one 16-byte chunk
  const int64_t chunks = n * k / 8;
  if (idx >= chunks) return;
  const int64_t row = idx / (k / 8), kc = idx % (k / 8);
  const int64_t kb = kc / 8, c = kc % 8;
  const int64_t nb = row / BN, r = row % BN;
  const int64_t rows_in_block = n - nb * BN < BN ? n - nb * BN : BN;
  const uint4 val = reinterpret_cast<const uint4*>(w + row * k)[kc];
  uint8_t* dst = reinterpret_cast<uint8_t*>(img) + nb * BN * k * 2 + kb * (rows_in_block * 128) + r * 128 +
                 ((c ^ (r & 7)) << 4);
  *reinterpret_cast<uint4*>(dst) = val;
}

static int g_num_sms = 0;

static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

// cuTensorMapEncodeTiled, fetched once through the runtime (no link-time
// dependency on the driver library).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// The (m, k) bf16 rows at x (leading dim ldx) as a tensor map of 64-column x
// 128-row boxes in the MMA's 128-byte-swizzled K-major layout.
static bool encode_rows_map(CUtensorMap* map, const void* x, int64_t m, int64_t k, int64_t ldx) {
  EncodeTiledFn encode = encode_tiled();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  const cuuint64_t strides[1] = {(cuuint64_t)(ldx * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The (m, n) bf16 output rows at out (leading dim ldo) as a tensor map of
// 32-column x 32-row boxes with the 64-byte swizzle of the staging boxes.
static bool encode_out_map(CUtensorMap* map, void* out, int64_t m, int64_t n, int64_t ldo) {
  EncodeTiledFn encode = encode_tiled();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)m};
  const cuuint64_t strides[1] = {(cuuint64_t)(ldo * 2)};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One persistent CTA per SM (or per tile when there are fewer tiles).
template <int PRO, int EPI, bool XS, int KB, bool WS = false>
static int launch_rowgemm(const Params& prm, cudaStream_t s, const char* what) {
  constexpr int smem_bytes = Plan<PRO, EPI, XS, KB, WS>::SMEM;
  auto kern = rowgemm_kernel<PRO, EPI, XS, KB, WS>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (Plan<PRO, EPI, XS, KB, WS>::L1_HEAVY)  // the smallest shared-memory carveout that fits: the rest is L1
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 0);
  const int64_t tiles = cdiv(prm.m, BM);
  // WS: n_blocks CTAs per tile group (see rowgemm_kernel)
  const int per = WS ? prm.n_blocks : 1;
  const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(tiles, num_sms() / per));
  const int grid = (int)(groups * per);
  kern<<<grid, THREADS, smem_bytes, s>>>(prm);
  return launch_status(what);
}

// Plan choices of the bf16-output launches: 0 = weights streamed per tile,
// 1 = weight-stationary (the default for the plain projections), 2 (LayerNorm
// prologue only) = per-row loads instead of staged 32-row groups.
static int g_store_plan = 1;
static int g_ln_plan = 2;

// The window path of the hex message pass (hex_sm100.cu).
static int hex_window_launch(const void* x, int64_t n, const int32_t* nbr, const void* w_image, const float* bias,
                             void* out, int64_t ldo, cudaStream_t s);

static Params base_params() {
  Params prm{};
  prm.n_blocks = 1;
  prm.n_last = BN;
  prm.w_blocks = 1;
  prm.w_last = BN;
  return prm;
}

}  // namespace sm100
}  // namespace mb

using namespace mb;

extern "C" {

int mb_gemm_weight_image(const void* w, int64_t n, int64_t k, void* image, void* stream) {
  MB_REQUIRE(w && image, "gemm_weight_image: null pointer");
  MB_REQUIRE(n >= 128 && n % 128 == 0 && (k == 256 || k == 512),
             "gemm_weight_image: supports N a multiple of 128 and K 256 or 512 (got %lld x %lld)", (long long)n,
             (long long)k);
  MB_REQUIRE(aligned(w, 16) && aligned(image, 16), "gemm_weight_image: pointers must be 16-byte aligned");
  const int64_t chunks = n * k / 8;
  sm100::swizzle_weight_kernel<<<(unsigned)cdiv(chunks, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)w, n, k, (__nv_bfloat16*)image);
  return launch_status("gemm_weight_image");
}

int mb_gemm_rows_ex(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, const float* gamma,
                    const float* beta, float eps, const void* w_image, int64_t n, const float* bias, int relu,
                    const float* add, int64_t ld_add, void* out, int64_t ldo, float* residual, int64_t ldr,
                    void* stream) {
  using namespace sm100;
  MB_REQUIRE(valid_dtype(x_dtype), "gemm_rows: bad dtype");
  MB_REQUIRE(m >= 0, "gemm_rows: negative m");
  MB_REQUIRE(k == 256 || k == 512, "gemm_rows: K must be 256 or 512 (got %lld)", (long long)k);
  MB_REQUIRE(n >= 128 && n % 128 == 0, "gemm_rows: N must be a positive multiple of 128 (got %lld)", (long long)n);
  if (m == 0) return MB_OK;
  MB_REQUIRE(x && w_image, "gemm_rows: null pointer");
  const bool ln = gamma != nullptr;
  MB_REQUIRE(!ln || (x_dtype == MB_F32 && beta && k == KDIM),
             "gemm_rows: the LayerNorm prologue takes fp32 rows of width 256 and beta");
  MB_REQUIRE(ln || x_dtype == MB_BF16, "gemm_rows: without LayerNorm the rows must be bf16");
  MB_REQUIRE((out != nullptr) != (residual != nullptr), "gemm_rows: exactly one of out / residual");
  MB_REQUIRE(ldx >= k && aligned(x, 16) && (ldx * dtype_size(x_dtype)) % 16 == 0,
             "gemm_rows: x rows must be 16-byte aligned");
  MB_REQUIRE(!out || (ldo >= n && aligned(out, 16) && (ldo * 2) % 16 == 0),
             "gemm_rows: out rows must be 16-byte aligned");
  MB_REQUIRE(!residual || (n == BN && ldr >= BN && aligned(residual, 16) && (ldr * 4) % 16 == 0),
             "gemm_rows: the residual update takes N = 256 and 16-byte aligned fp32 rows");
  MB_REQUIRE(!add || (out && ld_add >= n && aligned(add, 16) && (ld_add * 4) % 16 == 0),
             "gemm_rows: the addend takes a bf16 output and 16-byte aligned fp32 rows");
  MB_REQUIRE(!(ln && residual), "gemm_rows: the LayerNorm prologue writes a bf16 output");
  MB_REQUIRE(aligned(w_image, 16), "gemm_rows: weight image must be 16-byte aligned");
  MB_REQUIRE(!bias || aligned(bias, 16), "gemm_rows: bias must be 16-byte aligned");
  Params prm = base_params();
  prm.x = x;
  prm.ldx = ldx;
  prm.gamma = gamma;
  prm.beta = beta;
  prm.eps = eps;
  prm.w_img = (const __nv_bfloat16*)w_image;
  prm.bias = bias;
  prm.m = m;
  prm.relu = relu;
  prm.out = (__nv_bfloat16*)out;
  prm.ldo = ldo;
  prm.res = residual;
  prm.ldr = ldr;
  prm.add = add;
  prm.ld_add = ld_add;
  prm.n_blocks = (int)cdiv(n, BN);
  prm.n_last = (int)(n - (int64_t)(prm.n_blocks - 1) * BN);
  prm.w_blocks = prm.n_blocks;
  prm.w_last = prm.n_last;
  cudaStream_t s = as_stream(stream);
  if (out) {
    MB_REQUIRE(m < (int64_t(1) << 31), "gemm_rows: at most 2^31 - 1 rows per call");
    if (!encode_out_map(&prm.tmap_out, out, m, n, ldo))
      return ::mb::fail(MB_LAUNCH_FAILED, "gemm_rows: could not encode the output tensor map");
  }
  if (ln) {
    if (g_ln_plan == 1) return launch_rowgemm<PRO_LN, EPI_STORE, false, 4, true>(prm, s, "gemm_rows");
    // contiguous fp32 rows take the bulk-copy staged path (one block per 32-row group)
    if (ldx == KDIM && g_ln_plan == 0) return launch_rowgemm<PRO_LN, EPI_STORE, true, 4>(prm, s, "gemm_rows");
    return launch_rowgemm<PRO_LN, EPI_STORE, false, 4>(prm, s, "gemm_rows");
  }
  // bf16 rows: tensor-map loads of A K-blocks
  MB_REQUIRE(m < (int64_t(1) << 31), "gemm_rows: at most 2^31 - 1 rows per call");
  if (!encode_rows_map(&prm.tmap_x, x, m, k, ldx))
    return ::mb::fail(MB_LAUNCH_FAILED, "gemm_rows: could not encode the input tensor map");
  if (out) {
    if (k == 512) {
      // 128-column weight-stationary blocks; wider outputs stream W instead,
      // which measured faster there (four CTAs per tile group re-read A)
      if (g_store_plan == 1 && n <= BN) {
        prm.n_blocks = (int)(n / 128);
        prm.n_last = 128;
        return launch_rowgemm<PRO_TMA, EPI_STORE, false, 8, true>(prm, s, "gemm_rows");
      }
      return launch_rowgemm<PRO_TMA, EPI_STORE, false, 8>(prm, s, "gemm_rows");
    }
    if (g_store_plan == 1) return launch_rowgemm<PRO_TMA, EPI_STORE, false, 4, true>(prm, s, "gemm_rows");
    return launch_rowgemm<PRO_TMA, EPI_STORE, false, 4>(prm, s, "gemm_rows");
  }
  if (k == 512) return launch_rowgemm<PRO_TMA, EPI_RESIDUAL, false, 8>(prm, s, "gemm_rows");
  return launch_rowgemm<PRO_TMA, EPI_RESIDUAL, false, 4>(prm, s, "gemm_rows");
}

int mb_gemm_set_plan(int store_plan, int ln_plan) {
  MB_REQUIRE(store_plan >= 0 && store_plan <= 1 && ln_plan >= 0 && ln_plan <= 2, "gemm_set_plan: unknown plan");
  sm100::g_store_plan = store_plan;
  sm100::g_ln_plan = ln_plan;
  return MB_OK;
}

int mb_gemm_rows(const void* x, int x_dtype, int64_t ldx, int64_t m, const float* gamma, const float* beta, float eps,
                 const void* w_image, const float* bias, int relu, void* out, int64_t ldo, float* residual,
                 int64_t ldr, void* stream) {
  return mb_gemm_rows_ex(x, x_dtype, ldx, m, sm100::KDIM, gamma, beta, eps, w_image, sm100::BN, bias, relu, nullptr,
                         0, out, ldo, residual, ldr, stream);
}

int mb_gemm_rows_head(const void* x, int64_t ldx, int64_t m, const void* w_image, int64_t n, const float* bias,
                      const void* tok, int64_t ld_tok, int64_t n_tok, const int64_t* tok_idx, const float* w_out,
                      const float* b_out, int n_out, float* out, int64_t ldo, void* stream) {
  using namespace sm100;
  MB_REQUIRE(m >= 0, "gemm_rows_head: negative m");
  MB_REQUIRE(n == 128 || n == 256, "gemm_rows_head: the hidden width must be 128 or 256 (got %lld)", (long long)n);
  MB_REQUIRE(n_out >= 1 && n_out <= MAX_HEAD_OUT, "gemm_rows_head: 1 to %d outputs (got %d)", MAX_HEAD_OUT, n_out);
  if (m == 0) return MB_OK;
  MB_REQUIRE(x && w_image && tok && tok_idx && w_out && b_out && out, "gemm_rows_head: null pointer");
  MB_REQUIRE(ldx >= KDIM && aligned(x, 16) && (ldx * 2) % 16 == 0, "gemm_rows_head: x rows must be 16-byte aligned");
  MB_REQUIRE(ld_tok >= n && aligned(tok, 16) && (ld_tok * 2) % 16 == 0,
             "gemm_rows_head: tok rows must be 16-byte aligned");
  MB_REQUIRE(aligned(w_out, 16) && aligned(w_image, 16) && (!bias || aligned(bias, 16)),
             "gemm_rows_head: misaligned weights or bias");
  MB_REQUIRE(ldo >= n_out, "gemm_rows_head: ldo must hold the outputs");
  Params prm = base_params();
  prm.x = x;
  prm.ldx = ldx;
  prm.w_img = (const __nv_bfloat16*)w_image;
  prm.bias = bias;
  prm.m = m;
  prm.n_last = (int)n;
  prm.w_last = (int)n;
  prm.tok = (const __nv_bfloat16*)tok;
  prm.ld_tok = ld_tok;
  prm.n_tok = n_tok;
  prm.tok_idx = tok_idx;
  prm.w_out = w_out;
  prm.b_out = b_out;
  prm.n_out = n_out;
  prm.head_out = out;
  prm.ld_head = ldo;
  MB_REQUIRE(m < (int64_t(1) << 31), "gemm_rows_head: at most 2^31 - 1 rows per call");
  if (!encode_rows_map(&prm.tmap_x, x, m, KDIM, ldx))
    return ::mb::fail(MB_LAUNCH_FAILED, "gemm_rows_head: could not encode the input tensor map");
  return launch_rowgemm<PRO_TMA, EPI_HEAD, false, 4, true>(prm, as_stream(stream), "gemm_rows_head");
}

int mb_gemm_rows_ln(const void* a, int64_t lda, int64_t m, const void* w_image, const float* bias, float* residual,
                    int64_t ldr, float eps, const float* g0, const float* b0, void* o0, int o0_dtype, int64_t ld0,
                    const float* g1, const float* b1, void* o1, int o1_dtype, int64_t ld1, const float* g2,
                    const float* b2, void* o2, int o2_dtype, int64_t ld2, void* stream) {
  using namespace sm100;
  MB_REQUIRE(m >= 0, "gemm_rows_ln: negative m");
  if (m == 0) return MB_OK;
  MB_REQUIRE(a && w_image && residual, "gemm_rows_ln: null pointer");
  MB_REQUIRE(aligned(a, 16) && (lda * 2) % 16 == 0 && lda >= KDIM, "gemm_rows_ln: a rows must be 16-byte aligned");
  MB_REQUIRE(aligned(residual, 16) && ldr % 4 == 0 && ldr >= BN, "gemm_rows_ln: residual rows must be 16-byte aligned");
  MB_REQUIRE(aligned(w_image, 16) && (!bias || aligned(bias, 16)), "gemm_rows_ln: misaligned weight image or bias");
  Params prm = base_params();
  prm.x = a;
  prm.ldx = lda;
  prm.w_img = (const __nv_bfloat16*)w_image;
  prm.bias = bias;
  prm.m = m;
  prm.res = residual;
  prm.ldr = ldr;
  const float* gs[MAX_LN] = {g0, g1, g2};
  const float* bs[MAX_LN] = {b0, b1, b2};
  void* os[MAX_LN] = {o0, o1, o2};
  const int dts[MAX_LN] = {o0_dtype, o1_dtype, o2_dtype};
  const int64_t lds[MAX_LN] = {ld0, ld1, ld2};
  prm.n_ln = 0;
  prm.ln_eps = eps;
  for (int j = 0; j < MAX_LN; ++j) {
    if (!os[j]) break;
    MB_REQUIRE(gs[j] && bs[j], "gemm_rows_ln: LayerNorm output %d lacks gamma or beta", j);
    MB_REQUIRE(dts[j] == MB_BF16, "gemm_rows_ln: LayerNorm output %d must be bf16", j);
    MB_REQUIRE(aligned(os[j], 16) && (lds[j] * dtype_size(dts[j])) % 16 == 0 && lds[j] >= BN,
               "gemm_rows_ln: LayerNorm output %d rows must be 16-byte aligned", j);
    prm.ln_g[j] = gs[j];
    prm.ln_b[j] = bs[j];
    prm.ln_out[j] = os[j];
    prm.ln_dtype[j] = dts[j];
    prm.ln_ld[j] = lds[j];
    prm.n_ln = j + 1;
  }
  for (int j = prm.n_ln; j < MAX_LN; ++j) MB_REQUIRE(!os[j], "gemm_rows_ln: outputs must be given in order");
  return launch_rowgemm<PRO_COPY, EPI_RESID_LN, false, 4>(prm, as_stream(stream), "gemm_rows_ln");
}

int mb_hex_message_pass(const void* x, int64_t ldx, int64_t n, const int32_t* nbr, const void* w_image,
                        const float* bias, void* out, int64_t ldo, void* stream) {
  using namespace sm100;
  MB_REQUIRE(n >= 0, "hex_message_pass: negative n");
  if (n == 0) return MB_OK;
  MB_REQUIRE(x && nbr && w_image && out, "hex_message_pass: null pointer");
  MB_REQUIRE(x != out, "hex_message_pass: out must not alias x (neighbour rows are read while rows are written)");
  MB_REQUIRE(aligned(x, 16) && (ldx * 2) % 16 == 0 && ldx >= KDIM, "hex_message_pass: x rows must be 16-byte aligned");
  MB_REQUIRE(aligned(out, 16) && (ldo * 2) % 16 == 0 && ldo >= BN, "hex_message_pass: out rows must be 16-byte aligned");
  MB_REQUIRE(aligned(nbr, 4) && aligned(w_image, 16) && (!bias || aligned(bias, 16)),
             "hex_message_pass: misaligned table, weight image or bias");
  // contiguous rows: the kernel that keeps each tile's neighbour rows in
  // shared memory; strided rows: the row GEMM with a gathering prologue
  if (ldx == KDIM && n < (int64_t(1) << 31)) return hex_window_launch(x, n, nbr, w_image, bias, out, ldo, as_stream(stream));
  Params prm = base_params();
  prm.x = x;
  prm.ldx = ldx;
  prm.w_img = (const __nv_bfloat16*)w_image;
  prm.bias = bias;
  prm.m = n;
  prm.out = (__nv_bfloat16*)out;
  prm.ldo = ldo;
  prm.nbr = nbr;
  return launch_rowgemm<PRO_HEXMEAN, EPI_ADD_X, false, 4>(prm, as_stream(stream), "hex_message_pass");
}

}  // extern "C"
