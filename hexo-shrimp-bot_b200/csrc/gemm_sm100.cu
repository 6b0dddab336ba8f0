// Fused row GEMM on the 5th-generation tensor cores (sm_100a tcgen05):
//
//     out = epilogue( prologue(x) @ W^T + bias )
//
//   prologue: LN      - fp32 rows -> LayerNorm (fp32 statistics) -> bf16
//             COPY    - bf16 rows used as they are
//             HEXMEAN - mean of the bf16 rows of a node's present hex
//                       neighbours (six-slot int32 table, -1 = absent; fp32
//                       sum, zero when none is present) -> bf16
//   epilogue: STORE    - bf16 rows (optionally ReLU)
//             RESIDUAL - x_res[row] += result (fp32, in place)
//             ADD_X    - out[row] = x[row] + result (bf16), the fused
//                        message-passing update y = x + W mean(x[nbr]) + b
//             RESID_LN - RESIDUAL, then up to three LayerNorms of each
//                        updated row (bf16 outputs), from the same launch
//
// K = 256 (one model width), N = 256 output columns per launch, M any.
// The op is HBM-bound (about 1.5-4 KB of row traffic per 131 kFLOP), so the
// design is about keeping row bytes in flight and accesses coalesced.
//
// Persistent, warp-specialised CTA (one per SM, 16 warps = 4 per SM
// sub-partition, so every thread may hold 128 registers):
//   warp 0      lane 0 streams pre-swizzled 64-wide K-blocks of W (32 KB,
//               L2-resident) through a 1- or 2-stage ring with cp.async.bulk
//               and issues the tcgen05.mma stream (M=128, N=256, K=16, bf16 x
//               bf16 -> fp32) into a double-buffered TMEM accumulator,
//               signalling with tcgen05.commit.
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
#include "common.cuh"

namespace mb {
namespace sm100 {

constexpr int BM = 128, BN = 256, BK = 64, KDIM = 256;
constexpr int KBLOCKS = KDIM / BK;                 // 4
constexpr int A_BYTES = BM * KDIM * 2;             // 64 KB
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
constexpr int BAR_BYTES = 256;
constexpr long long kWaitCycles = 4000000000LL;   // ~2 s at 1.9 GHz

enum Prologue { PRO_LN = 0, PRO_COPY = 1, PRO_HEXMEAN = 2 };
enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_ADD_X = 2, EPI_RESID_LN = 3 };
constexpr int MAX_LN = 3;
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

// 16-byte cp.async (L2 only) that zero-fills the destination when `live` is
// false, and the group commit / wait that orders a warp's boxes.
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool live) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(live ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

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
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
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

struct Params {
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
};

// Shared-memory plan of one variant (all region offsets 1024-byte aligned).
template <int PRO, int EPI, bool XS>
struct Plan {
  // The residual epilogues stream the residual through a shared-memory ring,
  // which takes the second A buffer's space (the epilogue, not the MMA,
  // bounds these variants).
  static constexpr bool RESID = EPI == EPI_RESIDUAL || EPI == EPI_RESID_LN;
  static constexpr int A_BUFS = (XS || RESID) ? 1 : 2;
  // W K-blocks in flight. The residual epilogues are long enough to hide a
  // one-stage W stream; the freed 32 KB hold the output staging boxes.
  static constexpr int W_STAGES = RESID ? 1 : 2;
  // Residual boxes (32 rows x 32 fp32 columns, 4 KB) per epilogue warp.
  static constexpr int RING = 3;
  // Warps writing the A tile (1..PRODUCERS) and draining TMEM (the rest).
  // The neighbour-gather prologue is latency-bound, so it gets more warps and
  // the epilogue four (one per TMEM lane quadrant, all 256 columns each).
  static constexpr int PRODUCERS = PRO == PRO_HEXMEAN ? 11 : 7;
  static constexpr int EPI_WARPS = 16 - 1 - PRODUCERS;
  static constexpr int A_OFF = 0;
  static constexpr int W_OFF = A_OFF + A_BUFS * A_BYTES;
  static constexpr int X_OFF = W_OFF + W_STAGES * W_KB_BYTES;
  static constexpr int E_OFF = X_OFF + (XS ? X_STAGES * XG_BYTES : 0);
  static constexpr int OUT_OFF = E_OFF + (RESID ? EPILOGUE * RING * BOX_FLOATS * 4 : 0);
  // bias and the LayerNorms' gamma / beta, copied once per CTA (uniform
  // reads in the epilogue, kept out of the busy L1 miss path)
  static constexpr int PAR_OFF = OUT_OFF + (EPI == EPI_RESID_LN ? EPILOGUE * OUT_BOX_BYTES : 0);
  static constexpr int RED_OFF = PAR_OFF + (RESID ? (1 + 2 * MAX_LN) * BN * 4 : 0);
  static constexpr int BAR_OFF = RED_OFF + (EPI == EPI_RESID_LN ? 4 * 64 * 4 : 0);
  static constexpr int SMEM = BAR_OFF + BAR_BYTES + 1024 /*alignment slack*/;
  static_assert(SMEM <= 232448, "shared memory plan exceeds 227 KB");
};

template <int PRO, int EPI, bool XS>
__global__ void __launch_bounds__(THREADS, 1) rowgemm_kernel(const Params p) {
  using L = Plan<PRO, EPI, XS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_smem = smem + L::A_OFF;
  uint8_t* w_smem = smem + L::W_OFF;
  uint8_t* x_smem = smem + L::X_OFF;
  float* e_smem = reinterpret_cast<float*>(smem + L::E_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* a_full = bars;            // [2]
  uint64_t* a_empty = bars + 2;       // [2]
  uint64_t* w_full = bars + 4;        // [2]
  uint64_t* w_empty = bars + 6;       // [2]
  uint64_t* t_full = bars + 8;        // [2]
  uint64_t* t_empty = bars + 10;      // [2]
  uint64_t* x_full = bars + 12;       // [3]
  uint64_t* x_empty = bars + 15;      // [3]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 19);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_tiles = (p.m + BM - 1) / BM;
  const int64_t my_tiles = n_tiles > blockIdx.x ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&a_full[i]), L::PRODUCERS);
      mbar_init(smem_u32(&a_empty[i]), 1);
      mbar_init(smem_u32(&w_full[i]), 1);
      mbar_init(smem_u32(&w_empty[i]), 1);
      mbar_init(smem_u32(&t_full[i]), 1);
      mbar_init(smem_u32(&t_empty[i]), L::EPI_WARPS);
    }
    for (int i = 0; i < X_STAGES; ++i) {
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
      const uint64_t total_kb = (uint64_t)my_tiles * KBLOCKS;
      uint64_t issued = 0;
      auto issue_w = [&](uint64_t upto) -> bool {
        for (; issued < upto && issued < total_kb; ++issued) {
          const uint32_t s = issued % L::W_STAGES, ph = (issued / L::W_STAGES) & 1;
          if (!mbar_wait(smem_u32(&w_empty[s]), ph ^ 1, abort)) return false;
          mbar_expect_tx(smem_u32(&w_full[s]), W_KB_BYTES);
          bulk_g2s(smem_u32(w_smem + s * W_KB_BYTES),
                   reinterpret_cast<const uint8_t*>(p.w_img) + (size_t)(issued % KBLOCKS) * W_KB_BYTES, W_KB_BYTES,
                   smem_u32(&w_full[s]));
        }
        return true;
      };
      bool ok = issue_w(L::W_STAGES);
      uint64_t used = 0;
      for (int64_t t = 0; ok && t < my_tiles && !*abort; ++t) {
        const uint32_t tb = t & 1, tph = (t >> 1) & 1;
        const uint32_t ab = t % L::A_BUFS, aph = (t / L::A_BUFS) & 1;
        if (!mbar_wait(smem_u32(&t_empty[tb]), tph ^ 1, abort)) break;
        if (!mbar_wait(smem_u32(&a_full[ab]), aph, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + tb * BN;
        for (int kb = 0; kb < KBLOCKS; ++kb, ++used) {
          const uint32_t s = used % L::W_STAGES, ph = (used / L::W_STAGES) & 1;
          if (!mbar_wait(smem_u32(&w_full[s]), ph, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(a_smem + ab * A_BYTES + kb * A_KB_BYTES);
          const uint32_t b0 = smem_u32(w_smem + s * W_KB_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            umma(d, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), (kb | j) != 0);
          umma_commit(smem_u32(&w_empty[s]));  // frees the W stage once these MMAs finish
          // request block used + 1: with two stages it refills the stage the
          // previous block used (its MMAs are older, so the wait rarely
          // blocks); with one stage it waits for these MMAs
          if (!issue_w(used + 2)) { ok = false; break; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&a_empty[ab]));  // the A tile may be rewritten once these MMAs finish
        umma_commit(smem_u32(&t_full[tb]));
      }
    }
  }
  if (XS && warp == 0) {
    // ----------------------- staged rows: bulk-copy loader (warp 0, lane 1)
    if (lane == 1) {
      const float* x = reinterpret_cast<const float*>(p.x);
      for (int64_t t = 0; t < my_tiles && !*abort; ++t) {
        const int64_t tile = blockIdx.x + t * gridDim.x;
        bool ok = true;
        for (int grp = 0; grp < BM / XG_ROWS; ++grp) {
          const uint64_t seq = (uint64_t)t * (BM / XG_ROWS) + grp;
          const uint32_t s = seq % X_STAGES, ph = (seq / X_STAGES) & 1;
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
  } else if (warp >= 1 && warp < 1 + L::PRODUCERS) {
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
        const int64_t tile = blockIdx.x + t * gridDim.x;
        uint8_t* abuf = a_smem;
        bool ok = true;
        for (int grp = 0; grp < BM / XG_ROWS; ++grp) {
          const uint64_t seq = (uint64_t)t * (BM / XG_ROWS) + grp;
          const uint32_t s = seq % X_STAGES, ph = (seq / X_STAGES) & 1;
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
      for (int64_t t = 0; t < my_tiles && !*abort; ++t) {
        const int64_t tile = blockIdx.x + t * gridDim.x;
        const uint32_t ab = t % L::A_BUFS, aph = (t / L::A_BUFS) & 1;
        uint8_t* abuf = a_smem + ab * A_BYTES;
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
            cp_async16_zfill(smem_u32(abuf + kb * A_KB_BYTES + r * 128 + ((chunk ^ (r & 7)) << 4)),
                             xb + (live ? row : 0) * p.ldx + lane * 8, live);
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
        const int64_t tile = blockIdx.x + (k / CHUNKS) * gridDim.x;
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
    for (int64_t t = 0; t < my_tiles && !*abort; ++t) {
      const int64_t tile = blockIdx.x + t * gridDim.x;
      const uint32_t tb = t & 1, tph = (t >> 1) & 1;
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
      } else {
#pragma unroll 1
      for (int c0 = half * (BN / PARTS); c0 < (half + 1) * (BN / PARTS); c0 += 32) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + tb * BN + c0, v);
        if (p.bias) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(p.bias + c0) + i);
            v[4 * i] += bb.x; v[4 * i + 1] += bb.y; v[4 * i + 2] += bb.z; v[4 * i + 3] += bb.w;
          }
        }
        if (p.relu) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
        }
        if constexpr (EPI == EPI_STORE || EPI == EPI_ADD_X) {
          if (row < p.m) {
            if constexpr (EPI == EPI_ADD_X) {
              const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(p.x) + row * p.ldx + c0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float a[8];
                load_vec<8>(xr + 8 * i, a);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[8 * i + j] += a[j];
              }
            }
            __nv_bfloat16* o = p.out + row * p.ldo + c0;
#pragma unroll
            for (int i = 0; i < 4; ++i) store_vec<8>(o + 8 * i, v + 8 * i);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&t_empty[tb]));
      }
    }
    if constexpr (L::RESID) cp_async_wait<0>();  // no box load outlives the loop
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
// K-block kb holds rows n = 0..BN-1, 128 bytes each, 16-byte chunk c of row n
// stored at chunk c ^ (n % 8).
__global__ void swizzle_weight_kernel(const __nv_bfloat16* __restrict__ w, int64_t n, int64_t k,
                                      __nv_bfloat16* __restrict__ img) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // one 16-byte chunk
  const int64_t chunks = n * k / 8;
  if (idx >= chunks) return;
  const int64_t row = idx / (k / 8), kc = idx % (k / 8);
  const int64_t kb = kc / 8, c = kc % 8;
  const uint4 val = reinterpret_cast<const uint4*>(w + row * k)[kc];
  uint8_t* dst = reinterpret_cast<uint8_t*>(img) + kb * (n * 128) + row * 128 + ((c ^ (row & 7)) << 4);
  *reinterpret_cast<uint4*>(dst) = val;
}

static int g_num_sms = 0;

}  // namespace sm100
}  // namespace mb

using namespace mb;

extern "C" {

int mb_gemm_weight_image(const void* w, int64_t n, int64_t k, void* image, void* stream) {
  MB_REQUIRE(w && image, "gemm_weight_image: null pointer");
  MB_REQUIRE(n == sm100::BN && k == sm100::KDIM, "gemm_weight_image: supports N=%d, K=%d (got %lld x %lld)",
             sm100::BN, sm100::KDIM, (long long)n, (long long)k);
  MB_REQUIRE(aligned(w, 16) && aligned(image, 16), "gemm_weight_image: pointers must be 16-byte aligned");
  const int64_t chunks = n * k / 8;
  sm100::swizzle_weight_kernel<<<(unsigned)cdiv(chunks, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)w, n, k, (__nv_bfloat16*)image);
  return launch_status("gemm_weight_image");
}

int mb_gemm_rows(const void* x, int x_dtype, int64_t ldx, int64_t m, const float* gamma, const float* beta, float eps,
                 const void* w_image, const float* bias, int relu, void* out, int64_t ldo, float* residual,
                 int64_t ldr, void* stream) {
  using namespace sm100;
  MB_REQUIRE(valid_dtype(x_dtype), "gemm_rows: bad dtype");
  MB_REQUIRE(m >= 0, "gemm_rows: negative m");
  if (m == 0) return MB_OK;
  MB_REQUIRE(x && w_image, "gemm_rows: null pointer");
  const bool ln = gamma != nullptr;
  MB_REQUIRE(!ln || (x_dtype == MB_F32 && beta), "gemm_rows: the LayerNorm prologue takes fp32 rows and beta");
  MB_REQUIRE(ln || x_dtype == MB_BF16, "gemm_rows: without LayerNorm the rows must be bf16");
  MB_REQUIRE((out != nullptr) != (residual != nullptr), "gemm_rows: exactly one of out / residual");
  MB_REQUIRE(aligned(x, 16) && (ldx * dtype_size(x_dtype)) % 16 == 0, "gemm_rows: x rows must be 16-byte aligned");
  MB_REQUIRE(!out || (aligned(out, 16) && (ldo * 2) % 16 == 0), "gemm_rows: out rows must be 16-byte aligned");
  MB_REQUIRE(!residual || (aligned(residual, 16) && (ldr * 4) % 16 == 0),
             "gemm_rows: residual rows must be 16-byte aligned");
  MB_REQUIRE(aligned(w_image, 16), "gemm_rows: weight image must be 16-byte aligned");
  MB_REQUIRE(!bias || aligned(bias, 16), "gemm_rows: bias must be 16-byte aligned");
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  Params prm{x, ldx, gamma, beta, eps, (const __nv_bfloat16*)w_image, bias, m, relu, (__nv_bfloat16*)out, ldo,
             residual, ldr};
  const int64_t tiles = cdiv(m, BM);
  const int grid = (int)(tiles < g_num_sms ? tiles : g_num_sms);
  cudaStream_t s = as_stream(stream);
  auto launch = [&](auto kern, int smem_bytes) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    kern<<<grid, THREADS, smem_bytes, s>>>(prm);
  };
  // Contiguous fp32 rows take the bulk-copy staged path (rows are copied as
  // one block per 32-row group).
  const bool staged = ln && ldx == KDIM;
  if (ln) {
    MB_REQUIRE(out != nullptr, "gemm_rows: the LayerNorm prologue writes a bf16 output");
    if (staged) launch(rowgemm_kernel<PRO_LN, EPI_STORE, true>, Plan<PRO_LN, EPI_STORE, true>::SMEM);
    else launch(rowgemm_kernel<PRO_LN, EPI_STORE, false>, Plan<PRO_LN, EPI_STORE, false>::SMEM);
  } else {
    if (out) launch(rowgemm_kernel<PRO_COPY, EPI_STORE, false>, Plan<PRO_COPY, EPI_STORE, false>::SMEM);
    else launch(rowgemm_kernel<PRO_COPY, EPI_RESIDUAL, false>, Plan<PRO_COPY, EPI_RESIDUAL, false>::SMEM);
  }
  return launch_status("gemm_rows");
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
  Params prm{a, lda, nullptr, nullptr, 0.f, (const __nv_bfloat16*)w_image, bias, m, 0, nullptr, 0, residual, ldr,
             nullptr};
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
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  const int64_t tiles = cdiv(m, BM);
  const int grid = (int)(tiles < g_num_sms ? tiles : g_num_sms);
  auto kern = rowgemm_kernel<PRO_COPY, EPI_RESID_LN, false>;
  const int smem_bytes = Plan<PRO_COPY, EPI_RESID_LN, false>::SMEM;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  kern<<<grid, THREADS, smem_bytes, as_stream(stream)>>>(prm);
  return launch_status("gemm_rows_ln");
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
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  Params prm{x, ldx, nullptr, nullptr, 0.f, (const __nv_bfloat16*)w_image, bias, n, 0, (__nv_bfloat16*)out, ldo,
             nullptr, 0, nbr};
  const int64_t tiles = cdiv(n, BM);
  const int grid = (int)(tiles < g_num_sms ? tiles : g_num_sms);
  auto kern = rowgemm_kernel<PRO_HEXMEAN, EPI_ADD_X, false>;
  const int smem_bytes = Plan<PRO_HEXMEAN, EPI_ADD_X, false>::SMEM;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  kern<<<grid, THREADS, smem_bytes, as_stream(stream)>>>(prm);
  return launch_status("hex_message_pass");
}

}  // extern "C"
