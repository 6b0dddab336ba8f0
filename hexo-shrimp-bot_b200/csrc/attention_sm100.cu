// Axial-bias cell-token attention on the 5th-generation tensor cores
// (sm_100a tcgen05): per position b and head h over L <= 256 tokens,
//
//   out[b,h,i] = softmax_j( q_i . k_j / sqrt(32) + bias[dq+16, dr+16, h] ) v_j
//   dq = clamp(q-coord of key j - q-coord of query i, -16, 16), dr likewise,
//
// keys j < valid[b] only; query rows i >= valid[b] are written as zeros.
// head_dim 32, bf16 q/k/v/out, fp32 scores and softmax.
//
// One CTA per (position, head), eight warps, two CTAs per SM so that one
// CTA's staging and softmax overlap the other's. Q and K share one 128-byte
// swizzled row per token (Q in the first 64 bytes, K in the second; the
// UMMA descriptors start 0 or 64 bytes into the row), V is staged
// transposed. Query tiles of 128 run one after the other: one thread issues
// S = Q K^T into TMEM (M=128, N up to 256, two K=16 steps); a thread holds one
// query row of one key half (TMEM lane quadrant = warp % 4). A first pass adds
// the offset bias, writes the biased scores back into TMEM and finds the
// half-row maximum; the halves' maxima meet in shared memory. Then per half of
// the keys (128 at a time, through one 32 KB P buffer) a second pass writes
// exp(x - max) as bf16 into P and sums it, and P V^T (M=128, N=32) accumulates
// into the tile's first TMEM columns, whose scores are consumed by then. The
// row is scaled by 1/sum and stored. Work is bounded by each position's
// valid length. Every mbarrier wait is bounded (see gemm_sm100.cu).
#include "common.cuh"

namespace mb {
namespace sm100 {

constexpr int AX_L = 256;          // tokens per position (maximum)
constexpr int AX_D = 32;           // head dim
constexpr int AX_SPAN = 33;        // relative offsets -16..16
constexpr int AX_THREADS = 256;
constexpr int AX_QK_BYTES = AX_L * 128;          // 32 KB: Q | K per token row
constexpr int AX_VT_KB = AX_D * 128;             // 4 KB per 64-key block of V^T (32 rows)
constexpr int AX_VT_BYTES = 4 * AX_VT_KB;        // 16 KB
constexpr int AX_P_KB = 128 * 128;               // 16 KB per 64-key block of P
constexpr int AX_P_BYTES = 2 * AX_P_KB;          // one key half (128 keys)
constexpr int AX_QK_OFF = 0;
constexpr int AX_VT_OFF = AX_QK_OFF + AX_QK_BYTES;
constexpr int AX_P_OFF = AX_VT_OFF + AX_VT_BYTES;
constexpr int AX_BIAS_OFF = AX_P_OFF + AX_P_BYTES;
constexpr int AX_COORD_OFF = AX_BIAS_OFF + 4400;  // 33*33 floats, rounded up
constexpr int AX_KPK_OFF = AX_COORD_OFF + AX_L * 8;   // packed key offsets (int32 per key)
constexpr int AX_RED_OFF = AX_KPK_OFF + AX_L * 4;     // per-row half maxima / sums
constexpr int AX_BAR_OFF = AX_RED_OFF + 2 * 2 * 128 * 4;
constexpr int AX_SMEM = AX_BAR_OFF + 64 + 1024;   // + alignment slack
static_assert(2 * AX_SMEM <= 232448, "axial attention must fit two CTAs per SM");
constexpr int AX_TMEM_COLS = 256;                 // S of one tile; O reuses its first columns

constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
constexpr uint32_t AX_IDESC_O = idesc_f16(128, AX_D);
// Packed offsets: a key's coordinates relative to the position's first token,
// plus AX_OFF, in the two 16-bit halves of one word (q high, r low). With
// every coordinate within AX_NEAR of the first token's, key word - query word
// holds (dq + AX_OFF, dr + AX_OFF) in its halves with no borrow between them,
// and both halves are clamped at once with 16-bit SIMD min / max.
constexpr int AX_OFF = 16384, AX_NEAR = 8192;
constexpr unsigned AX_LO2 = (unsigned)(AX_OFF - 16) * 0x10001u, AX_HI2 = (unsigned)(AX_OFF + 16) * 0x10001u;
constexpr int AX_CIDX = (AX_OFF - 16) * (AX_SPAN + 1);  // the clamped halves' index at (-16, -16)
constexpr float AX_LOG2E = 1.4426950408889634f;

__device__ __forceinline__ float ax_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void umma_i(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled
// K-major block whose rows are 128 bytes.
__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__global__ void __launch_bounds__(AX_THREADS, 2) axial_attention_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    int64_t s_pos, int64_t s_head, int64_t s_row, int heads, int length, const int32_t* __restrict__ coords,
    const int32_t* __restrict__ valid, const float* __restrict__ bias, __nv_bfloat16* __restrict__ out,
    int64_t o_pos, int64_t o_head, int64_t o_row) {
  extern __shared__ uint8_t ax_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ax_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qk = smem + AX_QK_OFF;
  uint8_t* vt = smem + AX_VT_OFF;
  uint8_t* ps = smem + AX_P_OFF;
  float* bias_s = reinterpret_cast<float*>(smem + AX_BIAS_OFF);
  int2* kc = reinterpret_cast<int2*>(smem + AX_COORD_OFF);
  int* kpk = reinterpret_cast<int*>(smem + AX_KPK_OFF);
  float* red = reinterpret_cast<float*>(smem + AX_RED_OFF);  // [max | sum][half][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AX_BAR_OFF);
  uint64_t* s_done = bars;       // one phase per query tile
  uint64_t* o_done = bars + 1;   // one phase per (tile, key half)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 3);

  const int b = blockIdx.x / heads, h = blockIdx.x % heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int nv = valid[b];
  if (nv < 0 || nv > length) {
    if (tid == 0) report(ERR_INDEX);
    nv = nv < 0 ? 0 : length;
  }
  const int n_tiles = nv > 128 ? 2 : (nv > 0 ? 1 : 0);
  const __nv_bfloat16* qb = q + b * s_pos + h * s_head;
  const __nv_bfloat16* kb = k + b * s_pos + h * s_head;
  const __nv_bfloat16* vb = v + b * s_pos + h * s_head;
  __nv_bfloat16* ob = out + b * o_pos + h * o_head;
  const int32_t* cb = coords + (int64_t)b * length * 2;

  if (tid == 0) {
    mbar_init(smem_u32(&s_done[0]), 1);
    mbar_init(smem_u32(&o_done[0]), 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(AX_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // ---- stage Q | K rows, V^T, bias, key coords (zero past the valid length)
  // every global load of the thread is issued before the first shared store
  constexpr int PER = AX_L * 4 / AX_THREADS;  // 16-byte chunks of Q (and of K, V) per thread
  const uint4 zero = make_uint4(0, 0, 0, 0);
  uint4 qv[PER], kv[PER], vv[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int idx = tid + u * AX_THREADS, r = idx >> 2, c = idx & 3;
    qv[u] = kv[u] = vv[u] = zero;
    if (r < nv) {
      qv[u] = __ldg(reinterpret_cast<const uint4*>(qb + r * s_row) + c);
      kv[u] = __ldg(reinterpret_cast<const uint4*>(kb + r * s_row) + c);
      vv[u] = __ldg(reinterpret_cast<const uint4*>(vb + r * s_row) + c);
    }
  }
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int idx = tid + u * AX_THREADS, r = idx >> 2, c = idx & 3;
    *reinterpret_cast<uint4*>(qk + swz(r, c)) = qv[u];
    *reinterpret_cast<uint4*>(qk + swz(r, 4 + c)) = kv[u];
    // V row r, columns 8c..8c+7 -> V^T rows 8c..8c+7, column r
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&vv[u]);
    const int blk = r >> 6, jj = r & 63;
#pragma unroll
    for (int w = 0; w < 8; ++w)
      *reinterpret_cast<__nv_bfloat16*>(vt + blk * AX_VT_KB + swz(8 * c + w, jj >> 3) + (jj & 7) * 2) = e[w];
  }
  // scores are kept in log2 units: the bias table is stored times log2(e)
  for (int idx = tid; idx < AX_SPAN * AX_SPAN; idx += AX_THREADS)
    bias_s[idx] = __ldg(bias + (int64_t)idx * heads + h) * AX_LOG2E;
  const int bx = length > 0 ? __ldg(cb) : 0, by = length > 0 ? __ldg(cb + 1) : 0;
  bool near = true;
  if (tid < AX_L) {
    const int2 c = tid < length ? make_int2(__ldg(cb + 2 * tid), __ldg(cb + 2 * tid + 1)) : make_int2(0, 0);
    kc[tid] = c;
    const int64_t ox = (int64_t)c.x - bx, oy = (int64_t)c.y - by;
    const bool in = tid < nv;  // keys (and the queries that are written) are the first nv tokens
    near = !in || (ox > -AX_NEAR && ox < AX_NEAR && oy > -AX_NEAR && oy < AX_NEAR);
    // keys past the valid length sit at the first token (in range; masked later)
    kpk[tid] = in && near ? (int)((((uint32_t)(ox + AX_OFF)) << 16) | (uint32_t)(oy + AX_OFF))
                          : (int)(((uint32_t)AX_OFF << 16) | (uint32_t)AX_OFF);
  }
  fence_proxy_async();  // generic-proxy shared stores -> visible to the tensor cores
  tc_fence_before();
  // packed offsets are used when every valid token is near the first one
  const bool packed = __syncthreads_and(near) != 0;
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Warp roles: TMEM lane quadrant qd = warp % 4 (rows 32qd..32qd+31 of the
  // tile), key half hf = warp / 4. Work is bounded by the valid length:
  // score columns up to nv rounded to a 32-column load, P and P V up to nv
  // rounded to a 64-key block.
  const int qd = warp & 3, hf = warp >> 2;
  const int rl = qd * 32 + lane;
  const float scale = 0.17677669529663687f * AX_LOG2E;  // 1 / sqrt(32), in log2 units
  const int kend = min(AX_L, (nv + 31) & ~31);
  const int npad = (nv + 15) & ~15;
  const int kblocks = (nv + 63) >> 6;
  const int halves = (kblocks + 1) >> 1;
  const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16);
  float* red_m = red;
  float* red_s = red + 2 * 128;
  bool ok = true;
  int phase_s = 0, phase_o = 0;
  for (int t = 0; t < n_tiles; ++t) {
    const int row = t * 128 + rl;
    const bool warp_live = t * 128 + qd * 32 < nv;
    if (tid == 0 && !*abort) {
      const uint32_t a0 = smem_u32(qk + t * 128 * 128), b0 = smem_u32(qk);
#pragma unroll
      for (int j = 0; j < AX_D / 16; ++j)
        umma_i(tmem, smem_desc(a0 + j * 32), smem_desc(b0 + 64 + j * 32), idesc_f16(128, npad), j);
      umma_commit(smem_u32(&s_done[0]));
    }
    // pass 1: biased scores back into TMEM, the half-row maximum
    float m = -INFINITY;
    ok = ok && mbar_wait(smem_u32(&s_done[0]), phase_s, abort);
    phase_s ^= 1;
    tc_fence_after();
    if (ok && warp_live) {
      const int2 qc = row < length ? make_int2(__ldg(cb + 2 * row), __ldg(cb + 2 * row + 1)) : make_int2(0, 0);
      // the query's packed offsets (rows past the valid length are written as
      // zeros: they take the first token's, which keeps the index in range)
      const int qp = row < nv ? (int)((uint32_t)(qc.x - bx) << 16) + (qc.y - by) : 0;
      const int c_lo = hf * 128, c_hi = min(c_lo + 128, kend);
#pragma unroll 1
      for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        float sc[32];
        tmem_ld32(taddr + c0, sc);
        if (packed) {
          const int4* k4p = reinterpret_cast<const int4*>(kpk + c0);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int4 k4 = k4p[u];
            const int kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const unsigned d = __vmins2(__vmaxs2((unsigned)(kk[e] - qp), AX_LO2), AX_HI2);
              const int idx = (int)(d >> 16) * AX_SPAN + (int)(d & 0xffffu) - AX_CIDX;
              sc[4 * u + e] = fmaf(sc[4 * u + e], scale, bias_s[idx]);
            }
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int2 c = kc[c0 + jj];
            const int dq = min(max(c.x - qc.x, -16), 16) + 16, dr = min(max(c.y - qc.y, -16), 16) + 16;
            sc[jj] = fmaf(sc[jj], scale, bias_s[dq * AX_SPAN + dr]);
          }
        }
        if (c0 + 32 > nv) {  // the last chunk: keys past the valid length
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (c0 + jj >= nv) sc[jj] = -INFINITY;
        }
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) m = fmaxf(m, sc[jj]);
        tmem_st32(taddr + c0, sc);
      }
      tmem_st_wait();
    }
    red_m[hf * 128 + rl] = m;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    m = fmaxf(red_m[rl], red_m[128 + rl]);
    // per key half: P = exp(x - m) in bf16 (this warp's 64-key block of the
    // half), the partial sum, then P V^T accumulated into columns 0..31
    float sum = 0.f;
    for (int hh = 0; hh < halves; ++hh) {
      const int blk = 2 * hh + hf;  // this warp's P block
      if (hh > 0) {  // the previous half's MMA has read the P buffer
        ok = ok && mbar_wait(smem_u32(&o_done[0]), phase_o, abort);
        phase_o ^= 1;
        tc_fence_after();
      }
      if (blk < kblocks) {
        uint8_t* pb = ps + hf * AX_P_KB;
#pragma unroll 1
        for (int c0 = blk * 64; c0 < blk * 64 + 64; c0 += 32) {
          float sc[32];
          const bool live = ok && warp_live && c0 < kend;
          if (live) {
            tmem_ld32(taddr + c0, sc);
            // masked keys hold -inf and read 0
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const float p = ax_exp2(sc[jj] - m);
              sum += p;
              sc[jj] = p;
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) sc[jj] = 0.f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            store_vec<8>(reinterpret_cast<__nv_bfloat16*>(pb + swz(rl, ((c0 & 63) >> 3) + u)), sc + 8 * u);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();  // P written; this half's scores (and so columns 0..31 after half 0) are consumed
      if (tid == 0 && !*abort) {
        tc_fence_after();
        for (int kb2 = 2 * hh; kb2 < min(2 * hh + 2, kblocks); ++kb2) {
          const uint32_t a0 = smem_u32(ps + (kb2 & 1) * AX_P_KB), b0 = smem_u32(vt + kb2 * AX_VT_KB);
#pragma unroll
          for (int j = 0; j < 4; ++j) umma_i(tmem, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), AX_IDESC_O,
                                             (kb2 | j) != 0);
        }
        umma_commit(smem_u32(&o_done[0]));
      }
    }
    red_s[hf * 128 + rl] = sum;
    __syncthreads();
    ok = ok && (halves == 0 || mbar_wait(smem_u32(&o_done[0]), phase_o, abort));
    if (halves > 0) phase_o ^= 1;
    tc_fence_after();
    if (hf == 0) {
      float o[AX_D];
#pragma unroll
      for (int i = 0; i < AX_D; ++i) o[i] = 0.f;
      if (ok && warp_live) {
        const float tot = red_s[rl] + red_s[128 + rl];
        const float inv = tot > 0.f ? 1.f / tot : 0.f;
        tmem_ld32(taddr, o);
#pragma unroll
        for (int i = 0; i < AX_D; ++i) o[i] *= inv;
      }
      if (row < length) {
        if (row >= nv) {
#pragma unroll
          for (int i = 0; i < AX_D; ++i) o[i] = 0.f;
        }
        __nv_bfloat16* orow = ob + row * o_row;
#pragma unroll
        for (int i = 0; i < AX_D / 8; ++i) store_vec<8>(orow + 8 * i, o + 8 * i);
      }
    }
    tc_fence_before();
    __syncthreads();  // O read before the next tile's S overwrites it
    tc_fence_after();
  }
  // rows of tiles past the valid length (or every row without keys) read zero
  for (int r = n_tiles * 128 + tid; r < length; r += AX_THREADS) {
    float o[8] = {};
    __nv_bfloat16* orow = ob + r * o_row;
#pragma unroll
    for (int i = 0; i < AX_D / 8; ++i) store_vec<8>(orow + 8 * i, o);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AX_TMEM_COLS) : "memory");
  }
}

}  // namespace sm100
}  // namespace mb

using namespace mb;

extern "C" int mb_axial_attention(const void* q, const void* k, const void* v, int64_t n_pos, int heads,
                                  int head_dim, int64_t length, int64_t s_pos, int64_t s_head, int64_t s_row,
                                  const int32_t* coords, const int32_t* valid, const float* bias, void* out,
                                  int64_t o_pos, int64_t o_head, int64_t o_row, void* stream) {
  using namespace sm100;
  MB_REQUIRE(n_pos >= 0 && heads > 0, "axial_attention: bad sizes");
  MB_REQUIRE(head_dim == AX_D, "axial_attention: head_dim must be %d (got %d)", AX_D, head_dim);
  MB_REQUIRE(length > 0 && length <= AX_L, "axial_attention: length must be in [1, %d] (got %lld)", AX_L,
             (long long)length);
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(q && k && v && coords && valid && bias && out, "axial_attention: null pointer");
  MB_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16) &&
                 s_pos % 8 == 0 && s_head % 8 == 0 && s_row % 8 == 0 && o_pos % 8 == 0 && o_head % 8 == 0 &&
                 o_row % 8 == 0,
             "axial_attention: q/k/v/out rows must be 16-byte aligned");
  MB_REQUIRE(n_pos * heads <= INT32_MAX, "axial_attention: too many (position, head) pairs");
  auto kern = axial_attention_kernel;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AX_SMEM) != cudaSuccess)
    return fail(MB_LAUNCH_FAILED, "axial_attention: %d bytes of shared memory refused", AX_SMEM);
  kern<<<(unsigned)(n_pos * heads), AX_THREADS, AX_SMEM, as_stream(stream)>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, s_pos, s_head, s_row, heads,
      (int)length, coords, valid, bias, (__nv_bfloat16*)out, o_pos, o_head, o_row);
  return launch_status("axial_attention");
}
