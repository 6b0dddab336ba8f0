// Stone attention on the 5th-generation tensor cores (sm_100a tcgen05): the
// trunk's attention over each position's tokens [4 latents; stones]
// (reference model.py:621-669 through mantisnet::fused_attention,
// attention.py:44-162 / 892-904):
//
//   out[p,a,i] = sum_j softmax_j(q_i . k_j / sqrt(32)) v_j,  keys j < n_keys(p)
//
// head_dim 32, bf16 q/k/v, fp32 scores and softmax, up to 320 keys. One CTA
// per (position, head), eight warps. The position's K rows and V^T are
// staged in shared memory in the 128-byte-swizzled K-major layout the UMMA
// descriptors read; query rows go 128 at a time. Per query tile one thread
// issues S = Q K^T into TMEM (M=128, N up to 256 per instruction, two K=16
// steps); the warps split the keys in two halves, a thread holding one query
// row of one half (TMEM lane quadrant = warp % 4): a first pass finds the row
// maximum, a second writes exp(s - max) as bf16 into the P blocks and sums
// it; P V (M=128, N=32, K = keys in 64-key blocks) lands in its own TMEM
// columns and the row is scaled by 1 / sum and stored. Every mbarrier wait is
// bounded (see gemm_sm100.cu).
#include "common.cuh"

namespace mb {
namespace sm100 {

constexpr int ST_KEYS = 320;                      // most keys per position
constexpr int ST_D = 32;
constexpr int ST_THREADS = 256;
constexpr int ST_KB = ST_KEYS / 64;               // 64-key blocks
constexpr int ST_Q_BYTES = 128 * 128;             // one query tile, rows padded to 128 B
constexpr int ST_K_BYTES = ST_KEYS * 128;
constexpr int ST_VT_KB = ST_D * 128;              // 4 KB per 64-key block of V^T
constexpr int ST_P_KB = 128 * 128;                // 16 KB per 64-key block of P
constexpr int ST_Q_OFF = 0;
constexpr int ST_K_OFF = ST_Q_OFF + ST_Q_BYTES;
constexpr int ST_VT_OFF = ST_K_OFF + ST_K_BYTES;
constexpr int ST_P_OFF = ST_VT_OFF + ST_KB * ST_VT_KB;
constexpr int ST_RED_OFF = ST_P_OFF + ST_KB * ST_P_KB;
constexpr int ST_BAR_OFF = ST_RED_OFF + 2 * 128 * 4;
constexpr int ST_SMEM = ST_BAR_OFF + 64 + 1024;   // + alignment slack
constexpr int ST_O_COL = 384;                     // TMEM column of the P V accumulator
static_assert(ST_SMEM <= 232448, "stone attention shared memory exceeds 227 KB");

template <typename TO>
__global__ void __launch_bounds__(ST_THREADS, 1) stone_attention_tc_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, int64_t s_pos, int64_t s_head,
    int64_t s_row, const int32_t* __restrict__ seq_lens, int64_t t_pad, const int64_t* __restrict__ tok_off,
    int max_queries, int heads, TO* __restrict__ out, int64_t o_pos, int64_t o_head, int64_t o_row,
    float* __restrict__ lse, float scale) {
  extern __shared__ uint8_t st_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(st_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + ST_Q_OFF;
  uint8_t* ks = smem + ST_K_OFF;
  uint8_t* vt = smem + ST_VT_OFF;
  uint8_t* ps = smem + ST_P_OFF;
  float* red = reinterpret_cast<float*>(smem + ST_RED_OFF);  // [half][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST_BAR_OFF);
  uint64_t* s_done = bars;
  uint64_t* o_done = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 3);

  const int64_t p = blockIdx.x / heads;
  const int a = blockIdx.x % heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int64_t base_in, base_out, n_keys, n_rows;
  if (tok_off) {
    const int64_t t0 = tok_off[p];
    n_keys = tok_off[p + 1] - t0;
    n_rows = max_queries >= 0 && max_queries < n_keys ? max_queries : n_keys;
    base_in = t0 * s_row + a * s_head;
    base_out = (o_pos > 0 ? p * o_pos : t0 * o_row) + a * o_head;
  } else {
    n_keys = seq_lens[p];
    if (n_keys > t_pad) n_keys = t_pad;
    n_rows = t_pad;
    base_in = p * s_pos + a * s_head;
    base_out = p * o_pos + a * o_head;
  }
  if (n_keys < 0 || n_keys > ST_KEYS) {  // the host routes longer positions to the CUDA-core kernel
    if (tid == 0) report(ERR_RUN_BOUND);
    n_keys = n_keys < 0 ? 0 : ST_KEYS;
  }
  const int nk = (int)n_keys;
  const int kpad = (nk + 63) & ~63;   // keys covered by P and V^T blocks
  const int npad = (nk + 15) & ~15;   // S columns the MMA computes
  const int kend = (nk + 31) & ~31;   // S columns the softmax reads
  const __nv_bfloat16* qb = q + base_in;
  const __nv_bfloat16* kb = k + base_in;
  const __nv_bfloat16* vb = v + base_in;
  TO* ob = out + base_out;

  if (tid == 0) {
    mbar_init(smem_u32(s_done), 1);
    mbar_init(smem_u32(o_done), 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // ---- K rows and V^T of the position's keys (zero past n_keys)
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int idx = tid; idx < kpad * 4; idx += ST_THREADS) {
    const int r = idx >> 2, c = idx & 3;
    uint4 kv4 = zero, vv4 = zero;
    if (r < nk) {
      kv4 = __ldg(reinterpret_cast<const uint4*>(kb + r * s_row) + c);
      vv4 = __ldg(reinterpret_cast<const uint4*>(vb + r * s_row) + c);
    }
    *reinterpret_cast<uint4*>(ks + swz(r, c)) = kv4;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&vv4);
    const int blk = r >> 6, jj = r & 63;
#pragma unroll
    for (int w = 0; w < 8; ++w)
      *reinterpret_cast<__nv_bfloat16*>(vt + blk * ST_VT_KB + swz(8 * c + w, jj >> 3) + (jj & 7) * 2) = e[w];
  }
  tc_fence_before();
  __syncthreads();  // barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int qd = warp & 3, hf = warp >> 2;
  const int rl = qd * 32 + lane;
  // this half's S columns: 32-column loads, the halves together covering kpad
  const int units = kpad / 32;
  const int u_lo = hf == 0 ? 0 : (units + 1) / 2, u_hi = hf == 0 ? (units + 1) / 2 : units;
  const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16);
  bool ok = true;
  const int n_tiles = nk > 0 ? (int)((n_rows + 127) / 128) : 0;
  for (int t = 0; t < n_tiles; ++t) {
    // ---- this tile's query rows
    for (int idx = tid; idx < 128 * 4; idx += ST_THREADS) {
      const int r = idx >> 2, c = idx & 3;
      const int64_t row = (int64_t)t * 128 + r;
      uint4 q4 = zero;
      if (row < n_rows && row < nk) q4 = __ldg(reinterpret_cast<const uint4*>(qb + row * s_row) + c);
      *reinterpret_cast<uint4*>(qs + swz(r, c)) = q4;
    }
    fence_proxy_async();  // generic-proxy shared stores -> visible to the tensor cores
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && !*abort) {
      const uint32_t a0 = smem_u32(qs), b0 = smem_u32(ks);
      const int n1 = npad < 256 ? npad : 256;
#pragma unroll
      for (int j = 0; j < ST_D / 16; ++j)
        umma_i(tmem, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), idesc_f16(128, n1), j);
      if (npad > 256) {
#pragma unroll
        for (int j = 0; j < ST_D / 16; ++j)
          umma_i(tmem + 256, smem_desc(a0 + j * 32), smem_desc(b0 + 256 * 128 + j * 32), idesc_f16(128, npad - 256),
                 j);
      }
      umma_commit(smem_u32(s_done));
    }
    // pass 1: the half-row maximum of the scaled scores
    float m = -INFINITY, sum = 0.f;
    ok = ok && mbar_wait(smem_u32(s_done), t & 1, abort);
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int u = u_lo; u < u_hi; ++u) {
        const int c0 = u * 32;
        if (c0 >= kend) break;
        float sc[32];
        tmem_ld32(taddr + c0, sc);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (c0 + jj < nk) m = fmaxf(m, sc[jj] * scale);
      }
    }
    red[hf * 128 + rl] = m;
    __syncthreads();
    m = fmaxf(red[rl], red[128 + rl]);
    // pass 2: P = exp(s - m) in bf16 into the 64-key blocks, the half-row sum
#pragma unroll 1
    for (int u = u_lo; u < u_hi; ++u) {
      const int c0 = u * 32;
      float sc[32];
      if (ok && c0 < kend) tmem_ld32(taddr + c0, sc);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const float pv = (ok && c0 + jj < nk) ? __expf(sc[jj] * scale - m) : 0.f;
        sum += pv;
        sc[jj] = pv;
      }
      const int blk = c0 >> 6;
#pragma unroll
      for (int w = 0; w < 4; ++w)
        store_vec<8>(reinterpret_cast<__nv_bfloat16*>(ps + blk * ST_P_KB + swz(rl, ((c0 & 63) >> 3) + w)),
                     sc + 8 * w);
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();  // maxima read, P written, S consumed
    red[hf * 128 + rl] = sum;
    if (tid == 0 && !*abort) {
      tc_fence_after();
      for (int blk = 0; blk < kpad / 64; ++blk) {
        const uint32_t a0 = smem_u32(ps + blk * ST_P_KB), b0 = smem_u32(vt + blk * ST_VT_KB);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          umma_i(tmem + ST_O_COL, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), idesc_f16(128, ST_D),
                 (blk | j) != 0);
      }
      umma_commit(smem_u32(o_done));
    }
    __syncthreads();  // sums written
    if (hf == 0) {
      float o[ST_D];
#pragma unroll
      for (int i = 0; i < ST_D; ++i) o[i] = 0.f;
      const int64_t row = (int64_t)t * 128 + rl;
      ok = ok && mbar_wait(smem_u32(o_done), t & 1, abort);
      tc_fence_after();
      float row_lse = 0.f;
      if (ok) {
        tmem_ld32(taddr + ST_O_COL, o);
        const float tot = red[rl] + red[128 + rl];
        const float inv = tot > 0.f ? 1.f / tot : 0.f;
#pragma unroll
        for (int i = 0; i < ST_D; ++i) o[i] *= inv;
        if (tot > 0.f) row_lse = m + logf(tot);
      }
      // log-sum-exp of the scaled scores (0 for a padded query row), padded layout (P, heads, t_pad)
      if (lse && !tok_off && row < n_rows) lse[(p * heads + a) * t_pad + row] = row < nk ? row_lse : 0.f;
      if (row < n_rows) {
        if (row >= nk) {  // padded query rows read zero
#pragma unroll
          for (int i = 0; i < ST_D; ++i) o[i] = 0.f;
        }
        TO* orow = ob + row * o_row;
#pragma unroll
        for (int i = 0; i < ST_D / 8; ++i) store_vec<8>(orow + 8 * i, o + 8 * i);
      }
    }
    tc_fence_before();
    __syncthreads();  // O read before the next tile's MMAs
    tc_fence_after();
  }
  if (n_tiles == 0 && !tok_off) {
    // a padded position without keys: every query row reads zero
    for (int64_t row = tid; row < n_rows; row += ST_THREADS) {
      float o[ST_D] = {};
      TO* orow = ob + row * o_row;
#pragma unroll
      for (int i = 0; i < ST_D / 8; ++i) store_vec<8>(orow + 8 * i, o + 8 * i);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace sm100
}  // namespace mb

using namespace mb;

// The tensor-core path of mb_stone_attention (bf16 q/k/v, head_dim 32, at
// most 320 keys per position); returns -1 when the shape is not one it takes.
static int stone_attention_tc(const void* q, const void* k, const void* v, int dtype, int64_t n_pos, int heads,
                              int head_dim, int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* seq_lens,
                              int64_t t_pad, const int64_t* tok_off, int64_t max_tokens, int max_queries, void* out,
                              int out_dtype, int64_t o_pos, int64_t o_head, int64_t o_row, float* lse,
                              cudaStream_t s) {
  using namespace sm100;
  const int64_t keys = tok_off ? max_tokens : t_pad;
  if (dtype != MB_BF16 || head_dim != ST_D || keys > ST_KEYS || n_pos * heads > INT32_MAX) return -1;
  if (!(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16) && s_pos % 8 == 0 &&
        s_head % 8 == 0 && s_row % 8 == 0 && o_pos % 8 == 0 && o_head % 8 == 0 && o_row % 8 == 0))
    return -1;
  const float scale = 1.f / sqrtf((float)head_dim);
  int rc = MB_OK;
  MB_DISPATCH_T(out_dtype, TO, [&] {
    auto kern = stone_attention_tc_kernel<TO>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, ST_SMEM) != cudaSuccess) {
      rc = fail(MB_LAUNCH_FAILED, "stone_attention: %d bytes of shared memory refused", ST_SMEM);
      return;
    }
    kern<<<(unsigned)(n_pos * heads), ST_THREADS, ST_SMEM, s>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, s_pos, s_head, s_row, seq_lens,
        t_pad, tok_off, max_queries, heads, (TO*)out, o_pos, o_head, o_row, lse, scale);
  });
  if (rc != MB_OK) return rc;
  return launch_status("stone_attention");
}
