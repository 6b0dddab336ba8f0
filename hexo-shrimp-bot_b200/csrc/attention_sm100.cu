// Axial-bias cell-token attention on the 5th-generation tensor cores
// (sm_100a tcgen05): per position b and head h over L <= 256 tokens,
//
//   out[b,h,i] = softmax_j( q_i . k_j / sqrt(32) + bias[dq+16, dr+16, h] ) v_j
//   dq = clamp(q-coord of key j - q-coord of query i, -16, 16), dr likewise,
//
// keys j < valid[b] only; query rows i >= valid[b] are written as zeros.
// head_dim 32, bf16 q/k/v/out, fp32 scores and softmax.
//
// One CTA per (position, head), 16 warps. Q, K and V^T are staged in shared
// memory in the 128-byte-swizzled K-major layout the UMMA descriptors read
// (Q and K rows carry the 32 head columns in the first 64 bytes). One thread
// issues S = Q K^T for both 128-query tiles into TMEM (M=128, N=256, two
// K=16 steps each). The warps split each live tile's keys into parts (two
// parts per tile when both tiles are live, else four): a thread holds one
// query row of one part (TMEM lane quadrant = warp % 4). A first pass adds
// the offset bias, writes the biased scores back into TMEM and finds the part
// maximum; the parts' maxima meet in shared memory; a second pass writes
// exp(x - max) as bf16 into the P tile and sums it. P V^T (M=128, N=32,
// K up to 256) then lands in the tile's own, now consumed, TMEM columns, and
// the row is scaled by 1/sum and stored. Work is bounded by each position's
// valid length. Every mbarrier wait is bounded (see gemm_sm100.cu).
#include "common.cuh"

namespace mb {
namespace sm100 {

constexpr int AX_L = 256;          // tokens per position (maximum)
constexpr int AX_D = 32;           // head dim
constexpr int AX_SPAN = 33;        // relative offsets -16..16
constexpr int AX_THREADS = 512;
constexpr int AX_Q_BYTES = AX_L * 128;           // 32 KB, rows padded to 128 B
constexpr int AX_K_BYTES = AX_L * 128;           // 32 KB
constexpr int AX_VT_KB = AX_D * 128;             // 4 KB per 64-key block of V^T (32 rows)
constexpr int AX_VT_BYTES = 4 * AX_VT_KB;        // 16 KB
constexpr int AX_P_KB = 128 * 128;               // 16 KB per 64-key block of a P tile
constexpr int AX_P_BYTES = 4 * AX_P_KB;          // 64 KB per tile
constexpr int AX_Q_OFF = 0;
constexpr int AX_K_OFF = AX_Q_OFF + AX_Q_BYTES;
constexpr int AX_VT_OFF = AX_K_OFF + AX_K_BYTES;
constexpr int AX_P_OFF = AX_VT_OFF + AX_VT_BYTES;
constexpr int AX_BIAS_OFF = AX_P_OFF + 2 * AX_P_BYTES;
constexpr int AX_COORD_OFF = AX_BIAS_OFF + 4400;  // 33*33 floats, rounded up
constexpr int AX_RED_OFF = AX_COORD_OFF + AX_L * 8;  // per-row half maxima / sums
constexpr int AX_BAR_OFF = AX_RED_OFF + 2 * 2 * 128 * 4;
constexpr int AX_SMEM = AX_BAR_OFF + 64 + 1024;   // + alignment slack
static_assert(AX_SMEM <= 232448, "axial attention shared memory exceeds 227 KB");

constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
constexpr uint32_t AX_IDESC_S = idesc_f16(128, AX_L);
constexpr uint32_t AX_IDESC_O = idesc_f16(128, AX_D);

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

__global__ void __launch_bounds__(AX_THREADS, 1) axial_attention_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    int64_t s_pos, int64_t s_head, int64_t s_row, int heads, int length, const int32_t* __restrict__ coords,
    const int32_t* __restrict__ valid, const float* __restrict__ bias, __nv_bfloat16* __restrict__ out,
    int64_t o_pos, int64_t o_head, int64_t o_row) {
  extern __shared__ uint8_t ax_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ax_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + AX_Q_OFF;
  uint8_t* ks = smem + AX_K_OFF;
  uint8_t* vt = smem + AX_VT_OFF;
  uint8_t* ps = smem + AX_P_OFF;
  float* bias_s = reinterpret_cast<float*>(smem + AX_BIAS_OFF);
  int2* kc = reinterpret_cast<int2*>(smem + AX_COORD_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AX_BAR_OFF);
  uint64_t* s_done = bars;       // [2]
  uint64_t* o_done = bars + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 5);

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
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s_done[i]), 1);
      mbar_init(smem_u32(&o_done[i]), 1);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // ---- stage Q, K (4 logical 16-byte chunks per row), V^T, bias, key coords.
  // Every global load of the thread is issued before the first shared store.
  constexpr int PER = AX_L * 4 / AX_THREADS;  // 16-byte chunks of Q (and of K, V) per thread
  constexpr int BPER = (AX_SPAN * AX_SPAN + AX_THREADS - 1) / AX_THREADS;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  uint4 qv[PER], kv[PER], vv[PER];
  float bv[BPER];
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
  for (int u = 0; u < BPER; ++u) {
    const int idx = tid + u * AX_THREADS;
    bv[u] = idx < AX_SPAN * AX_SPAN ? __ldg(bias + (int64_t)idx * heads + h) : 0.f;
  }
  const int2 kcv = tid < length && tid < AX_L ? make_int2(__ldg(cb + 2 * tid), __ldg(cb + 2 * tid + 1))
                                              : make_int2(0, 0);
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int idx = tid + u * AX_THREADS, r = idx >> 2, c = idx & 3;
    *reinterpret_cast<uint4*>(qs + swz(r, c)) = qv[u];
    *reinterpret_cast<uint4*>(ks + swz(r, c)) = kv[u];
    // V row r, columns 8c..8c+7 -> V^T rows 8c..8c+7, column r
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&vv[u]);
    const int blk = r >> 6, jj = r & 63;
#pragma unroll
    for (int w = 0; w < 8; ++w)
      *reinterpret_cast<__nv_bfloat16*>(vt + blk * AX_VT_KB + swz(8 * c + w, jj >> 3) + (jj & 7) * 2) = e[w];
  }
#pragma unroll
  for (int u = 0; u < BPER; ++u) {
    const int idx = tid + u * AX_THREADS;
    if (idx < AX_SPAN * AX_SPAN) bias_s[idx] = bv[u];
  }
  if (tid < AX_L) kc[tid] = kcv;
  fence_proxy_async();  // generic-proxy shared stores -> visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- S = Q K^T for each live query tile
  if (tid == 0) {
    for (int t = 0; t < n_tiles; ++t) {
      const uint32_t d = tmem + t * AX_L;
      const uint32_t a0 = smem_u32(qs + t * 128 * 128), b0 = smem_u32(ks);
#pragma unroll
      for (int j = 0; j < AX_D / 16; ++j) umma_i(d, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), AX_IDESC_S, j);
      umma_commit(smem_u32(&s_done[t]));
    }
  }

  // Warp roles: tile t = warp / 8 (queries 128t..128t+127), key half hf =
  // (warp / 4) % 2 (keys 128hf..128hf+127), TMEM lane quadrant qd = warp % 4
  // (rows 32qd..32qd+31 of the tile); a thread owns one query row of one half.
  // With one live query tile all sixteen warps work on it in four key parts;
  // with two, eight warps per tile in two parts.
  const int NP = n_tiles == 2 ? 2 : 4;
  const int t = warp / (4 * NP), hf = (warp >> 2) % NP, qd = warp & 3;
  const int row = t * 128 + qd * 32 + lane;  // this thread's query
  const int rl = qd * 32 + lane;             // row within the tile
  const float scale = 0.17677669529663687f;  // 1 / sqrt(32)
  // Work is bounded by the valid length: score columns up to nv rounded to a
  // 32-column load, P and the P V product up to nv rounded to a 64-key block,
  // and warps whose 32 queries all lie past nv skip the softmax (their rows
  // are written as zeros). TMEM loads are warp-collective, so the bound is
  // per warp.
  const int kend = min(AX_L, (nv + 31) & ~31);
  const int kblocks = (nv + 63) >> 6;
  const bool warp_live = t < n_tiles && t * 128 + qd * 32 < nv;
  // this part's keys: a multiple of 32, parts together covering kblocks * 64
  const int span = ((kend + NP * 32 - 1) / (NP * 32)) * 32;
  const int c_lo = hf * span, c_hi = min(c_lo + span, kend), p_hi = min(c_lo + span, kblocks * 64);
  const int nthr = 128 * NP;  // threads of this tile's group
  float* red = reinterpret_cast<float*>(smem + AX_RED_OFF);  // [tile][part][128 rows]
  float* red_t = red + t * NP * 128;
  bool ok = true;
  float m = -INFINITY, sum = 0.f;
  const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16) + t * AX_L;
  if (warp_live) {
    ok = mbar_wait(smem_u32(&s_done[t]), 0, abort);
    tc_fence_after();
    const int2 qc = row < length ? make_int2(__ldg(cb + 2 * row), __ldg(cb + 2 * row + 1)) : make_int2(0, 0);
    // pass 1: biased scores back into TMEM, the half-row maximum
    if (ok) {
#pragma unroll 1
      for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        float s[32];
        tmem_ld32(taddr + c0, s);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = c0 + jj;
          const int2 c = kc[j];
          const int dq = min(max(c.x - qc.x, -16), 16) + 16, dr = min(max(c.y - qc.y, -16), 16) + 16;
          s[jj] = j < nv ? s[jj] * scale + bias_s[dq * AX_SPAN + dr] : -INFINITY;
          m = fmaxf(m, s[jj]);
        }
        tmem_st32(taddr + c0, s);
      }
      tmem_st_wait();
    }
    red_t[hf * 128 + rl] = m;
  }
  asm volatile("bar.sync %0, %1;" ::"r"(1 + t), "r"(nthr) : "memory");
  if (warp_live) {
    for (int pp = 0; pp < NP; ++pp) m = fmaxf(m, red_t[pp * 128 + rl]);
    // pass 2: P = exp(x - m) in bf16 into the tile's P blocks, the half-row sum
    uint8_t* pt = ps + t * AX_P_BYTES;
#pragma unroll 1
    for (int c0 = c_lo; c0 < p_hi; c0 += 32) {
      float s[32];
      if (ok && c0 < c_hi) tmem_ld32(taddr + c0, s);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const float p = (ok && c0 + jj < nv) ? __expf(s[jj] - m) : 0.f;
        sum += p;
        s[jj] = p;
      }
      const int blk = c0 >> 6;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        store_vec<8>(reinterpret_cast<__nv_bfloat16*>(pt + blk * AX_P_KB + swz(rl, ((c0 & 63) >> 3) + u)), s + 8 * u);
    }
    fence_proxy_async();
    tc_fence_before();
  }
  // the maxima are read; the sums reuse the same slots after the barrier
  asm volatile("bar.sync %0, %1;" ::"r"(1 + t), "r"(nthr) : "memory");
  if (warp_live) red_t[hf * 128 + rl] = sum;
  asm volatile("bar.sync %0, %1;" ::"r"(1 + t), "r"(nthr) : "memory");
  // the tile's eight warps have written P and read all of S: O may overwrite S
  if (t < n_tiles && hf == 0 && qd == 0 && lane == 0) {
    tc_fence_after();
    const uint32_t d = tmem + t * AX_L;
    for (int blk = 0; blk < kblocks; ++blk) {
      const uint32_t a0 = smem_u32(ps + t * AX_P_BYTES + blk * AX_P_KB), b0 = smem_u32(vt + blk * AX_VT_KB);
#pragma unroll
      for (int j = 0; j < 4; ++j) umma_i(d, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), AX_IDESC_O, (blk | j) != 0);
    }
    umma_commit(smem_u32(&o_done[t]));
  }
  if (hf == 0) {
    float o[AX_D];
#pragma unroll
    for (int i = 0; i < AX_D; ++i) o[i] = 0.f;
    if (warp_live && ok) {
      float tot = 0.f;
      for (int pp = 0; pp < NP; ++pp) tot += red_t[pp * 128 + rl];
      const float inv = tot > 0.f ? 1.f / tot : 0.f;
      if (mbar_wait(smem_u32(&o_done[t]), 0, abort)) {
        tc_fence_after();
        tmem_ld32(taddr, o);
#pragma unroll
        for (int i = 0; i < AX_D; ++i) o[i] *= inv;
      }
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
  } else if (NP == 4 && hf == 1) {
    // fewer than two live tiles: every warp worked on tile 0, so these warps
    // write tile 1's rows, all past the valid length, as zeros
    const int zrow = 128 + qd * 32 + lane;
    if (zrow < length) {
      float o[8] = {};
      __nv_bfloat16* orow = ob + zrow * o_row;
#pragma unroll
      for (int i = 0; i < AX_D / 8; ++i) store_vec<8>(orow + 8 * i, o);
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
