// Attention kernels of the MantisNet trunk (CUDA cores, fp32 math):
//
//  K3  typed segment attention (cells<-windows, cells<-stones radius,
//      windows<-cells, cell adjacency): one warp per query row covering every
//      head; lane l holds VEC columns, lanes_per_head = head_dim / VEC lanes
//      share one head; two edges per iteration. The grouped form (radius
//      read) stages each position's sources in shared memory and rescales
//      once per chunk of eight edges.
//  K4  window-latent read (a cluster of CTAs per position, merged through
//      distributed shared memory), broadcast (warp per window) and the
//      dense 4x4 latent mix.
//  K1  stone attention over [4 latents; stones] per position: one thread per
//      query row, K/V tiles staged in shared memory as fp32 and read by
//      broadcast, online softmax in chunks of 8 keys.
//
// Scores use exp(x - running max); an empty run returns zero with l = 0.
#include <math.h>

#include <algorithm>
#include <type_traits>

#include <cooperative_groups.h>

#include "common.cuh"

namespace mb {

constexpr float kNegInf = -INFINITY;

// ------------------------------------------------------- row loads
// VEC elements of T as loaded from memory, unpacked to fp32 on use.
template <typename T, int VEC> struct Raw;
template <int VEC> struct Raw<float, VEC> { float w[VEC]; };
template <int VEC> struct Raw<__nv_bfloat16, VEC> { uint32_t w[VEC >= 2 ? VEC / 2 : 1]; };

template <bool SMEM, int VEC>
__device__ __forceinline__ void raw_load(const float* p, Raw<float, VEC>& r) {
  if constexpr (VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC / 4; ++i) {
      const float4 f = SMEM ? reinterpret_cast<const float4*>(p)[i] : __ldg(reinterpret_cast<const float4*>(p) + i);
      r.w[4 * i] = f.x; r.w[4 * i + 1] = f.y; r.w[4 * i + 2] = f.z; r.w[4 * i + 3] = f.w;
    }
  } else if constexpr (VEC == 2) {
    const float2 f = SMEM ? *reinterpret_cast<const float2*>(p) : __ldg(reinterpret_cast<const float2*>(p));
    r.w[0] = f.x; r.w[1] = f.y;
  } else {
    r.w[0] = SMEM ? *p : __ldg(p);
  }
}
template <bool SMEM, int VEC>
__device__ __forceinline__ void raw_load(const __nv_bfloat16* p, Raw<__nv_bfloat16, VEC>& r) {
  if constexpr (VEC % 8 == 0) {
#pragma unroll
    for (int i = 0; i < VEC / 8; ++i) {
      const uint4 u = SMEM ? reinterpret_cast<const uint4*>(p)[i] : __ldg(reinterpret_cast<const uint4*>(p) + i);
      r.w[4 * i] = u.x; r.w[4 * i + 1] = u.y; r.w[4 * i + 2] = u.z; r.w[4 * i + 3] = u.w;
    }
  } else if constexpr (VEC == 4) {
    const uint2 u = SMEM ? *reinterpret_cast<const uint2*>(p) : __ldg(reinterpret_cast<const uint2*>(p));
    r.w[0] = u.x; r.w[1] = u.y;
  } else if constexpr (VEC == 2) {
    r.w[0] = SMEM ? *reinterpret_cast<const uint32_t*>(p) : __ldg(reinterpret_cast<const unsigned int*>(p));
  } else {
    const unsigned short b = SMEM ? *reinterpret_cast<const unsigned short*>(p)
                                  : __ldg(reinterpret_cast<const unsigned short*>(p));
    r.w[0] = (uint32_t)b;
  }
}
template <int VEC>
__device__ __forceinline__ void raw_unpack(const Raw<float, VEC>& r, float* out) {
#pragma unroll
  for (int i = 0; i < VEC; ++i) out[i] = r.w[i];
}
template <int VEC>
__device__ __forceinline__ void raw_unpack(const Raw<__nv_bfloat16, VEC>& r, float* out) {
  if constexpr (VEC >= 2) {
#pragma unroll
    for (int i = 0; i < VEC / 2; ++i) {
      out[2 * i] = __uint_as_float(r.w[i] << 16);
      out[2 * i + 1] = __uint_as_float(r.w[i] & 0xffff0000u);
    }
  } else {
    out[0] = __uint_as_float(r.w[0] << 16);
  }
}

// Sum over aligned groups of LPH lanes; LPH == 0 reads the group from `lph`.
template <int LPH>
__device__ __forceinline__ float head_sum(float x, int lph) {
  if constexpr (LPH > 0) {
#pragma unroll
    for (int o = LPH >> 1; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
  } else {
    return group_sum(x, lph);
  }
}

// ------------------------------------------------------- segment attention
// One warp per batch of kSegRows consecutive query rows (blocks of 2 warps,
// scheduled in row order, so the GPU works on a narrow band of positions at a
// time and the gathered source rows stay L2-resident). A lane holds VEC
// columns of a row; the warp covers the row's full width.
//
// The warp walks its rows' edges as one stream (the rows are consecutive, so
// their edges are one contiguous CSR range): kSegEdges edges at a time, it
// requests all their K, V and class value rows before using any, and switches
// row state whenever the stream crosses a run bound. Every query row and the
// run bounds are requested together at the start, and the edge indices come
// 32 at a time by one coalesced load, broadcast by shuffle. A row with few
// edges (the incidence reads average 2.5 and 4.9) so no longer costs a
// dependent round trip of its own. Edge order, and so the fp32 arithmetic,
// is the one of a per-row loop.
constexpr int kSegWarps = 2;   // small blocks: a block's slot frees as soon as its 2 warps finish
constexpr int kSegRows = 4;
// Edges requested together: 4 for 16-bit rows, 2 for fp32 rows of 4 or more
// columns per lane (whose raw rows take twice the registers). At 8 columns
// per lane that is ~125 registers: 8 blocks (16 warps) per SM there, 10 at
// narrower lanes.
template <typename T, int VEC> constexpr int seg_edges() { return sizeof(T) == 4 && VEC >= 4 ? 2 : 4; }
template <int VEC> constexpr int seg_blocks_per_sm() { return VEC >= 8 ? 8 : 10; }

template <typename T, typename TO, typename TV, int VEC, bool HAS_VCLS>
__global__ void __launch_bounds__(kSegWarps * 32, seg_blocks_per_sm<VEC>()) segment_attention_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, const T* __restrict__ v, int64_t ldkv, int64_t n_q,
    int64_t n_src, int heads, int hd, const float* __restrict__ bias, int64_t n_cls, const TV* __restrict__ vcls,
    const int64_t* __restrict__ seg_ptr, const int64_t* __restrict__ src, const int64_t* __restrict__ cls,
    const int64_t* __restrict__ skip_ptr, TO* __restrict__ out, int64_t ldo, float* __restrict__ m_out,
    float* __restrict__ l_out, float scale) {
  const int64_t row0 = ((int64_t)blockIdx.x * kSegWarps + (threadIdx.x >> 5)) * kSegRows;
  if (row0 >= n_q) return;
  const int lane = threadIdx.x & 31;
  const int nrows = (int)(n_q - row0 < kSegRows ? n_q - row0 : kSegRows);
  const int lph = hd / VEC;  // lanes per head
  const int head = lane / lph;
  const int H = heads * hd;
  const int col = lane * VEC;
  // Widths below one warp (H < 32, VEC == 1) leave the upper lanes idle; they
  // still join the shuffles with zero partial sums.
  const bool live = col < H;
  const float* brow = bias + (int64_t)(live ? head : 0) * n_cls;
  // lane i holds the batch's run bound i and whether row i is skipped
  const int64_t bound = lane <= nrows ? seg_ptr[row0 + lane] : 0;
  int skipped = 0;
  if (skip_ptr && lane < nrows) skipped = skip_ptr[row0 + lane + 1] > skip_ptr[row0 + lane];
  Raw<T, VEC> qr[kSegRows];
#pragma unroll
  for (int r = 0; r < kSegRows; ++r) {
    if (live && r < nrows) raw_load<false, VEC>(q + (row0 + r) * ldq + col, qr[r]);
    else qr[r] = Raw<T, VEC>{};
  }
  const int64_t e0 = __shfl_sync(0xffffffffu, bound, 0), e1 = __shfl_sync(0xffffffffu, bound, nrows);

  // Edge indices [eb, eb + 32): lane i holds edge eb + i (source -1: none, or
  // out of range, which is reported once here and the edge skipped).
  int64_t eb = e0;
  int my_src = -1, my_cls = 0;
  auto refill = [&](int64_t base) {
    eb = base;
    my_src = -1;
    my_cls = 0;
    const int64_t e = base + lane;
    if (e < e1) {
      const int64_t s_ = src[e], c_ = cls[e];
      if (s_ < 0 || s_ >= n_src || c_ < 0 || c_ >= n_cls) {
        report(ERR_INDEX);
      } else {
        my_src = (int)s_;
        my_cls = (int)c_;
      }
    }
  };
  refill(e0);

  int r = 0;
  int64_t rend = 0;
  int rskip = 0;
  float qf[VEC], acc[VEC], m = kNegInf, l = 0.f;
  auto start_row = [&](int rr) {  // rr is warp-uniform
    Raw<T, VEC> sel = qr[0];
#pragma unroll
    for (int i = 1; i < kSegRows; ++i)
      if (rr == i) sel = qr[i];
    raw_unpack(sel, qf);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      qf[i] *= scale;
      acc[i] = 0.f;
    }
    m = kNegInf;
    l = 0.f;
    rend = __shfl_sync(0xffffffffu, bound, rr + 1);
    rskip = __shfl_sync(0xffffffffu, skipped, rr);
  };
  auto finish_row = [&](int rr) {
    const float inv = l > 0.f ? 1.f / l : 1.f;
    float o[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = acc[i] * inv;
    if (live) {
      const int64_t row = row0 + rr;
      store_vec<VEC>(out + row * ldo + col, o);
      if (m_out && (lane % lph) == 0) {
        m_out[row * heads + head] = m;
        l_out[row * heads + head] = l;
      }
    }
  };
  start_row(0);

  constexpr int kSegEdges = seg_edges<T, VEC>();
  for (int64_t e = e0; e < e1; e += kSegEdges) {
    if (e + kSegEdges > eb + 32) refill(e);  // warp-uniform
    int sj[kSegEdges], cj[kSegEdges];
    Raw<T, VEC> kr[kSegEdges], vr[kSegEdges];
    Raw<TV, VEC> cr[kSegEdges];
#pragma unroll
    for (int j = 0; j < kSegEdges; ++j) {
      const int at = (int)(e - eb) + j;
      sj[j] = __shfl_sync(0xffffffffu, my_src, at);
      cj[j] = __shfl_sync(0xffffffffu, my_cls, at);
      if (live && sj[j] >= 0) {
        raw_load<false, VEC>(k + (int64_t)sj[j] * ldkv + col, kr[j]);
        raw_load<false, VEC>(v + (int64_t)sj[j] * ldkv + col, vr[j]);
        if constexpr (HAS_VCLS) raw_load<false, VEC>(vcls + (int64_t)cj[j] * H + col, cr[j]);
      } else {
        kr[j] = Raw<T, VEC>{};
        vr[j] = Raw<T, VEC>{};
        if constexpr (HAS_VCLS) cr[j] = Raw<TV, VEC>{};
      }
    }
#pragma unroll
    for (int j = 0; j < kSegEdges; ++j) {
      if (e + j >= e1) break;
      while (e + j >= rend) {  // the stream crossed into the next row(s)
        finish_row(r);
        ++r;
        start_row(r);
      }
      if (rskip || sj[j] < 0) continue;
      float kv_[VEC], vv[VEC];
      raw_unpack(kr[j], kv_);
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) d += qf[i] * kv_[i];
      d = group_sum(d, lph) + __ldg(brow + cj[j]);
      raw_unpack(vr[j], vv);
      if constexpr (HAS_VCLS) {
        float a[VEC];
        raw_unpack(cr[j], a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) vv[i] += a[i];
      }
      const float m_new = fmaxf(m, d);
      const float corr = __expf(m - m_new);
      const float p = __expf(d - m_new);
      l = l * corr + p;
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] = acc[i] * corr + p * vv[i];
      m = m_new;
    }
  }
  for (;;) {
    finish_row(r);
    if (++r >= nrows) break;
    start_row(r);
  }
}

// ---------------------------------------- grouped (source-staged) segment
// When query rows and sources split into aligned groups (the radius read:
// a position's cells attend only to that position's stones), one CTA takes
// one group and one 64-column block (whole heads): it copies the group's K|V
// columns, the class value rows and the bias rows into shared memory once,
// so every gathered source row is a conflict-free shared-memory read instead
// of an L2 round trip. Eight lanes hold one query row (8 bf16 columns each),
// a warp carries four rows and a CTA 16 warps. Edges go in chunks of eight:
// the row's lanes fetch the chunk's indices at once and broadcast them by
// shuffle, a first pass scores every edge of the chunk, and a second pass
// rescales the running state once and accumulates the value rows. Nothing
// is held in registers across the passes but the scores and the packed
// indices, so 32 warps fit on an SM to hide the shared-memory latency.
constexpr int kGrpCols = 64;
constexpr int kGrpWarps = 16;
constexpr int kGrpChunk = 8;
constexpr int kGrpClsBits = 11;  // packed edge: local source << 11 | class
constexpr int kGrpKvRowBytes = 2 * kGrpCols * 2;  // K then V, bf16

template <typename TV>
__host__ __device__ constexpr int grp_vcls_bytes(int64_t n_cls) {
  return (int)(((n_cls * kGrpCols * (int64_t)sizeof(TV)) + 15) / 16 * 16);
}
__host__ __device__ constexpr int grp_bias_bytes(int heads_in_block, int64_t n_cls) {
  return (int)((heads_in_block * n_cls * 4 + 15) / 16 * 16);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// One chunk-by-chunk pass over the four rows a warp holds. Source r's K and V
// columns are at kb + r * ld and vb + r * ld (offset by the lane's column).
template <int LPH, bool KV_SMEM, bool HAS_VCLS, typename TV>
__device__ __forceinline__ void grouped_rows(const float (&qv)[8], int64_t beg, int n, int nmax,
                                             const int64_t* __restrict__ src, const int64_t* __restrict__ cls,
                                             int64_t s0, int64_t ns, int64_t n_cls, const __nv_bfloat16* kb,
                                             const __nv_bfloat16* vb, int64_t ld, const float* brow, const TV* vc,
                                             int lph, float& m, float& l, float (&acc)[8]) {
  const int lane = threadIdx.x & 31;
  const int g0 = lane & ~7, li = lane & 7;
  for (int j0 = 0; j0 < nmax; j0 += kGrpChunk) {
    int mine = -1;
    if (j0 + li < n) {
      const int64_t s = src[beg + j0 + li] - s0, c = cls[beg + j0 + li];
      if ((uint64_t)s < (uint64_t)ns && (uint64_t)c < (uint64_t)n_cls) mine = (int)(s << kGrpClsBits | c);
      else report(ERR_INDEX);
    }
    const int steps = min(kGrpChunk, nmax - j0);
    int pk[kGrpChunk];
    float sc[kGrpChunk];
    float cmax = kNegInf;
#pragma unroll
    for (int j = 0; j < kGrpChunk; ++j) {
      pk[j] = -1;
      sc[j] = kNegInf;
      if (j < steps) {
        pk[j] = __shfl_sync(0xffffffffu, mine, g0 + j);
        float d = 0.f;
        if (pk[j] >= 0) {
          Raw<__nv_bfloat16, 8> kr;
          raw_load<KV_SMEM, 8>(kb + (int64_t)(pk[j] >> kGrpClsBits) * ld, kr);
          float kk[8];
          raw_unpack<8>(kr, kk);
#pragma unroll
          for (int i = 0; i < 8; ++i) d += qv[i] * kk[i];
        }
        d = head_sum<LPH>(d, lph);
        if (pk[j] >= 0) {
          sc[j] = d + brow[pk[j] & ((1 << kGrpClsBits) - 1)];
          cmax = fmaxf(cmax, sc[j]);
        }
      }
    }
    if (cmax != kNegInf) {
      const float m_new = fmaxf(m, cmax);
      const float corr = __expf(m - m_new);
      l *= corr;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= corr;
#pragma unroll
      for (int j = 0; j < kGrpChunk; ++j) {
        if (j < steps && pk[j] >= 0) {
          const float p = __expf(sc[j] - m_new);
          l += p;
          Raw<__nv_bfloat16, 8> vr;
          raw_load<KV_SMEM, 8>(vb + (int64_t)(pk[j] >> kGrpClsBits) * ld, vr);
          float vv[8];
          raw_unpack<8>(vr, vv);
          if constexpr (HAS_VCLS) {
            Raw<TV, 8> cr;
            raw_load<true, 8>(vc + (int64_t)(pk[j] & ((1 << kGrpClsBits) - 1)) * kGrpCols, cr);
            float a[8];
            raw_unpack<8>(cr, a);
#pragma unroll
            for (int i = 0; i < 8; ++i) vv[i] += a[i];
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += p * vv[i];
        }
      }
      m = m_new;
    }
  }
}

template <typename TO, typename TV, int LPH, bool HAS_VCLS>
__global__ void __launch_bounds__(kGrpWarps * 32, 2) segment_attention_grouped_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, int64_t ldkv, int64_t n_q, int64_t n_src, int hd,
    const float* __restrict__ bias, int64_t n_cls, const TV* __restrict__ vcls, int64_t ld_vcls,
    const int64_t* __restrict__ seg_ptr, const int64_t* __restrict__ src, const int64_t* __restrict__ cls,
    const int64_t* __restrict__ skip_ptr, const int64_t* __restrict__ q_off, const int64_t* __restrict__ s_off,
    int stage_rows, TO* __restrict__ out, int64_t ldo, float scale) {
  extern __shared__ __align__(16) unsigned char grp_smem[];
  unsigned char* smem = grp_smem;
  const int grp = blockIdx.x;
  const int cb = blockIdx.y * kGrpCols;
  const int nh = kGrpCols / hd;
  const int64_t q0 = q_off[grp], q1 = q_off[grp + 1], s0 = s_off[grp], s1 = s_off[grp + 1];
  if (q0 < 0 || q1 < q0 || q1 > n_q || s0 < 0 || s1 < s0 || s1 > n_src || s1 - s0 >= (int64_t(1) << 20)) {
    if (threadIdx.x == 0) report(ERR_RUN_BOUND);
    return;
  }
  if (q1 == q0) return;
  const int64_t ns = s1 - s0;
  const bool staged = ns <= stage_rows;

  float* bias_s = reinterpret_cast<float*>(smem);
  TV* vcls_s = reinterpret_cast<TV*>(smem + grp_bias_bytes(nh, n_cls));
  __nv_bfloat16* kv_s = reinterpret_cast<__nv_bfloat16*>(smem + grp_bias_bytes(nh, n_cls) +
                                                         (HAS_VCLS ? grp_vcls_bytes<TV>(n_cls) : 0));
  const int head0 = cb / hd;
  for (int64_t i = threadIdx.x; i < nh * n_cls; i += blockDim.x) bias_s[i] = bias[head0 * n_cls + i];
  if constexpr (HAS_VCLS) {
    constexpr int per_row = kGrpCols * (int)sizeof(TV) / 16;
    for (int64_t i = threadIdx.x; i < n_cls * per_row; i += blockDim.x) {
      const int64_t c = i / per_row, part = i % per_row;
      cp_async16(reinterpret_cast<unsigned char*>(vcls_s + c * kGrpCols) + part * 16,
                 reinterpret_cast<const unsigned char*>(vcls + c * ld_vcls + cb) + part * 16);
    }
  }
  if (staged) {
    constexpr int per_half = kGrpCols * 2 / 16;  // 16-byte pieces of the K (or V) columns
    for (int64_t i = threadIdx.x; i < ns * 2 * per_half; i += blockDim.x) {
      const int64_t r = i / (2 * per_half);
      const int part = (int)(i % (2 * per_half));
      const __nv_bfloat16* g = (part < per_half ? k : v) + (s0 + r) * ldkv + cb;
      cp_async16(reinterpret_cast<unsigned char*>(kv_s) + r * kGrpKvRowBytes + part * 16,
                 reinterpret_cast<const unsigned char*>(g) + (part % per_half) * 16);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 3, sl = lane & 7;
  const int col = sl * 8;
  const int lph = hd / 8;
  const float* brow = bias_s + (col / hd) * n_cls;
  for (int64_t base = q0 + warp * 4; base < q1; base += kGrpWarps * 4) {
    const int64_t row = base + sub;
    const bool rv = row < q1;
    float qv[8] = {};
    int64_t beg = 0;
    int n = 0;
    if (rv) {
      load_vec<8>(q + row * ldq + cb + col, qv);
      beg = seg_ptr[row];
      n = (int)(seg_ptr[row + 1] - beg);
      if (skip_ptr && skip_ptr[row + 1] > skip_ptr[row]) n = 0;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[i] *= scale;
    int nmax = n;
    nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, 8));
    nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, 16));
    float m = kNegInf, l = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    if (staged)
      grouped_rows<LPH, true, HAS_VCLS, TV>(qv, beg, n, nmax, src, cls, s0, ns, n_cls, kv_s + col,
                                           kv_s + kGrpCols + col, kGrpKvRowBytes / 2, brow, vcls_s + col, lph, m, l,
                                           acc);
    else
      grouped_rows<LPH, false, HAS_VCLS, TV>(qv, beg, n, nmax, src, cls, s0, ns, n_cls, k + s0 * ldkv + cb + col,
                                            v + s0 * ldkv + cb + col, ldkv, brow, vcls_s + col, lph, m, l, acc);
    const float inv = l > 0.f ? 1.f / l : 1.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
    if (rv) store_vec<8>(out + row * ldo + cb + col, acc);
  }
}

// --------------------------------------------------------- stone attention
// Whether mb_stone_attention takes the tensor-core kernel for the shapes it
// serves (1, the default) or always the CUDA-core kernel below (0).
static int g_stone_tc = 1;
constexpr int kStoneThreads = 128;
constexpr int kKeyTile = 64;

template <typename T, typename TO, int D>
__global__ void __launch_bounds__(kStoneThreads) stone_attention_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, int64_t s_pos, int64_t s_head,
    int64_t s_row, const int32_t* __restrict__ seq_lens, int64_t t_pad, const int64_t* __restrict__ tok_off,
    int max_queries, TO* __restrict__ out, int64_t o_pos, int64_t o_head, int64_t o_row, float* __restrict__ lse,
    int heads, float scale) {
  __shared__ float ks[kKeyTile][D];
  __shared__ float vs[kKeyTile][D];
  const int64_t p = blockIdx.y;
  const int a = blockIdx.z;
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
  const int64_t row0 = (int64_t)blockIdx.x * kStoneThreads;
  if (row0 >= n_rows) return;
  const int64_t t = row0 + threadIdx.x;
  const bool active = t < n_rows && t < n_keys;
  float qv[D], acc[D];
  float m = kNegInf, l = 0.f;
#pragma unroll
  for (int i = 0; i < D; ++i) acc[i] = 0.f;
  if (active) {
    load_vec<D>(q + base_in + t * s_row, qv);
#pragma unroll
    for (int i = 0; i < D; ++i) qv[i] *= scale;
  }
  for (int64_t j0 = 0; j0 < n_keys; j0 += kKeyTile) {
    const int nk = (int)min((int64_t)kKeyTile, n_keys - j0);
    __syncthreads();
    // cooperative tile load: D/4 float4-equivalents per row
    for (int idx = threadIdx.x; idx < nk * (D / 4); idx += kStoneThreads) {
      const int r = idx / (D / 4), c = (idx % (D / 4)) * 4;
      float tk[4], tv[4];
      load_vec<4>(k + base_in + (j0 + r) * s_row + c, tk);
      load_vec<4>(v + base_in + (j0 + r) * s_row + c, tv);
#pragma unroll
      for (int i = 0; i < 4; ++i) { ks[r][c + i] = tk[i]; vs[r][c + i] = tv[i]; }
    }
    __syncthreads();
    if (active) {
      for (int jj = 0; jj < nk; jj += 8) {
        float sc[8];
        float cm = kNegInf;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float d = kNegInf;
          if (jj + u < nk) {
            d = 0.f;
#pragma unroll
            for (int i = 0; i < D; ++i) d += qv[i] * ks[jj + u][i];
          }
          sc[u] = d;
          cm = fmaxf(cm, d);
        }
        const float m_new = fmaxf(m, cm);
        const float corr = __expf(m - m_new);
        l *= corr;
#pragma unroll
        for (int i = 0; i < D; ++i) acc[i] *= corr;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (jj + u < nk) {
            const float pr = __expf(sc[u] - m_new);
            l += pr;
#pragma unroll
            for (int i = 0; i < D; ++i) acc[i] += pr * vs[jj + u][i];
          }
        }
        m = m_new;
      }
    }
  }
  if (t < n_rows) {
    const float inv = (active && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) acc[i] *= inv;
    store_vec<D>(out + base_out + t * o_row, acc);
    // log-sum-exp of the scaled scores (0 for a padded query row), padded layout (P, heads, t_pad)
    if (lse && !tok_off) lse[(p * heads + a) * t_pad + t] = (active && l > 0.f) ? m + logf(l) : 0.f;
  }
}

// ------------------------------------------------------- window latents
// Read: a position's 4 latent queries attend over its windows. The windows
// of one position are split over a cluster of kReadSplit CTAs (8 warps each,
// every warp a strided share of the split, two windows per step so four K/V
// rows are in flight); each CTA merges its warps' partial softmax states in
// shared memory, then the cluster's first CTA merges the kReadSplit CTA
// states through distributed shared memory and writes the output.
constexpr int kReadWarps = 8;
constexpr int kReadSplit = 4;

template <typename T, typename TO, int VEC>
__global__ void __cluster_dims__(1, kReadSplit, 1) __launch_bounds__(kReadWarps * 32) latent_read_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, const T* __restrict__ v, int64_t ldkv,
    int64_t n_windows, int heads, int hd, const int64_t* __restrict__ offsets, const int64_t* __restrict__ order,
    TO* __restrict__ out, float* __restrict__ m_out, float* __restrict__ l_out, float scale) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ float smem[];
  const int64_t p = blockIdx.x;
  const int rank = (int)cluster.block_rank();
  const int H = heads * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lph = hd / VEC;
  const int chunks = (H + 32 * VEC - 1) / (32 * VEC);  // column chunks per row
  const int64_t b0 = offsets[p], len = offsets[p + 1] - b0;
  const int64_t beg = b0 + len * rank / kReadSplit, end = b0 + len * (rank + 1) / kReadSplit;
  // shared layout: [warp][slot][H] acc, [warp][slot][heads] m and l, then the
  // CTA's merged state: [slot][H] acc, [slot][heads] m and l
  float* s_acc = smem;
  float* s_m = s_acc + kReadWarps * 4 * H;
  float* s_l = s_m + kReadWarps * 4 * heads;
  float* c_acc = s_l + kReadWarps * 4 * heads;
  float* c_m = c_acc + 4 * H;
  float* c_l = c_m + 4 * heads;
  for (int ch = 0; ch < chunks; ++ch) {
    const int col = ch * 32 * VEC + lane * VEC;
    const bool live = col < H;  // H < 32 leaves upper lanes idle
    const int hcur = col / hd;
    float qv[4][VEC] = {}, acc[4][VEC], m[4], l[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (live) load_vec<VEC>(q + (p * 4 + s) * ldq + col, qv[s]);
#pragma unroll
      for (int i = 0; i < VEC; ++i) { qv[s][i] *= scale; acc[s][i] = 0.f; }
      m[s] = kNegInf;
      l[s] = 0.f;
    }
    auto consume = [&](const Raw<T, VEC>& kr, const Raw<T, VEC>& vr) {
      float kv[VEC], vv[VEC];
      raw_unpack<VEC>(kr, kv);
      raw_unpack<VEC>(vr, vv);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        float d = 0.f;
#pragma unroll
        for (int u = 0; u < VEC; ++u) d += qv[s][u] * kv[u];
        d = group_sum(d, lph);
        const float m_new = fmaxf(m[s], d);
        const float corr = __expf(m[s] - m_new), pr = __expf(d - m_new);
        l[s] = l[s] * corr + pr;
#pragma unroll
        for (int u = 0; u < VEC; ++u) acc[s][u] = acc[s][u] * corr + pr * vv[u];
        m[s] = m_new;
      }
    };
    // the next step's order entries are requested a step ahead, so a step
    // waits on its K/V rows only
    int64_t n0 = beg + warp < end ? order[beg + warp] : -1;
    int64_t n1 = beg + warp + kReadWarps < end ? order[beg + warp + kReadWarps] : -1;
    for (int64_t i = beg + warp; i < end; i += 2 * kReadWarps) {
      const int64_t i1 = i + kReadWarps;
      int64_t w0 = n0, w1 = i1 < end ? n1 : -1;
      const int64_t j = i + 2 * kReadWarps;
      if (j < end) n0 = order[j];
      if (j + kReadWarps < end) n1 = order[j + kReadWarps];
      const bool ok0 = w0 >= 0 && w0 < n_windows, ok1 = i1 < end && w1 >= 0 && w1 < n_windows;
      if (!ok0 || (i1 < end && !ok1)) report(ERR_INDEX);
      Raw<T, VEC> k0 = {}, v0 = {}, k1 = {}, v1 = {};
      if (live && ok0) {
        raw_load<false, VEC>(k + w0 * ldkv + col, k0);
        raw_load<false, VEC>(v + w0 * ldkv + col, v0);
      }
      if (live && ok1) {
        raw_load<false, VEC>(k + w1 * ldkv + col, k1);
        raw_load<false, VEC>(v + w1 * ldkv + col, v1);
      }
      if (ok0) consume(k0, v0);
      if (ok1) consume(k1, v1);
    }
    if (!live) continue;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int u = 0; u < VEC; ++u) s_acc[(warp * 4 + s) * H + col + u] = acc[s][u];
      if (lane % lph == 0) {
        s_m[(warp * 4 + s) * heads + hcur] = m[s];
        s_l[(warp * 4 + s) * heads + hcur] = l[s];
      }
    }
  }
  __syncthreads();
  // this CTA's state: merge the warps (acc stays unnormalised)
  for (int idx = threadIdx.x; idx < 4 * H; idx += blockDim.x) {
    const int s = idx / H, col = idx % H, hh = col / hd;
    float mm = kNegInf;
    for (int w = 0; w < kReadWarps; ++w) mm = fmaxf(mm, s_m[(w * 4 + s) * heads + hh]);
    float ll = 0.f, aa = 0.f;
    if (mm != kNegInf) {
      for (int w = 0; w < kReadWarps; ++w) {
        const float mw = s_m[(w * 4 + s) * heads + hh];
        if (mw == kNegInf) continue;
        const float f = __expf(mw - mm);
        ll += f * s_l[(w * 4 + s) * heads + hh];
        aa += f * s_acc[(w * 4 + s) * H + col];
      }
    }
    c_acc[s * H + col] = aa;
    if (col % hd == 0) {
      c_m[s * heads + hh] = mm;
      c_l[s * heads + hh] = ll;
    }
  }
  cluster.sync();
  if (rank == 0) {
    for (int idx = threadIdx.x; idx < 4 * H; idx += blockDim.x) {
      const int s = idx / H, col = idx % H, hh = col / hd;
      float mr[kReadSplit], mm = kNegInf;
#pragma unroll
      for (int r = 0; r < kReadSplit; ++r) {
        mr[r] = cluster.map_shared_rank(c_m, r)[s * heads + hh];
        mm = fmaxf(mm, mr[r]);
      }
      float ll = 0.f, aa = 0.f;
      if (mm != kNegInf) {
#pragma unroll
        for (int r = 0; r < kReadSplit; ++r) {
          if (mr[r] == kNegInf) continue;
          const float f = __expf(mr[r] - mm);
          ll += f * cluster.map_shared_rank(c_l, r)[s * heads + hh];
          aa += f * cluster.map_shared_rank(c_acc, r)[s * H + col];
        }
      }
      out[(p * 4 + s) * H + col] = from_f<TO>(ll > 0.f ? aa / ll : 0.f);
      if (m_out && (col % hd) == 0) {
        m_out[(p * 4 + s) * heads + hh] = mm;
        l_out[(p * 4 + s) * heads + hh] = ll;
      }
    }
  }
  cluster.sync();  // every CTA's shared state stays alive until the first CTA has read it
}

// Broadcast: a warp takes kBcastWindows consecutive windows. Their positions
// come in one load (a lane each) and their query rows are all requested at
// once; a position's four latent K and V rows are fetched when the position
// changes, so the run of windows of one position shares them.
constexpr int kBcastWindows = 4;

template <typename T, typename TO, int VEC>
__global__ void __launch_bounds__(256) latent_broadcast_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, const T* __restrict__ v, int64_t ldkv,
    int64_t n_pos, int64_t n_windows, int heads, int hd, const int64_t* __restrict__ window_pos, TO* __restrict__ out,
    float* __restrict__ m_out, float* __restrict__ l_out, float scale) {
  const int64_t w0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kBcastWindows;
  if (w0 >= n_windows) return;
  const int lane = threadIdx.x & 31;
  const int nw = (int)(n_windows - w0 < kBcastWindows ? n_windows - w0 : kBcastWindows);
  const int H = heads * hd;
  const int lph = hd / VEC;
  const int64_t my_pos = lane < nw ? window_pos[w0 + lane] : 0;
  for (int c0 = 0; c0 < H; c0 += 32 * VEC) {
    const int col = c0 + lane * VEC;
    const bool live = col < H;  // H < 32 leaves upper lanes idle
    Raw<T, VEC> qr[kBcastWindows] = {}, kr[4] = {}, vr[4] = {};
    if (live) {
#pragma unroll
      for (int u = 0; u < kBcastWindows; ++u)
        if (u < nw) raw_load<false, VEC>(q + (w0 + u) * ldq + col, qr[u]);
    }
    int64_t have = -1;  // the position whose latent rows kr / vr hold
#pragma unroll
    for (int u = 0; u < kBcastWindows; ++u) {
      if (u >= nw) break;
      const int64_t w = w0 + u;
      const int64_t p = __shfl_sync(0xffffffffu, my_pos, u);
      if (p < 0 || p >= n_pos) {
        report(ERR_INDEX);
        continue;
      }
      if (p != have) {
        have = p;
        if (live) {
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            raw_load<false, VEC>(k + (p * 4 + s) * ldkv + col, kr[s]);
            raw_load<false, VEC>(v + (p * 4 + s) * ldkv + col, vr[s]);
          }
        }
      }
      float qv[VEC], sc[4], mx = kNegInf;
      raw_unpack<VEC>(qr[u], qv);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        float kv[VEC];
        raw_unpack<VEC>(kr[s], kv);
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < VEC; ++i) d += qv[i] * kv[i];
        sc[s] = group_sum(d, lph) * scale;
        mx = fmaxf(mx, sc[s]);
      }
      float l = 0.f, acc[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const float pr = __expf(sc[s] - mx);
        l += pr;
        float vv[VEC];
        raw_unpack<VEC>(vr[s], vv);
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] += pr * vv[i];
      }
      const float inv = 1.f / l;
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] *= inv;
      if (!live) continue;
      store_vec<VEC>(out + w * H + col, acc);
      if (m_out && lane % lph == 0) {
        m_out[w * heads + col / hd] = mx;
        l_out[w * heads + col / hd] = l;
      }
    }
  }
}

// Dense 4x4 mix: block per position; scores per (query slot, head, key slot)
// by one thread each, then one thread per output element.
template <typename T, typename TO>
__global__ void latent_mix_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                  int64_t ld, int heads, int hd, TO* __restrict__ out, float scale) {
  extern __shared__ float wts[];  // [4][heads][4]
  const int64_t p = blockIdx.x;
  const int H = heads * hd;
  const T* qp = q + p * 4 * ld;
  const T* kp = k + p * 4 * ld;
  const T* vp = v + p * 4 * ld;
  for (int idx = threadIdx.x; idx < 4 * heads * 4; idx += blockDim.x) {
    const int qs = idx / (heads * 4), hh = (idx / 4) % heads, ks = idx % 4;
    float d = 0.f;
    for (int i = 0; i < hd; ++i) d += to_f(qp[qs * ld + hh * hd + i]) * to_f(kp[ks * ld + hh * hd + i]);
    wts[idx] = d * scale;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 4 * heads; idx += blockDim.x) {
    float* r = wts + idx * 4;
    const float mx = fmaxf(fmaxf(r[0], r[1]), fmaxf(r[2], r[3]));
    float e[4], sum = 0.f;
    for (int s = 0; s < 4; ++s) { e[s] = __expf(r[s] - mx); sum += e[s]; }
    for (int s = 0; s < 4; ++s) r[s] = e[s] / sum;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 4 * H; idx += blockDim.x) {
    const int qs = idx / H, col = idx % H, hh = col / hd;
    const float* r = wts + (qs * heads + hh) * 4;
    float o = 0.f;
    for (int s = 0; s < 4; ++s) o += r[s] * to_f(vp[s * ld + col]);
    out[p * 4 * H + idx] = from_f<TO>(o);
  }
}

// Lane tiling for warp-per-row attention: VEC columns per lane, head_dim / VEC
// lanes per head (a power of two). Widths below 32 run with idle upper lanes.
static int attn_vec(int heads, int head_dim) {
  const int H = heads * head_dim;
  if (heads <= 0 || head_dim <= 0) return 0;
  int vec = pick_vec(H);
  if (vec == 0) {
    if (H > 32) return 0;
    vec = 1;
  }
  if (head_dim % vec != 0) return 0;
  const int lph = head_dim / vec;
  if (lph > 32 || (lph & (lph - 1))) return 0;
  return vec;
}

}  // namespace mb

using namespace mb;

extern "C" {

int mb_segment_attention(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                         int64_t n_q, int64_t n_src, int heads, int head_dim, const float* bias, int64_t n_cls,
                         const void* vcls, int vcls_dtype, const int64_t* seg_ptr, const int64_t* src,
                         const int64_t* cls, const int64_t* skip_ptr, void* out, int out_dtype, int64_t ldo, float* m,
                         float* l, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "segment_attention: bad dtype");
  MB_REQUIRE(heads > 0 && head_dim > 0 && n_q >= 0 && n_src >= 0 && n_src <= INT32_MAX,
             "segment_attention: bad sizes");
  if (n_q == 0) return MB_OK;
  const int H = heads * head_dim;
  const int vec = attn_vec(heads, head_dim);
  MB_REQUIRE(vec > 0 && H <= 32 * vec, "segment_attention: unsupported heads=%d head_dim=%d", heads, head_dim);
  MB_REQUIRE(q && out && seg_ptr && bias, "segment_attention: null pointer");
  MB_REQUIRE((m == nullptr) == (l == nullptr), "segment_attention: m and l go together");
  MB_REQUIRE(valid_dtype(vcls_dtype), "segment_attention: bad vcls dtype");
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  dim3 grid((unsigned)cdiv(n_q, kSegWarps * kSegRows));
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_T(vcls_dtype, TV, [&] {
        MB_DISPATCH_VEC(vec, V, [&] {
          if (vcls)
            segment_attention_kernel<T, TO, TV, V, true><<<grid, kSegWarps * 32, 0, s>>>(
                (const T*)q, ldq, (const T*)k, (const T*)v, ldkv, n_q, n_src, heads, head_dim, bias, n_cls,
                (const TV*)vcls, seg_ptr, src, cls, skip_ptr, (TO*)out, ldo, m, l, scale);
          else
            segment_attention_kernel<T, TO, TV, V, false><<<grid, kSegWarps * 32, 0, s>>>(
                (const T*)q, ldq, (const T*)k, (const T*)v, ldkv, n_q, n_src, heads, head_dim, bias, n_cls,
                (const TV*)vcls, seg_ptr, src, cls, skip_ptr, (TO*)out, ldo, m, l, scale);
        });
      });
    });
  });
  return launch_status("segment_attention");
}

int mb_segment_attention_grouped(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                                 int64_t n_q, int64_t n_src, int heads, int head_dim, const float* bias,
                                 int64_t n_cls, const void* vcls, int vcls_dtype, const int64_t* seg_ptr,
                                 const int64_t* src, const int64_t* cls, const int64_t* skip_ptr,
                                 const int64_t* q_off, const int64_t* s_off, int64_t n_groups, int64_t stage_rows,
                                 void* out, int out_dtype, int64_t ldo, void* stream) {
  MB_REQUIRE(dtype == MB_BF16, "segment_attention_grouped: q/k/v must be bf16");
  MB_REQUIRE(valid_dtype(out_dtype) && valid_dtype(vcls_dtype), "segment_attention_grouped: bad dtype");
  MB_REQUIRE(heads > 0 && head_dim > 0 && n_q >= 0 && n_groups >= 0 && n_src >= 0 && n_src <= INT32_MAX,
             "segment_attention_grouped: bad sizes");
  const int64_t H = (int64_t)heads * head_dim;
  MB_REQUIRE(H % kGrpCols == 0 && kGrpCols % head_dim == 0 && head_dim % 8 == 0,
             "segment_attention_grouped: unsupported heads=%d head_dim=%d (needs head_dim in {8,16,32,64} and "
             "width a multiple of %d)", heads, head_dim, kGrpCols);
  MB_REQUIRE(n_cls > 0 && n_cls <= (1 << kGrpClsBits), "segment_attention_grouped: n_cls out of range");
  MB_REQUIRE(stage_rows >= 1, "segment_attention_grouped: stage_rows must be >= 1");
  MB_REQUIRE(q && k && v && out && bias && seg_ptr && src && cls && q_off && s_off,
             "segment_attention_grouped: null pointer");
  MB_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && ldq % 8 == 0 && ldkv % 8 == 0 &&
                 ldo % 8 == 0 && aligned(out, 16) && (!vcls || aligned(vcls, 16)),
             "segment_attention_grouped: q/k/v/out need 16-byte aligned rows");
  if (n_q == 0 || n_groups == 0) return MB_OK;
  const int nh = kGrpCols / head_dim;
  const int fixed = grp_bias_bytes(nh, n_cls) +
                    (vcls ? (vcls_dtype == MB_BF16 ? grp_vcls_bytes<__nv_bfloat16>(n_cls) : grp_vcls_bytes<float>(n_cls))
                          : 0);
  const int limit = 227 * 1024;
  MB_REQUIRE(fixed + kGrpKvRowBytes <= limit, "segment_attention_grouped: %lld classes do not fit shared memory",
             (long long)n_cls);
  // Groups with more sources than fit read K/V from global memory instead.
  const int64_t rows = std::min<int64_t>(stage_rows, (limit - fixed) / kGrpKvRowBytes);
  const int smem = fixed + (int)rows * kGrpKvRowBytes;
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  dim3 grid((unsigned)n_groups, (unsigned)(H / kGrpCols));
  int rc = MB_OK;
  MB_DISPATCH_T(out_dtype, TO, [&] {
    MB_DISPATCH_T(vcls_dtype, TV, [&] {
      auto kern = head_dim == 32
                      ? (vcls ? segment_attention_grouped_kernel<TO, TV, 4, true>
                              : segment_attention_grouped_kernel<TO, TV, 4, false>)
                      : (vcls ? segment_attention_grouped_kernel<TO, TV, 0, true>
                              : segment_attention_grouped_kernel<TO, TV, 0, false>);
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        rc = fail(MB_LAUNCH_FAILED, "segment_attention_grouped: %d bytes of shared memory refused", smem);
        return;
      }
      kern<<<grid, kGrpWarps * 32, smem, s>>>((const __nv_bfloat16*)q, ldq, (const __nv_bfloat16*)k,
                                             (const __nv_bfloat16*)v, ldkv, n_q, n_src, head_dim, bias, n_cls,
                                             (const TV*)vcls, H, seg_ptr, src, cls, skip_ptr, q_off, s_off,
                                             (int)rows, (TO*)out, ldo, scale);
    });
  });
  if (rc != MB_OK) return rc;
  return launch_status("segment_attention_grouped");
}

}  // extern "C"

// Defined with the tcgen05 kernels (stone_sm100.cu): the tensor-core path of
// mb_stone_attention, -1 when it does not take the shape.
static int stone_attention_tc(const void* q, const void* k, const void* v, int dtype, int64_t n_pos, int heads,
                              int head_dim, int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* seq_lens,
                              int64_t t_pad, const int64_t* tok_off, int64_t max_tokens, int max_queries, void* out,
                              int out_dtype, int64_t o_pos, int64_t o_head, int64_t o_row, float* lse,
                              cudaStream_t s);

extern "C" {

int mb_stone_attention(const void* q, const void* k, const void* v, int dtype, int64_t n_pos, int heads, int head_dim,
                       int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* seq_lens, int64_t t_pad,
                       const int64_t* tok_off, int64_t max_tokens, int max_queries, void* out, int out_dtype,
                       int64_t o_pos, int64_t o_head, int64_t o_row, float* lse, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "stone_attention: bad dtype");
  MB_REQUIRE(!lse || !tok_off, "stone_attention: the log-sum-exp output takes the padded layout");
  MB_REQUIRE(head_dim == 16 || head_dim == 32 || head_dim == 64, "stone_attention: head_dim %d unsupported", head_dim);
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(q && k && v && out, "stone_attention: null pointer");
  MB_REQUIRE(tok_off || seq_lens, "stone_attention: need seq_lens (padded) or tok_off (ragged)");
  MB_REQUIRE(n_pos <= 65535 && heads <= 65535, "stone_attention: grid too large");
  const int64_t rows = tok_off ? (max_queries >= 0 ? max_queries : max_tokens) : t_pad;
  if (rows <= 0) return MB_OK;
  // bf16, head_dim 32, at most 320 keys: QK^T and PV on the tensor cores
  if (g_stone_tc) {
    const int rc = stone_attention_tc(q, k, v, dtype, n_pos, heads, head_dim, s_pos, s_head, s_row, seq_lens, t_pad,
                                      tok_off, max_tokens, max_queries, out, out_dtype, o_pos, o_head, o_row, lse,
                                      as_stream(stream));
    if (rc >= 0) return rc;
  }
  dim3 grid((unsigned)cdiv(rows, kStoneThreads), (unsigned)n_pos, (unsigned)heads);
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      auto go = [&](auto dtag) {
        constexpr int D = decltype(dtag)::value;
        stone_attention_kernel<T, TO, D><<<grid, kStoneThreads, 0, s>>>(
            (const T*)q, (const T*)k, (const T*)v, s_pos, s_head, s_row, seq_lens, t_pad, tok_off, max_queries,
            (TO*)out, o_pos, o_head, o_row, lse, heads, scale);
      };
      if (head_dim == 16) go(std::integral_constant<int, 16>{});
      else if (head_dim == 32) go(std::integral_constant<int, 32>{});
      else go(std::integral_constant<int, 64>{});
    });
  });
  return launch_status("stone_attention");
}

static int latent_vec(int heads, int head_dim) { return attn_vec(heads, head_dim); }

int mb_stone_attention_engine(int tensor_cores) {
  MB_REQUIRE(tensor_cores == 0 || tensor_cores == 1, "stone_attention_engine: 0 or 1");
  g_stone_tc = tensor_cores;
  return MB_OK;
}

int mb_window_latent_read(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                          int64_t n_pos, int64_t n_windows, int heads, int head_dim, const int64_t* offsets,
                          const int64_t* order, void* out, int out_dtype, float* m, float* l, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "window_latent_read: bad dtype");
  if (n_pos == 0) return MB_OK;
  const int vec = latent_vec(heads, head_dim);
  MB_REQUIRE(vec > 0, "window_latent_read: unsupported heads=%d head_dim=%d", heads, head_dim);
  MB_REQUIRE(q && out && offsets && (n_windows == 0 || (k && v && order)), "window_latent_read: null pointer");
  const int H = heads * head_dim;
  const size_t smem = sizeof(float) * ((size_t)kReadWarps * 4 * (H + 2 * heads) + 4 * (H + 2 * heads));
  MB_REQUIRE(smem <= 200 * 1024, "window_latent_read: width too large");
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        auto kern = latent_read_kernel<T, TO, V>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<dim3((unsigned)n_pos, kReadSplit), kReadWarps * 32, smem, s>>>(
            (const T*)q, ldq, (const T*)k, (const T*)v, ldkv, n_windows, heads, head_dim, offsets, order, (TO*)out,
            m, l, scale);
      });
    });
  });
  return launch_status("window_latent_read");
}

int mb_window_latent_broadcast(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                               int64_t n_pos, int64_t n_windows, int heads, int head_dim, const int64_t* window_pos,
                               void* out, int out_dtype, float* m, float* l, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "window_latent_broadcast: bad dtype");
  if (n_windows == 0) return MB_OK;
  const int vec = latent_vec(heads, head_dim);
  MB_REQUIRE(vec > 0, "window_latent_broadcast: unsupported heads=%d head_dim=%d", heads, head_dim);
  MB_REQUIRE(q && k && v && out && window_pos, "window_latent_broadcast: null pointer");
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        latent_broadcast_kernel<T, TO, V><<<(unsigned)cdiv(n_windows, 8 * kBcastWindows), 256, 0, s>>>(
            (const T*)q, ldq, (const T*)k, (const T*)v, ldkv, n_pos, n_windows, heads, head_dim, window_pos,
            (TO*)out, m, l, scale);
      });
    });
  });
  return launch_status("window_latent_broadcast");
}

int mb_latent_mix(const void* q, const void* k, const void* v, int64_t ld, int dtype, int64_t n_pos, int heads,
                  int head_dim, void* out, int out_dtype, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "latent_mix: bad dtype");
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(q && k && v && out && heads > 0 && head_dim > 0, "latent_mix: bad arguments");
  const float scale = 1.f / sqrtf((float)head_dim);
  const size_t smem = sizeof(float) * 16 * heads;
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      latent_mix_kernel<T, TO><<<(unsigned)n_pos, 256, smem, s>>>((const T*)q, (const T*)k, (const T*)v, ld, heads,
                                                                  head_dim, (TO*)out, scale);
    });
  });
  return launch_status("latent_mix");
}

}  // extern "C"
