// Radius read (cells <- stones within hex distance 8): the typed segment
// attention of the production trunk's cell stage over block-diagonal edges
// (reference cell_latents.py:213-285 kernel, called from model.py:439-451 with
// the radius tables of model.py:864-875 / cell_nodes.py:23-123).
//
// The radius tables are the same for every trunk block, so two things are
// derived once per forward and reused by all blocks:
//   packed edges  int32 (local stone << 11) | class per edge, the local stone
//                 counted from the position's first stone; range-checked once
//                 here instead of per edge per block;
//   row order     the position's cells by ascending edge count, so the four
//                 rows a warp carries have about the same number of edges
//                 (a warp steps to the largest of its four counts).
//
// Kernel: one CTA per (position, 64-column block = whole heads). It stages the
// position's stone K|V columns, the class value rows and the class bias in
// shared memory, then each warp carries four cells at a time, eight lanes per
// cell, eight bf16 columns per lane. Per edge: the row's packed index comes by
// shuffle from the lane that loaded it (eight indices per load), the K row and
// the class row are conflict-free 16-byte shared-memory reads, and the online
// softmax update runs on packed f32x2 arithmetic (fma.rn.f32x2).
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace mb {
namespace radius {

constexpr int kCols = 64;                 // columns per CTA
constexpr int kWarps = 16;
constexpr int kClsBits = 11;              // packed edge: local stone << 11 | class
constexpr int kKvRowBytes = 2 * kCols * 2;  // K then V, bf16

// ------------------------------------------------------------ f32x2 math
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// a bf16x2 word -> (low, high) as an f32x2
__device__ __forceinline__ uint64_t bf2(uint32_t w) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(w << 16), "r"(w & 0xffff0000u));
  return r;
}

// ------------------------------------------------------------ edge packing
__global__ void pack_edges_kernel(const int64_t* __restrict__ src, const int64_t* __restrict__ cls,
                                  const int64_t* __restrict__ seg_ptr, const int64_t* __restrict__ q_off,
                                  const int64_t* __restrict__ s_off, int64_t n_q, int64_t n_edges, int64_t n_src,
                                  int64_t n_cls, int32_t* __restrict__ packed) {
  const int64_t g = blockIdx.x;
  const int64_t q0 = q_off[g], q1 = q_off[g + 1], s0 = s_off[g], s1 = s_off[g + 1];
  if (q0 < 0 || q1 < q0 || q1 > n_q || s0 < 0 || s1 < s0 || s1 > n_src || s1 - s0 >= (int64_t(1) << 20)) {
    if (threadIdx.x == 0) report(ERR_RUN_BOUND);
    return;
  }
  const int64_t e0 = seg_ptr[q0], e1 = seg_ptr[q1];
  if (e0 < 0 || e1 < e0 || e1 > n_edges) {
    if (threadIdx.x == 0) report(ERR_RUN_BOUND);
    return;
  }
  for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
    const int64_t s = src[e] - s0, c = cls[e];
    if ((uint64_t)s < (uint64_t)(s1 - s0) && (uint64_t)c < (uint64_t)n_cls) {
      packed[e] = (int32_t)((s << kClsBits) | c);
    } else {
      report(ERR_INDEX);
      packed[e] = -1;
    }
  }
}

// ------------------------------------------------------------ attention
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}
__device__ __forceinline__ float lds32f(uint32_t addr) {
  float r;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(addr));
  return r;
}

// One softmax step of a row's edge: score, running max / sum, and the
// accumulator update with the edge's value row (+ class value row).
template <bool HAS_VCLS>
__device__ __forceinline__ void edge_step(float d, float b, const uint4& vr, const uint4& cr, float& m, float& l,
                                          uint64_t (&acc)[4]) {
  const float score = d + b;
  const float m_new = fmaxf(m, score);
  const float corr = __expf(m - m_new);  // m = -inf on the first live edge: exp(-inf) = 0
  const float p = __expf(score - m_new);
  l = l * corr + p;
  uint64_t v2[4] = {bf2(vr.x), bf2(vr.y), bf2(vr.z), bf2(vr.w)};
  if constexpr (HAS_VCLS) {
    v2[0] = add2(v2[0], bf2(cr.x));
    v2[1] = add2(v2[1], bf2(cr.y));
    v2[2] = add2(v2[2], bf2(cr.z));
    v2[3] = add2(v2[3], bf2(cr.w));
  }
  const uint64_t c2 = pack2(corr, corr), p2 = pack2(p, p);
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = fma2(p2, v2[i], mul2(acc[i], c2));
  m = m_new;
}

__device__ __forceinline__ float dot8(const uint64_t (&q2)[4], const uint4& kr) {
  uint64_t d2 = mul2(q2[0], bf2(kr.x));
  d2 = fma2(q2[1], bf2(kr.y), d2);
  d2 = fma2(q2[2], bf2(kr.z), d2);
  d2 = fma2(q2[3], bf2(kr.w), d2);
  float da, db;
  unpack2(d2, da, db);
  float d = da + db;
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  return d + __shfl_xor_sync(0xffffffffu, d, 2);  // head of 32 columns = 4 lanes
}

// A row's edges with the position's K|V staged in shared memory: every
// shared-memory read is a 32-bit-addressed ld.shared. kv: the lane's K
// columns of stone 0 (V columns 128 bytes further, one stone per 256 bytes);
// bias: the lane's head's bias row; vc: the lane's columns of class 0.
template <bool HAS_VCLS>
__device__ __forceinline__ void row_edges_staged(const uint64_t (&q2)[4], int64_t beg, int n, int nmax,
                                                 const int32_t* __restrict__ packed, uint32_t kv, uint32_t bias,
                                                 uint32_t vc, float& m, float& l, uint64_t (&acc)[4]) {
  const int lane = threadIdx.x & 31;
  const int g0 = lane & ~7, li = lane & 7;
  const int32_t* pe = packed + beg + li;
  int mine = -1;
  for (int j = 0; j < nmax; ++j) {
    if ((j & 7) == 0) mine = (j + li < n) ? __ldg(pe + j) : -1;
    const int pk = __shfl_sync(0xffffffffu, mine, g0 + (j & 7));
    const bool live = pk >= 0;
    const uint32_t s = (uint32_t)pk >> kClsBits, c = (uint32_t)pk & ((1u << kClsBits) - 1);
    const uint32_t ka = kv + s * kKvRowBytes;
    const uint4 kr = live ? lds128(ka) : make_uint4(0, 0, 0, 0);
    const float d = dot8(q2, kr);
    if (!live) continue;
    const float b = lds32f(bias + c * 4);
    const uint4 vr = lds128(ka + kCols * 2);
    uint4 cr = make_uint4(0, 0, 0, 0);
    if constexpr (HAS_VCLS) cr = lds128(vc + c * (kCols * 2));
    edge_step<HAS_VCLS>(d, b, vr, cr, m, l, acc);
  }
}

// The same from global memory (a position with more stones than fit).
template <bool HAS_VCLS>
__device__ __forceinline__ void row_edges_global(const uint64_t (&q2)[4], int64_t beg, int n, int nmax,
                                                 const int32_t* __restrict__ packed, const __nv_bfloat16* kb,
                                                 const __nv_bfloat16* vb, int64_t ld, uint32_t bias, uint32_t vc,
                                                 float& m, float& l, uint64_t (&acc)[4]) {
  const int lane = threadIdx.x & 31;
  const int g0 = lane & ~7, li = lane & 7;
  int mine = -1;
  for (int j = 0; j < nmax; ++j) {
    if ((j & 7) == 0) mine = (j + li < n) ? __ldg(packed + beg + j + li) : -1;
    const int pk = __shfl_sync(0xffffffffu, mine, g0 + (j & 7));
    const bool live = pk >= 0;
    const int s = pk >> kClsBits;
    const uint32_t c = (uint32_t)pk & ((1u << kClsBits) - 1);
    const uint4 kr = live ? __ldg(reinterpret_cast<const uint4*>(kb + (int64_t)s * ld)) : make_uint4(0, 0, 0, 0);
    const float d = dot8(q2, kr);
    if (!live) continue;
    const float b = lds32f(bias + c * 4);
    const uint4 vr = __ldg(reinterpret_cast<const uint4*>(vb + (int64_t)s * ld));
    uint4 cr = make_uint4(0, 0, 0, 0);
    if constexpr (HAS_VCLS) cr = lds128(vc + c * (kCols * 2));
    edge_step<HAS_VCLS>(d, b, vr, cr, m, l, acc);
  }
}

template <typename TO, bool HAS_VCLS>
__global__ void __launch_bounds__(kWarps * 32, 2) radius_read_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, int64_t ldkv, int64_t n_q, int64_t n_src, const float* __restrict__ bias,
    int64_t n_cls, const __nv_bfloat16* __restrict__ vcls, int64_t ld_vcls, const int64_t* __restrict__ seg_ptr,
    const int32_t* __restrict__ packed, const int64_t* __restrict__ skip_ptr, const int64_t* __restrict__ q_off,
    const int64_t* __restrict__ s_off, const int64_t* __restrict__ order, int stage_rows, TO* __restrict__ out,
    int64_t ldo, float scale) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int grp = blockIdx.x;
  const int cb = blockIdx.y * kCols;
  constexpr int nh = kCols / 32;  // heads per column block (head_dim 32)
  const int64_t q0 = q_off[grp], q1 = q_off[grp + 1], s0 = s_off[grp], s1 = s_off[grp + 1];
  if (q0 < 0 || q1 < q0 || q1 > n_q || s0 < 0 || s1 < s0 || s1 > n_src) {
    if (threadIdx.x == 0) report(ERR_RUN_BOUND);
    return;
  }
  if (q1 == q0) return;
  const int64_t ns = s1 - s0;
  const bool staged = ns <= stage_rows;

  const int bias_bytes = (int)((nh * n_cls * 4 + 15) / 16 * 16);
  const int vcls_bytes = HAS_VCLS ? (int)((n_cls * kCols * 2 + 15) / 16 * 16) : 0;
  float* bias_s = reinterpret_cast<float*>(smem);
  __nv_bfloat16* vcls_s = reinterpret_cast<__nv_bfloat16*>(smem + bias_bytes);
  __nv_bfloat16* kv_s = reinterpret_cast<__nv_bfloat16*>(smem + bias_bytes + vcls_bytes);
  const int head0 = cb / 32;
  for (int64_t i = threadIdx.x; i < nh * n_cls; i += blockDim.x) bias_s[i] = bias[head0 * n_cls + i];
  auto cp16 = [](void* dst, const void* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
  };
  if constexpr (HAS_VCLS) {
    constexpr int per_row = kCols * 2 / 16;
    for (int64_t i = threadIdx.x; i < n_cls * per_row; i += blockDim.x) {
      const int64_t c = i / per_row, part = i % per_row;
      cp16(reinterpret_cast<unsigned char*>(vcls_s + c * kCols) + part * 16,
           reinterpret_cast<const unsigned char*>(vcls + c * ld_vcls + cb) + part * 16);
    }
  }
  if (staged) {
    constexpr int per_half = kCols * 2 / 16;  // 16-byte pieces of the K (or V) columns
    for (int64_t i = threadIdx.x; i < ns * 2 * per_half; i += blockDim.x) {
      const int64_t r = i / (2 * per_half);
      const int part = (int)(i % (2 * per_half));
      const __nv_bfloat16* g = (part < per_half ? k : v) + (s0 + r) * ldkv + cb;
      cp16(reinterpret_cast<unsigned char*>(kv_s) + r * kKvRowBytes + part * 16,
           reinterpret_cast<const unsigned char*>(g) + (part % per_half) * 16);
    }
  }
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 3, li = lane & 7;
  const int col = li * 8;
  const float* brow = bias_s + (col / 32) * n_cls;
  for (int64_t base = q0 + warp * 4; base < q1; base += kWarps * 4) {
    const int64_t slot = base + sub;
    const bool rv = slot < q1;
    const int64_t row = rv ? (order ? order[slot] : slot) : 0;
    uint64_t q2[4] = {0, 0, 0, 0};
    int64_t beg = 0;
    int n = 0;
    if (rv) {
      if (row < q0 || row >= q1) {  // the order must permute the position's own rows
        report(ERR_INDEX);
      } else {
        const uint4 qr = __ldg(reinterpret_cast<const uint4*>(q + row * ldq + cb + col));
        const uint64_t s2 = pack2(scale, scale);
        q2[0] = mul2(bf2(qr.x), s2);
        q2[1] = mul2(bf2(qr.y), s2);
        q2[2] = mul2(bf2(qr.z), s2);
        q2[3] = mul2(bf2(qr.w), s2);
        beg = seg_ptr[row];
        n = (int)(seg_ptr[row + 1] - beg);
        if (skip_ptr && skip_ptr[row + 1] > skip_ptr[row]) n = 0;
      }
    }
    int nmax = n;
    nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, 8));
    nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, 16));
    float m = -INFINITY, l = 0.f;
    uint64_t acc[4] = {0, 0, 0, 0};
    const uint32_t bias_a = (uint32_t)__cvta_generic_to_shared(brow);
    const uint32_t vc_a = (uint32_t)__cvta_generic_to_shared(vcls_s + col);
    if (staged)
      row_edges_staged<HAS_VCLS>(q2, beg, n, nmax, packed, (uint32_t)__cvta_generic_to_shared(kv_s + col), bias_a,
                                 vc_a, m, l, acc);
    else
      row_edges_global<HAS_VCLS>(q2, beg, n, nmax, packed, k + s0 * ldkv + cb + col, v + s0 * ldkv + cb + col, ldkv,
                                 bias_a, vc_a, m, l, acc);
    if (rv && row >= q0 && row < q1) {
      const float inv = l > 0.f ? 1.f / l : 0.f;  // an empty run reads zero
      float o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        unpack2(acc[i], o[2 * i], o[2 * i + 1]);
        o[2 * i] *= inv;
        o[2 * i + 1] *= inv;
      }
      store_vec<8>(out + row * ldo + cb + col, o);
    }
  }
}

}  // namespace radius
}  // namespace mb

using namespace mb;

extern "C" {

int mb_radius_pack_edges(const int64_t* src, const int64_t* cls, const int64_t* seg_ptr, const int64_t* q_off,
                         const int64_t* s_off, int64_t n_groups, int64_t n_q, int64_t n_edges, int64_t n_src,
                         int64_t n_cls, int32_t* packed, void* stream) {
  MB_REQUIRE(n_groups >= 0 && n_q >= 0 && n_edges >= 0 && n_src >= 0, "radius_pack_edges: negative size");
  MB_REQUIRE(n_cls > 0 && n_cls <= (1 << radius::kClsBits), "radius_pack_edges: n_cls out of range");
  if (n_groups == 0 || n_edges == 0) return MB_OK;
  MB_REQUIRE(src && cls && seg_ptr && q_off && s_off && packed, "radius_pack_edges: null pointer");
  MB_REQUIRE(n_groups <= INT32_MAX, "radius_pack_edges: too many groups");
  radius::pack_edges_kernel<<<(unsigned)n_groups, 256, 0, as_stream(stream)>>>(src, cls, seg_ptr, q_off, s_off, n_q,
                                                                               n_edges, n_src, n_cls, packed);
  return launch_status("radius_pack_edges");
}

int mb_radius_read(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int64_t n_q, int64_t n_src,
                   int heads, int head_dim, const float* bias, int64_t n_cls, const void* vcls,
                   const int64_t* seg_ptr, const int32_t* packed, const int64_t* skip_ptr, const int64_t* q_off,
                   const int64_t* s_off, const int64_t* order, int64_t n_groups, int64_t stage_rows, void* out,
                   int out_dtype, int64_t ldo, void* stream) {
  MB_REQUIRE(valid_dtype(out_dtype), "radius_read: bad dtype");
  MB_REQUIRE(head_dim == 32 && heads > 0 && (heads * 32) % radius::kCols == 0,
             "radius_read: head_dim must be 32 and the width a multiple of %d (got heads=%d head_dim=%d)", radius::kCols,
             heads, head_dim);
  MB_REQUIRE(n_q >= 0 && n_groups >= 0 && n_src >= 0 && n_src <= INT32_MAX, "radius_read: bad sizes");
  MB_REQUIRE(n_cls > 0 && n_cls <= (1 << radius::kClsBits), "radius_read: n_cls out of range");
  MB_REQUIRE(stage_rows >= 1, "radius_read: stage_rows must be >= 1");
  if (n_q == 0 || n_groups == 0) return MB_OK;
  MB_REQUIRE(q && k && v && out && bias && seg_ptr && packed && q_off && s_off, "radius_read: null pointer");
  MB_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && ldq % 8 == 0 && ldkv % 8 == 0 && ldo % 8 == 0 &&
                 aligned(out, 16) && (!vcls || aligned(vcls, 16)),
             "radius_read: q/k/v/out need 16-byte aligned rows");
  MB_REQUIRE(n_groups <= INT32_MAX, "radius_read: too many groups");
  const int64_t H = (int64_t)heads * head_dim;
  const int fixed = (int)((radius::kCols / 32 * n_cls * 4 + 15) / 16 * 16) + (vcls ? (int)((n_cls * radius::kCols * 2 + 15) / 16 * 16) : 0);
  const int limit = 227 * 1024 / 2;  // two CTAs per SM
  MB_REQUIRE(fixed + radius::kKvRowBytes <= limit, "radius_read: %lld classes do not fit shared memory", (long long)n_cls);
  // groups with more stones than fit read K/V from global memory instead
  const int64_t rows = std::min<int64_t>(stage_rows, (limit - fixed) / radius::kKvRowBytes);
  const int smem = fixed + (int)rows * radius::kKvRowBytes;
  const float scale = 1.f / sqrtf((float)head_dim);
  dim3 grid((unsigned)n_groups, (unsigned)(H / radius::kCols));
  int rc = MB_OK;
  MB_DISPATCH_T(out_dtype, TO, [&] {
    auto kern = vcls ? radius::radius_read_kernel<TO, true> : radius::radius_read_kernel<TO, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      rc = fail(MB_LAUNCH_FAILED, "radius_read: %d bytes of shared memory refused", smem);
      return;
    }
    kern<<<grid, radius::kWarps * 32, smem, as_stream(stream)>>>(
        (const __nv_bfloat16*)q, ldq, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, ldkv, n_q, n_src, bias, n_cls,
        (const __nv_bfloat16*)vcls, H, seg_ptr, packed, skip_ptr, q_off, s_off, order, (int)rows, (TO*)out, ldo,
        scale);
  });
  if (rc != MB_OK) return rc;
  return launch_status("radius_read");
}

}  // extern "C"
