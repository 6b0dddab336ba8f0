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
// Kernel: one CTA per (position, 64-column block = two heads). It stages the
// position's stone K|V columns, the class value rows and the class bias in
// shared memory; then one thread carries one (cell, head) pair through the
// cell's edges, a warp sixteen cells in the position's edge-count order (the
// two lanes of a cell step together, and the sixteen cells have about the
// same number of edges). A thread holds its query row (32 columns, scaled)
// and its 32 accumulator columns as packed f32x2 registers. Per edge: the
// packed index (one 4-byte load), the K row's 64 bytes (four 16-byte
// shared-memory reads), the dot product on fma.rn.f32x2, the class bias;
// the running maximum is raised (and the accumulator rescaled) only when the
// score exceeds it; then the V row and the class value row (eight more
// 16-byte reads) go into the accumulator. Staged rows keep their 16-byte
// units XOR-swizzled by the row index, so the eight lanes of a read phase,
// which hold eight different stones, spread over the banks.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace mb {
namespace radius {

constexpr int kCols = 64;                   // columns per CTA
constexpr int kHeads = kCols / 32;          // heads per CTA (head_dim 32)
constexpr int kThreads = 256;               // 8 warps
constexpr int kCellsPerWarp = 32 / kHeads;  // a warp: 16 cells x 2 heads
constexpr int kClsBits = 11;                // packed edge: local stone << 11 | class
constexpr int kKvRowBytes = 2 * kCols * 2;  // K then V, bf16
constexpr int kClsRowBytes = kCols * 2;     // one class value row, bf16

// Shared-memory reads are conflict-free by lane rotation instead of a
// swizzle: the two lanes of a cell hold its two heads (lane = 2 x cell +
// head), and at its i-th 16-byte read a lane takes unit (i + rot) mod 4 of its
// head's four, rot = cell mod 4. The eight lanes of a read phase (four cells
// x two heads) so address eight different 16-byte bank groups whatever rows
// they read. A lane keeps its query and accumulator columns in that rotated
// unit order.
__device__ __forceinline__ uint32_t unit_off(uint32_t u) { return u << 4; }

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

// The slot table and the slot-ordered edges. One CTA per position walks its
// cells in the read order and writes, per slot, the cell's row, where its
// edges start and how many there are (0 for a skipped row); it also copies
// the cell's packed edges there, padded with -1 to a multiple of four, so
// that the read fetches a cell's edges four at a time with one aligned
// 16-byte load and the cells of a warp find theirs side by side. Position g's
// edges start at a multiple of four at or after
// seg_ptr[q0] + 3 * (q0 + g), which leaves room for its padding.
constexpr int kSlotThreads = 256;

__host__ __device__ inline int64_t slot_region(int64_t first_edge, int64_t first_row, int64_t g) {
  return (first_edge + 3 * (first_row + g) + 3) & ~int64_t(3);
}

__global__ void __launch_bounds__(kSlotThreads) slots_kernel(
    const int32_t* __restrict__ packed, const int64_t* __restrict__ seg_ptr, const int64_t* __restrict__ skip_ptr,
    const int64_t* __restrict__ order, const int64_t* __restrict__ q_off, int64_t n_q, int4* __restrict__ slots,
    int32_t* __restrict__ out, int64_t out_len) {
  __shared__ int warp_sums[kSlotThreads / 32];
  __shared__ int64_t carry;
  const int64_t g = blockIdx.x;
  const int64_t q0 = q_off[g], q1 = q_off[g + 1];
  if (q0 < 0 || q1 < q0 || q1 > n_q) {
    if (threadIdx.x == 0) report(ERR_RUN_BOUND);
    return;
  }
  if (threadIdx.x == 0) carry = slot_region(seg_ptr[q0], q0, g);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t c0 = q0; c0 < q1; c0 += kSlotThreads) {
    const int64_t i = c0 + threadIdx.x;
    int64_t row = -1, beg = 0;
    int n = 0;
    if (i < q1) {
      row = order ? order[i] : i;
      if (row >= q0 && row < q1) {
        beg = seg_ptr[row];
        n = (int)(seg_ptr[row + 1] - beg);
        if (skip_ptr && skip_ptr[row + 1] > skip_ptr[row]) n = 0;
      } else {
        report(ERR_INDEX);  // the order must permute the position's own rows
        row = -1;
      }
    }
    const int padded = (n + 3) & ~3;
    int incl = padded;  // inclusive scan over the block
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kSlotThreads / 32; ++w) {
      if (w < warp) before += warp_sums[w];
      total += warp_sums[w];
    }
    const int64_t start = carry + before + incl - padded;
    if (i < q1) {
      const bool fits = start + padded <= out_len && start <= INT32_MAX;
      if (!fits) report(ERR_RUN_BOUND);
      slots[i] = make_int4((int)row, fits ? (int)start : 0, fits ? n : 0, 0);
      if (fits)
        for (int j = 0; j < padded; ++j) out[start + j] = j < n ? packed[beg + j] : -1;
    }
    __syncthreads();  // warp sums and carry read
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
}

// ------------------------------------------------------------ attention
// q . k over one head (32 columns): q as 16 packed pairs, k as 4 x 8 bf16;
// four independent partial sums keep the dependent chains short.
__device__ __forceinline__ float dot32(const uint64_t (&q2)[16], const uint4 (&k)[4]) {
  uint64_t d[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    d[i] = mul2(q2[4 * i], bf2(k[i].x));
    d[i] = fma2(q2[4 * i + 1], bf2(k[i].y), d[i]);
    d[i] = fma2(q2[4 * i + 2], bf2(k[i].z), d[i]);
    d[i] = fma2(q2[4 * i + 3], bf2(k[i].w), d[i]);
  }
  const uint64_t t = add2(add2(d[0], d[1]), add2(d[2], d[3]));
  float a, b;
  unpack2(t, a, b);
  return a + b;
}

// One edge of a (cell, head): the online-softmax update with the score and
// the edge's value row (+ class value row), both 4 x 8 bf16.
constexpr float kSlack = 8.f;

template <bool HAS_VCLS>
__device__ __forceinline__ void edge_update(float score, const uint4 (&vr)[4], const uint4 (&cr)[4], float& m,
                                            float& l, uint64_t (&acc)[16]) {
  // The reference point m is raised only when a score passes it by more than
  // kSlack (or on the first edge, m = -inf), so the rescale runs about once
  // per run; weights exp(score - m) stay below exp(kSlack), well inside fp32.
  if (score > m + kSlack) {
    const float corr = __expf(m - score);  // m = -inf before the first edge: exp(-inf) = 0
    l *= corr;
    const uint64_t c2 = pack2(corr, corr);
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = mul2(acc[i], c2);
    m = score;
  }
  const float p = __expf(score - m);
  l += p;
  const uint64_t p2 = pack2(p, p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w[4] = {vr[i].x, vr[i].y, vr[i].z, vr[i].w};
    const uint32_t c[4] = {cr[i].x, cr[i].y, cr[i].z, cr[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint64_t v2 = bf2(w[j]);
      if constexpr (HAS_VCLS) v2 = add2(v2, bf2(c[j]));
      acc[4 * i + j] = fma2(p2, v2, acc[4 * i + j]);
    }
  }
}

template <typename TO, bool HAS_VCLS>
__global__ void __launch_bounds__(kThreads, 2) radius_read_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, int64_t ldkv, int64_t n_q, int64_t n_src, const float* __restrict__ bias,
    int64_t n_cls, const __nv_bfloat16* __restrict__ vcls, int64_t ld_vcls, const int64_t* __restrict__ seg_ptr,
    const int32_t* __restrict__ packed, const int64_t* __restrict__ skip_ptr, const int64_t* __restrict__ q_off,
    const int64_t* __restrict__ s_off, const int64_t* __restrict__ order, const int4* __restrict__ slots,
    int stage_rows, int split, TO* __restrict__ out, int64_t ldo, float scale) {
  extern __shared__ __align__(16) unsigned char smem[];
  // `split` CTAs share a group's rows (small batches: more CTAs than groups)
  const int grp = blockIdx.x / split, part = blockIdx.x % split;
  const int cb = blockIdx.y * kCols;
  const int64_t q0 = q_off[grp], q1 = q_off[grp + 1], s0 = s_off[grp], s1 = s_off[grp + 1];
  if (q0 < 0 || q1 < q0 || q1 > n_q || s0 < 0 || s1 < s0 || s1 > n_src) {
    if (threadIdx.x == 0 && part == 0) report(ERR_RUN_BOUND);
    return;
  }
  const int64_t qa = q0 + (q1 - q0) * part / split, qb = q0 + (q1 - q0) * (part + 1) / split;  // this CTA's slots
  if (qb == qa) return;
  const int64_t ns = s1 - s0;
  const bool staged = ns <= stage_rows;

  // bias [head][class] fp32, class value rows [class][64 columns] bf16, then
  // the stones' K|V rows [stone][K 64 | V 64] bf16 (16-byte units swizzled)
  const int bias_bytes = (int)((kHeads * n_cls * 4 + 15) / 16 * 16);
  const int vcls_bytes = HAS_VCLS ? (int)(n_cls * kClsRowBytes) : 0;
  float* bias_s = reinterpret_cast<float*>(smem);
  unsigned char* vcls_s = smem + bias_bytes;
  unsigned char* kv_s = smem + bias_bytes + vcls_bytes;
  const int head0 = cb / 32;
  for (int64_t i = threadIdx.x; i < kHeads * n_cls; i += blockDim.x) bias_s[i] = bias[head0 * n_cls + i];
  auto cp16 = [](void* dst, const void* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
  };
  if constexpr (HAS_VCLS) {
    constexpr int per_row = kClsRowBytes / 16;
    for (int64_t i = threadIdx.x; i < n_cls * per_row; i += blockDim.x) {
      const int64_t c = i / per_row;
      const uint32_t u = (uint32_t)(i % per_row);
      cp16(vcls_s + c * kClsRowBytes + unit_off(u),
           reinterpret_cast<const unsigned char*>(vcls + c * ld_vcls + cb) + u * 16);
    }
  }
  if (staged) {
    constexpr int per_half = kCols * 2 / 16;  // 16-byte units of the K (or V) columns
    for (int64_t i = threadIdx.x; i < ns * 2 * per_half; i += blockDim.x) {
      const int64_t r = i / (2 * per_half);
      const uint32_t u = (uint32_t)(i % (2 * per_half));
      const __nv_bfloat16* g = (u < per_half ? k : v) + (s0 + r) * ldkv + cb;
      cp16(kv_s + r * kKvRowBytes + unit_off(u),
           reinterpret_cast<const unsigned char*>(g) + (u % per_half) * 16);
    }
  }
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hh = lane % kHeads;           // head within the CTA
  const int ci = lane / kHeads;           // cell within the warp's sixteen
  const int rot = ci & 3;                 // unit rotation (see unit_off)
  const float* bias_h = bias_s + hh * n_cls;
  const int col = cb + hh * 32;           // this thread's first column
  // A cell's (row, first edge, edge count): from the slot table when there is
  // one (one 16-byte load, the next batch's requested a batch ahead), else
  // from the order, run bounds and skip runs.
  constexpr int64_t kStep = (kThreads / 32) * kCellsPerWarp;
  auto cell_of = [&](int64_t slot, int64_t& row, int64_t& beg, int& n) {
    row = order ? order[slot] : slot;
    beg = 0;
    n = 0;
    if (row >= q0 && row < q1) {
      beg = seg_ptr[row];
      n = (int)(seg_ptr[row + 1] - beg);
      if (skip_ptr && skip_ptr[row + 1] > skip_ptr[row]) n = 0;
    }
  };
  int4 next_info = make_int4(0, 0, 0, 0);
  if (slots && qa + warp * kCellsPerWarp + ci < qb) next_info = __ldg(slots + qa + warp * kCellsPerWarp + ci);
  for (int64_t base = qa + warp * kCellsPerWarp; base < qb; base += kStep) {
    const int64_t slot = base + ci;
    const bool rv = slot < qb;
    int64_t row = 0, beg = 0;
    int n = 0;
    if (rv) {
      if (slots) {
        row = next_info.x;
        beg = next_info.y;
        n = next_info.z;
      } else {
        cell_of(slot, row, beg, n);
      }
    }
    if (slots && slot + kStep < qb) next_info = __ldg(slots + slot + kStep);
    const bool own = rv && row >= q0 && row < q1;  // the order must permute the position's own rows
    if (rv && !own) report(ERR_INDEX);
    if (!own) n = 0;
    uint64_t q2[16];
    if (own) {
      const uint4* qp = reinterpret_cast<const uint4*>(q + row * ldq + col);
      const uint64_t s2 = pack2(scale, scale);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 w = __ldg(qp + ((i + rot) & 3));
        q2[4 * i] = mul2(bf2(w.x), s2);
        q2[4 * i + 1] = mul2(bf2(w.y), s2);
        q2[4 * i + 2] = mul2(bf2(w.z), s2);
        q2[4 * i + 3] = mul2(bf2(w.w), s2);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) q2[i] = 0;
    }
    float m = -INFINITY, l = 0.f;
    uint64_t acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0;
    const int32_t* pe = packed + beg;
    auto edge = [&](int pk) {
      if (pk < 0) return;  // padding, or refused when packing (reported there)
      const uint32_t s = (uint32_t)pk >> kClsBits, c = (uint32_t)pk & ((1u << kClsBits) - 1);
      // every row of the edge requested before any is used; unit i of this
      // lane is its head's unit (i + rot) mod 4
      uint4 kr[4], vr[4], cr[4];
      if (staged) {
        const unsigned char* ra = kv_s + s * kKvRowBytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t u = hh * 4 + ((i + rot) & 3);
          kr[i] = *reinterpret_cast<const uint4*>(ra + unit_off(u));
          vr[i] = *reinterpret_cast<const uint4*>(ra + unit_off(8 + u));
        }
      } else {
        const uint4* kp = reinterpret_cast<const uint4*>(k + (s0 + s) * ldkv + col);
        const uint4* vp = reinterpret_cast<const uint4*>(v + (s0 + s) * ldkv + col);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          kr[i] = __ldg(kp + ((i + rot) & 3));
          vr[i] = __ldg(vp + ((i + rot) & 3));
        }
      }
      if constexpr (HAS_VCLS) {
        const unsigned char* ca = vcls_s + c * kClsRowBytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) cr[i] = *reinterpret_cast<const uint4*>(ca + unit_off(hh * 4 + ((i + rot) & 3)));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) cr[i] = make_uint4(0, 0, 0, 0);
      }
      const float score = dot32(q2, kr) + bias_h[c];
      edge_update<HAS_VCLS>(score, vr, cr, m, l, acc);
    };
    if (slots) {
      // slot-ordered edges: a cell's run starts at a multiple of four and is
      // padded with -1, so four indices come with one 16-byte load
      const int4* pe4 = reinterpret_cast<const int4*>(pe);
      int4 nxt4 = n > 0 ? __ldg(pe4) : make_int4(-1, -1, -1, -1);
#pragma unroll 1
      for (int j = 0; j < n; j += 4) {
        const int4 cur = nxt4;
        if (j + 4 < n) nxt4 = __ldg(pe4 + (j >> 2) + 1);
        edge(cur.x);
        edge(cur.y);
        edge(cur.z);
        edge(cur.w);
      }
    } else {
      int nxt = n > 0 ? __ldg(pe) : -1;
#pragma unroll 1
      for (int j = 0; j < n; ++j) {
        const int pk = nxt;
        nxt = j + 1 < n ? __ldg(pe + j + 1) : -1;
        edge(pk);
      }
    }
    if (own) {
      const float inv = l > 0.f ? 1.f / l : 0.f;  // an empty run reads zero
      float o[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        unpack2(acc[i], o[2 * i], o[2 * i + 1]);
        o[2 * i] *= inv;
        o[2 * i + 1] *= inv;
      }
      TO* orow = out + row * ldo + col;
#pragma unroll
      for (int i = 0; i < 4; ++i) store_vec<8>(orow + 8 * ((i + rot) & 3), o + 8 * i);
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

int mb_radius_slots_size(int64_t n_q, int64_t n_groups, int64_t n_edges, int64_t* len) {
  MB_REQUIRE(len != nullptr, "radius_slots_size: len is NULL");
  MB_REQUIRE(n_q >= 0 && n_groups >= 0 && n_edges >= 0, "radius_slots_size: negative size");
  *len = radius::slot_region(n_edges, n_q, n_groups) + 4;
  return MB_OK;
}

int mb_radius_slots(const int32_t* packed, const int64_t* seg_ptr, const int64_t* skip_ptr, const int64_t* order,
                    const int64_t* q_off, int64_t n_groups, int64_t n_q, int64_t n_edges, int32_t* slots,
                    int32_t* packed_slots, int64_t packed_slots_len, void* stream) {
  MB_REQUIRE(n_q >= 0 && n_edges >= 0 && n_groups >= 0, "radius_slots: negative size");
  MB_REQUIRE(n_q <= INT32_MAX, "radius_slots: rows must fit int32");
  const int64_t need = radius::slot_region(n_edges, n_q, n_groups) + 4;
  MB_REQUIRE(need <= INT32_MAX, "radius_slots: padded edges must fit int32");
  MB_REQUIRE(packed_slots_len >= need, "radius_slots: packed_slots holds %lld entries, %lld needed",
             (long long)packed_slots_len, (long long)need);
  if (n_q == 0 || n_groups == 0) return MB_OK;
  MB_REQUIRE(packed && seg_ptr && q_off && slots && packed_slots, "radius_slots: null pointer");
  MB_REQUIRE(aligned(slots, 16) && aligned(packed_slots, 16), "radius_slots: slots and packed_slots must be 16-byte aligned");
  MB_REQUIRE(n_groups <= INT32_MAX, "radius_slots: too many groups");
  radius::slots_kernel<<<(unsigned)n_groups, radius::kSlotThreads, 0, as_stream(stream)>>>(
      packed, seg_ptr, skip_ptr, order, q_off, n_q, reinterpret_cast<int4*>(slots), packed_slots, packed_slots_len);
  return launch_status("radius_slots");
}

int mb_radius_read(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int64_t n_q, int64_t n_src,
                   int heads, int head_dim, const float* bias, int64_t n_cls, const void* vcls,
                   const int64_t* seg_ptr, const int32_t* packed, const int64_t* skip_ptr, const int64_t* q_off,
                   const int64_t* s_off, const int64_t* order, const int32_t* slots, int64_t n_groups,
                   int64_t stage_rows, void* out, int out_dtype, int64_t ldo, void* stream) {
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
  MB_REQUIRE(!slots || aligned(slots, 16), "radius_read: slots must be 16-byte aligned");
  const int64_t H = (int64_t)heads * head_dim;
  const int fixed = (int)((radius::kHeads * n_cls * 4 + 15) / 16 * 16) + (vcls ? (int)(n_cls * radius::kClsRowBytes) : 0);
  const int limit = 227 * 1024 / 2;  // two CTAs per SM
  MB_REQUIRE(fixed + radius::kKvRowBytes <= limit, "radius_read: %lld classes do not fit shared memory", (long long)n_cls);
  // groups with more stones than fit read K/V from global memory instead
  const int64_t rows = std::min<int64_t>(stage_rows, (limit - fixed) / radius::kKvRowBytes);
  const int smem = fixed + (int)rows * radius::kKvRowBytes;
  const float scale = 1.f / sqrtf((float)head_dim);
  // Enough CTAs for two per SM: a small batch's groups are split over
  // several CTAs (each at least one 128-row step on average).
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t col_blocks = H / radius::kCols;
  const int64_t want = (2 * (int64_t)sms + n_groups * col_blocks - 1) / (n_groups * col_blocks);
  const int64_t most = std::max<int64_t>(1, n_q / (n_groups * radius::kThreads / radius::kHeads));
  const int split = (int)std::max<int64_t>(1, std::min<int64_t>({want, most, 64}));
  MB_REQUIRE(n_groups * split <= INT32_MAX, "radius_read: too many groups");
  dim3 grid((unsigned)(n_groups * split), (unsigned)col_blocks);
  int rc = MB_OK;
  MB_DISPATCH_T(out_dtype, TO, [&] {
    auto kern = vcls ? radius::radius_read_kernel<TO, true> : radius::radius_read_kernel<TO, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      rc = fail(MB_LAUNCH_FAILED, "radius_read: %d bytes of shared memory refused", smem);
      return;
    }
    kern<<<grid, radius::kThreads, smem, as_stream(stream)>>>(
        (const __nv_bfloat16*)q, ldq, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, ldkv, n_q, n_src, bias, n_cls,
        (const __nv_bfloat16*)vcls, H, seg_ptr, packed, skip_ptr, q_off, s_off, order,
        reinterpret_cast<const int4*>(slots), (int)rows, split, (TO*)out, ldo, scale);
  });
  if (rc != MB_OK) return rc;
  return launch_status("radius_read");
}

}  // extern "C"
