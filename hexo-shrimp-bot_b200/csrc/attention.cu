// Attention kernels of the MantisNet trunk (CUDA cores, fp32 math):
//
//  K3  typed segment attention (cells<-windows, cells<-stones radius,
//      windows<-cells, cell adjacency): one warp per query row covering every
//      head; lane l holds VEC columns, lanes_per_head = head_dim / VEC lanes
//      share one head. Edges are consumed two at a time so two gathered K/V
//      rows are in flight per warp.
//  K1  stone attention over [4 latents; stones] per position: one thread per
//      query row, K/V tiles staged in shared memory as fp32 and read by
//      broadcast, online softmax in chunks of 8 keys.
//  K4  window-latent read (block per position, warps split the window run,
//      merged through shared memory), broadcast (warp per window) and the
//      dense 4x4 latent mix.
//
// Scores use exp(x - running max); an empty run returns zero with l = 0.
#include <math.h>

#include <type_traits>

#include "common.cuh"

namespace mb {

constexpr float kNegInf = -INFINITY;

// ------------------------------------------------------- segment attention
// One warp per query row, blocks of 8 warps over consecutive rows, scheduled
// in row order: the GPU works on a narrow band of positions at a time, so the
// gathered source rows stay L2-resident. Two edges per iteration keep two
// K/V row pairs in flight per lane at 80 registers (3 blocks per SM); wider
// per-lane pipelines were measured slower at the bench's sizes because they
// cost resident warps.
constexpr int kSegWarps = 8;

template <typename T, typename TO, typename TV, int VEC, bool HAS_VCLS>
__global__ void __launch_bounds__(kSegWarps * 32) segment_attention_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, const T* __restrict__ v, int64_t ldkv, int64_t n_q,
    int64_t n_src, int heads, int hd, const float* __restrict__ bias, int64_t n_cls, const TV* __restrict__ vcls,
    const int64_t* __restrict__ seg_ptr, const int64_t* __restrict__ src, const int64_t* __restrict__ cls,
    const int64_t* __restrict__ skip_ptr, TO* __restrict__ out, int64_t ldo, float* __restrict__ m_out,
    float* __restrict__ l_out, float scale) {
  const int64_t row = (int64_t)blockIdx.x * kSegWarps + (threadIdx.x >> 5);
  if (row >= n_q) return;
  const int lane = threadIdx.x & 31;
  const int lph = hd / VEC;  // lanes per head
  const int head = lane / lph;
  const int H = heads * hd;
  const int col = lane * VEC;
  // Widths below one warp (H < 32, VEC == 1) leave the upper lanes idle; they
  // still join the shuffles with zero partial sums.
  const bool live = col < H;
  float qv[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) qv[i] = 0.f;
  if (live) load_vec<VEC>(q + row * ldq + col, qv);
#pragma unroll
  for (int i = 0; i < VEC; ++i) qv[i] *= scale;
  int64_t beg = seg_ptr[row], end = seg_ptr[row + 1];
  if (skip_ptr && skip_ptr[row + 1] > skip_ptr[row]) end = beg;
  const float* brow = bias + (int64_t)(live ? head : 0) * n_cls;
  float m = kNegInf, l = 0.f, acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;

  auto consume = [&](float score, const float* vv) {
    const float m_new = fmaxf(m, score);
    const float corr = __expf(m - m_new);
    const float p = __expf(score - m_new);
    l = l * corr + p;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = acc[i] * corr + p * vv[i];
    m = m_new;
  };
  auto add_class_row = [&](int64_t c, float* vv) {
    if constexpr (HAS_VCLS) {
      if (live) {
        float a[VEC];
        load_vec<VEC>(vcls + c * H + col, a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) vv[i] += a[i];
      }
    }
  };

  int64_t e = beg;
  for (; e + 1 < end; e += 2) {
    const int64_t s0 = src[e], s1 = src[e + 1], c0 = cls[e], c1 = cls[e + 1];
    if (s0 < 0 || s0 >= n_src || s1 < 0 || s1 >= n_src || c0 < 0 || c0 >= n_cls || c1 < 0 || c1 >= n_cls) {
      report(ERR_INDEX);
      continue;
    }
    float k0[VEC] = {}, k1[VEC] = {}, v0[VEC] = {}, v1[VEC] = {};
    if (live) {
      load_vec<VEC>(k + s0 * ldkv + col, k0);
      load_vec<VEC>(k + s1 * ldkv + col, k1);
      load_vec<VEC>(v + s0 * ldkv + col, v0);
      load_vec<VEC>(v + s1 * ldkv + col, v1);
    }
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) { d0 += qv[i] * k0[i]; d1 += qv[i] * k1[i]; }
    d0 = group_sum(d0, lph) + __ldg(brow + c0);
    d1 = group_sum(d1, lph) + __ldg(brow + c1);
    add_class_row(c0, v0);
    add_class_row(c1, v1);
    consume(d0, v0);
    consume(d1, v1);
  }
  if (e < end) {
    const int64_t s0 = src[e], c0 = cls[e];
    if (s0 < 0 || s0 >= n_src || c0 < 0 || c0 >= n_cls) {
      report(ERR_INDEX);
    } else {
      float k0[VEC] = {}, v0[VEC] = {};
      if (live) {
        load_vec<VEC>(k + s0 * ldkv + col, k0);
        load_vec<VEC>(v + s0 * ldkv + col, v0);
      }
      float d0 = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) d0 += qv[i] * k0[i];
      d0 = group_sum(d0, lph) + __ldg(brow + c0);
      add_class_row(c0, v0);
      consume(d0, v0);
    }
  }
  const float inv = l > 0.f ? 1.f / l : 1.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] *= inv;
  if (!live) return;
  store_vec<VEC>(out + row * ldo + col, acc);
  if (m_out && (lane % lph) == 0) {
    m_out[row * heads + head] = m;
    l_out[row * heads + head] = l;
  }
}

// --------------------------------------------------------- stone attention
constexpr int kStoneThreads = 128;
constexpr int kKeyTile = 64;

template <typename T, typename TO, int D>
__global__ void __launch_bounds__(kStoneThreads) stone_attention_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, int64_t s_pos, int64_t s_head,
    int64_t s_row, const int32_t* __restrict__ seq_lens, int64_t t_pad, const int64_t* __restrict__ tok_off,
    int max_queries, TO* __restrict__ out, int64_t o_pos, int64_t o_head, int64_t o_row, float scale) {
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
  }
}

// ------------------------------------------------------- window latents
constexpr int kReadWarps = 8;

template <typename T, typename TO, int VEC>
__global__ void __launch_bounds__(kReadWarps * 32) latent_read_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, const T* __restrict__ v, int64_t ldkv,
    int64_t n_windows, int heads, int hd, const int64_t* __restrict__ offsets, const int64_t* __restrict__ order,
    TO* __restrict__ out, float* __restrict__ m_out, float* __restrict__ l_out, float scale) {
  extern __shared__ float smem[];
  const int64_t p = blockIdx.x;
  const int H = heads * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lph = hd / VEC;
  const int head = lane / lph;
  const int chunks = (H + 32 * VEC - 1) / (32 * VEC);  // column chunks per row
  const int64_t beg = offsets[p], end = offsets[p + 1];
  // shared layout: [warp][slot][H] acc, then [warp][slot][heads] m and l
  float* s_acc = smem;
  float* s_m = s_acc + kReadWarps * 4 * H;
  float* s_l = s_m + kReadWarps * 4 * heads;
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
    for (int64_t i = beg + warp; i < end; i += kReadWarps) {
      const int64_t w = order[i];
      if (w < 0 || w >= n_windows) { report(ERR_INDEX); continue; }
      float kv[VEC] = {}, vv[VEC] = {};
      if (live) {
        load_vec<VEC>(k + w * ldkv + col, kv);
        load_vec<VEC>(v + w * ldkv + col, vv);
      }
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
  (void)head;
  __syncthreads();
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
    out[(p * 4 + s) * H + col] = from_f<TO>(ll > 0.f ? aa / ll : 0.f);
    if (m_out && (col % hd) == 0) {
      m_out[(p * 4 + s) * heads + hh] = mm;
      l_out[(p * 4 + s) * heads + hh] = ll;
    }
  }
}

template <typename T, typename TO, int VEC>
__global__ void __launch_bounds__(256) latent_broadcast_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, const T* __restrict__ v, int64_t ldkv,
    int64_t n_pos, int64_t n_windows, int heads, int hd, const int64_t* __restrict__ window_pos, TO* __restrict__ out,
    float* __restrict__ m_out, float* __restrict__ l_out, float scale) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= n_windows) return;
  const int lane = threadIdx.x & 31;
  const int H = heads * hd;
  const int lph = hd / VEC;
  const int64_t p = window_pos[w];
  if (p < 0 || p >= n_pos) { report(ERR_INDEX); return; }
  for (int c0 = 0; c0 < H; c0 += 32 * VEC) {
    const int col = c0 + lane * VEC;
    const bool live = col < H;  // H < 32 leaves upper lanes idle
    float qv[VEC] = {}, sc[4], mx = kNegInf;
    if (live) load_vec<VEC>(q + w * ldq + col, qv);
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      float kv[VEC] = {};
      if (live) load_vec<VEC>(k + (p * 4 + s) * ldkv + col, kv);
      float d = 0.f;
#pragma unroll
      for (int u = 0; u < VEC; ++u) d += qv[u] * kv[u];
      sc[s] = group_sum(d, lph) * scale;
      mx = fmaxf(mx, sc[s]);
    }
    float l = 0.f, acc[VEC];
#pragma unroll
    for (int u = 0; u < VEC; ++u) acc[u] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const float pr = __expf(sc[s] - mx);
      l += pr;
      float vv[VEC] = {};
      if (live) load_vec<VEC>(v + (p * 4 + s) * ldkv + col, vv);
#pragma unroll
      for (int u = 0; u < VEC; ++u) acc[u] += pr * vv[u];
    }
    const float inv = 1.f / l;
#pragma unroll
    for (int u = 0; u < VEC; ++u) acc[u] *= inv;
    if (!live) continue;
    store_vec<VEC>(out + w * H + col, acc);
    if (m_out && lane % lph == 0) {
      m_out[w * heads + col / hd] = mx;
      l_out[w * heads + col / hd] = l;
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
  MB_REQUIRE(heads > 0 && head_dim > 0 && n_q >= 0, "segment_attention: bad sizes");
  if (n_q == 0) return MB_OK;
  const int H = heads * head_dim;
  const int vec = attn_vec(heads, head_dim);
  MB_REQUIRE(vec > 0 && H <= 32 * vec, "segment_attention: unsupported heads=%d head_dim=%d", heads, head_dim);
  MB_REQUIRE(q && out && seg_ptr && bias, "segment_attention: null pointer");
  MB_REQUIRE((m == nullptr) == (l == nullptr), "segment_attention: m and l go together");
  MB_REQUIRE(valid_dtype(vcls_dtype), "segment_attention: bad vcls dtype");
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  dim3 grid((unsigned)cdiv(n_q, kSegWarps));
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

int mb_stone_attention(const void* q, const void* k, const void* v, int dtype, int64_t n_pos, int heads, int head_dim,
                       int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* seq_lens, int64_t t_pad,
                       const int64_t* tok_off, int64_t max_tokens, int max_queries, void* out, int out_dtype,
                       int64_t o_pos, int64_t o_head, int64_t o_row, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "stone_attention: bad dtype");
  MB_REQUIRE(head_dim == 16 || head_dim == 32 || head_dim == 64, "stone_attention: head_dim %d unsupported", head_dim);
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(q && k && v && out, "stone_attention: null pointer");
  MB_REQUIRE(tok_off || seq_lens, "stone_attention: need seq_lens (padded) or tok_off (ragged)");
  MB_REQUIRE(n_pos <= 65535 && heads <= 65535, "stone_attention: grid too large");
  const int64_t rows = tok_off ? (max_queries >= 0 ? max_queries : max_tokens) : t_pad;
  if (rows <= 0) return MB_OK;
  dim3 grid((unsigned)cdiv(rows, kStoneThreads), (unsigned)n_pos, (unsigned)heads);
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      auto go = [&](auto dtag) {
        constexpr int D = decltype(dtag)::value;
        stone_attention_kernel<T, TO, D><<<grid, kStoneThreads, 0, s>>>(
            (const T*)q, (const T*)k, (const T*)v, s_pos, s_head, s_row, seq_lens, t_pad, tok_off, max_queries,
            (TO*)out, o_pos, o_head, o_row, scale);
      };
      if (head_dim == 16) go(std::integral_constant<int, 16>{});
      else if (head_dim == 32) go(std::integral_constant<int, 32>{});
      else go(std::integral_constant<int, 64>{});
    });
  });
  return launch_status("stone_attention");
}

static int latent_vec(int heads, int head_dim) { return attn_vec(heads, head_dim); }

int mb_window_latent_read(const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, int dtype,
                          int64_t n_pos, int64_t n_windows, int heads, int head_dim, const int64_t* offsets,
                          const int64_t* order, void* out, int out_dtype, float* m, float* l, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(out_dtype), "window_latent_read: bad dtype");
  if (n_pos == 0) return MB_OK;
  const int vec = latent_vec(heads, head_dim);
  MB_REQUIRE(vec > 0, "window_latent_read: unsupported heads=%d head_dim=%d", heads, head_dim);
  MB_REQUIRE(q && out && offsets && (n_windows == 0 || (k && v && order)), "window_latent_read: null pointer");
  const int H = heads * head_dim;
  const size_t smem = sizeof(float) * (size_t)kReadWarps * 4 * (H + 2 * heads);
  MB_REQUIRE(smem <= 200 * 1024, "window_latent_read: width too large");
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        auto kern = latent_read_kernel<T, TO, V>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<(unsigned)n_pos, kReadWarps * 32, smem, s>>>((const T*)q, ldq, (const T*)k, (const T*)v, ldkv,
                                                            n_windows, heads, head_dim, offsets, order, (TO*)out, m,
                                                            l, scale);
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
        latent_broadcast_kernel<T, TO, V><<<(unsigned)cdiv(n_windows, 8), 256, 0, s>>>(
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
