// Bandwidth-bound row kernels: run reductions (K2), the action-row encoder
// (K5), the relay cell pass (K6), LayerNorm, embeddings, residual updates,
// token layout moves and the Q composition.
//
// Layout convention: one warp owns one destination row; lane l owns columns
// [c0 + l*VEC, c0 + l*VEC + VEC) of each 32*VEC-wide column chunk, so every
// gathered row is read with 16-byte vector loads, fully coalesced.
#include "common.cuh"

namespace mb {

constexpr int kWarps = 8;  // warps per block for row kernels

__device__ __forceinline__ int64_t warp_row() {
  return (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
}

// ---------------------------------------------------------- run reduce --
template <typename TV, typename TO, int VEC>
__global__ void __launch_bounds__(kWarps * 32) run_reduce_kernel(
    const TV* __restrict__ values, int64_t ldv, int64_t n_values, const int64_t* __restrict__ gather,
    const int64_t* __restrict__ ptr, int64_t n_dest, int64_t width, const float* __restrict__ add, int64_t ld_add,
    const int64_t* __restrict__ add_idx, int64_t n_add, TO* __restrict__ out, int64_t ldo) {
  const int64_t d = warp_row();
  if (d >= n_dest) return;
  const int lane = threadIdx.x & 31;
  const int64_t beg = ptr[d], end = ptr[d + 1];
  int64_t arow = -1;
  if (add) {
    arow = add_idx ? add_idx[d] : d;
    if (arow < 0 || arow >= n_add) { report(ERR_INDEX); arow = -1; }
  }
  for (int64_t c0 = 0; c0 < width; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= width) continue;  // only the VEC == 1 path has a ragged tail
    float acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
    int64_t e = beg;
    // two rows in flight per iteration
    for (; e + 1 < end; e += 2) {
      int64_t s0 = gather[e], s1 = gather[e + 1];
      if (s0 < 0 || s0 >= n_values || s1 < 0 || s1 >= n_values) { report(ERR_INDEX); continue; }
      float a[VEC], b[VEC];
      load_vec<VEC>(values + s0 * ldv + col, a);
      load_vec<VEC>(values + s1 * ldv + col, b);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += a[i] + b[i];
    }
    if (e < end) {
      int64_t s0 = gather[e];
      if (s0 < 0 || s0 >= n_values) {
        report(ERR_INDEX);
      } else {
        float a[VEC];
        load_vec<VEC>(values + s0 * ldv + col, a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] += a[i];
      }
    }
    if (arow >= 0) {
      float a[VEC];
      load_vec<VEC>(add + arow * ld_add + col, a);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += a[i];
    }
    store_vec<VEC>(out + d * ldo + col, acc);
  }
}

// --------------------------------------------------------- row encoder --
template <typename TP, typename TO, int VEC>
__global__ void __launch_bounds__(kWarps * 32) row_encode_kernel(
    const TP* __restrict__ pre, int64_t n_pre, const float* __restrict__ table, int64_t n_table,
    const int64_t* __restrict__ edge_window, const int64_t* __restrict__ edge_class,
    const int64_t* __restrict__ cell_ptr, int64_t n_cells, const int64_t* __restrict__ empty_counts,
    const float* __restrict__ empty_base, const int64_t* __restrict__ empty_cls, int n_empty, int64_t h,
    TO* __restrict__ out, int64_t ld_out) {
  const int64_t c = warp_row();
  if (c >= n_cells) return;
  const int lane = threadIdx.x & 31;
  const int64_t beg = cell_ptr[c], end = cell_ptr[c + 1];
  for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= h) continue;  // only the VEC == 1 path has a ragged tail
    float acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
    for (int64_t e = beg; e < end; ++e) {
      const int64_t w = edge_window[e], k = edge_class[e];
      if (w < 0 || w >= n_pre || k < 0 || k >= n_table) { report(ERR_INDEX); continue; }
      float a[VEC], b[VEC];
      load_vec<VEC>(pre + w * h + col, a);
      load_vec<VEC>(table + k * h + col, b);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += fmaxf(a[i] + b[i], 0.f);
    }
    if (empty_counts) {
      for (int o = 0; o < n_empty; ++o) {
        const float cnt = (float)empty_counts[c * n_empty + o];
        const int64_t k = empty_cls[o];
        float a[VEC], b[VEC];
        load_vec<VEC>(empty_base + col, a);
        load_vec<VEC>(table + k * h + col, b);
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] += cnt * fmaxf(a[i] + b[i], 0.f);
      }
    }
    store_vec<VEC>(out + c * ld_out + col, acc);
  }
}

// ---------------------------------------------------------- relay pass --
template <typename TX, int VEC>
__global__ void __launch_bounds__(kWarps * 32) relay_cells_kernel(
    const TX* __restrict__ x, int64_t n_windows, const float* __restrict__ emb, int64_t n_cls,
    const int64_t* __restrict__ cell_ptr, int64_t n_cov, const int64_t* __restrict__ edge_window,
    const int64_t* __restrict__ edge_class, int64_t h, float* __restrict__ val) {
  const int64_t c = warp_row();
  if (c >= n_cov) return;
  const int lane = threadIdx.x & 31;
  for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= h) continue;  // only the VEC == 1 path has a ragged tail
    float acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
    for (int64_t e = cell_ptr[c]; e < cell_ptr[c + 1]; ++e) {
      const int64_t w = edge_window[e], k = edge_class[e];
      if (w < 0 || w >= n_windows || k < 0 || k >= n_cls) { report(ERR_INDEX); continue; }
      float a[VEC], b[VEC];
      load_vec<VEC>(x + w * h + col, a);
      load_vec<VEC>(emb + k * h + col, b);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += a[i] + b[i];
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaxf(acc[i], 0.f);
    store_vec<VEC>(val + c * h + col, acc);
  }
}

// ----------------------------------------------------------- LayerNorm --
// Warp per row; the row lives in registers as CH chunks of 32 * VEC columns
// (h <= 32 * VEC * kMaxChunks). CH is a compile-time count so a 256-wide row
// costs 8 registers, not 32: the kernels are HBM streams and need every
// resident warp they can get to keep enough bytes in flight.
constexpr int kMaxChunks = 4;

inline int row_chunks(int64_t h, int vec) {
  const int64_t c = cdiv(h, 32 * (int64_t)vec);
  return c <= 1 ? 1 : (c <= 2 ? 2 : 4);
}

template <typename TX, typename TO, int VEC, int CH>
__global__ void __launch_bounds__(kWarps * 32) layer_norm_kernel(
    const TX* __restrict__ x, int64_t ldx, const int64_t* __restrict__ in_rows, int64_t n, int64_t h,
    const float* __restrict__ gamma, const float* __restrict__ beta, float eps, TO* __restrict__ out, int64_t ldo) {
  const int64_t r = warp_row();
  if (r >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t src = in_rows ? in_rows[r] : r;
  const int chunks = (int)((h + 32 * VEC - 1) / (32 * VEC));
  float v[CH][VEC];
  float sum = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int64_t col = ch * 32 * VEC + lane * VEC;
    const bool live = ch < chunks && col < h;  // ragged tail only when VEC == 1
    if (live) {
      load_vec<VEC>(x + src * ldx + col, v[ch]);
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum += v[ch][i];
    }
  }
  const float mean = warp_sum(sum) / (float)h;
  float sq = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int64_t col = ch * 32 * VEC + lane * VEC;
    if (ch < chunks && col < h) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float d = v[ch][i] - mean;
        sq += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / (float)h + eps);
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int64_t col = ch * 32 * VEC + lane * VEC;
    if (ch < chunks && col < h) {
      float g[VEC], b[VEC], o[VEC];
      load_vec<VEC>(gamma + col, g);
      load_vec<VEC>(beta + col, b);
#pragma unroll
      for (int i = 0; i < VEC; ++i) o[i] = (v[ch][i] - mean) * rstd * g[i] + b[i];
      store_vec<VEC>(out + r * ldo + col, o);
    }
  }
}

// ------------------------------------------- residual update + LayerNorms --
// x[r] += y[r] (+ y_bias), then up to three LayerNorms of the updated row, each
// with its own affine parameters, destination and dtype: one read and one
// write of the residual row feed every consumer that normalises it next.
struct LnOut {
  const float* g;
  const float* b;
  void* out;
  int dtype;
  int64_t ld;
};

template <int VEC>
__device__ __forceinline__ void ln_store(const LnOut& o, int64_t r, int64_t col, const float* v, float mean,
                                         float rstd) {
  float g[VEC], b[VEC], y[VEC];
  load_vec<VEC>(o.g + col, g);
  load_vec<VEC>(o.b + col, b);
#pragma unroll
  for (int i = 0; i < VEC; ++i) y[i] = (v[i] - mean) * rstd * g[i] + b[i];
  if (o.dtype == MB_BF16)
    store_vec<VEC>(reinterpret_cast<__nv_bfloat16*>(o.out) + r * o.ld + col, y);
  else
    store_vec<VEC>(reinterpret_cast<float*>(o.out) + r * o.ld + col, y);
}

template <typename TY, int VEC, int CH>
__global__ void __launch_bounds__(kWarps * 32) add_ln_kernel(float* __restrict__ x, int64_t ldx,
                                                             const TY* __restrict__ y, int64_t ldy,
                                                             const float* __restrict__ y_bias, int64_t n, int64_t h,
                                                             float eps, int n_out, LnOut o0, LnOut o1, LnOut o2) {
  const int64_t r = warp_row();
  if (r >= n) return;
  const int lane = threadIdx.x & 31;
  const int chunks = (int)((h + 32 * VEC - 1) / (32 * VEC));
  float v[CH][VEC];
  float sum = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int64_t col = ch * 32 * VEC + lane * VEC;
    if (ch < chunks && col < h) {
      load_vec<VEC>(x + r * ldx + col, v[ch]);
      if (y) {
        float a[VEC];
        load_vec<VEC>(y + r * ldy + col, a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[ch][i] += a[i];
        if (y_bias) {
          load_vec<VEC>(y_bias + col, a);
#pragma unroll
          for (int i = 0; i < VEC; ++i) v[ch][i] += a[i];
        }
        store_vec<VEC>(x + r * ldx + col, v[ch]);
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) sum += v[ch][i];
    }
  }
  if (n_out == 0) return;
  const float mean = warp_sum(sum) / (float)h;
  float sq = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int64_t col = ch * 32 * VEC + lane * VEC;
    if (ch < chunks && col < h) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float d = v[ch][i] - mean;
        sq += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / (float)h + eps);
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int64_t col = ch * 32 * VEC + lane * VEC;
    if (ch < chunks && col < h) {
      ln_store<VEC>(o0, r, col, v[ch], mean, rstd);
      if (n_out > 1) ln_store<VEC>(o1, r, col, v[ch], mean, rstd);
      if (n_out > 2) ln_store<VEC>(o2, r, col, v[ch], mean, rstd);
    }
  }
}

// ------------------------------------------------------------ misc rows --
template <int VEC>
__global__ void __launch_bounds__(kWarps * 32) embed_kernel(
    const float* __restrict__ ta, int64_t n_ta, const int64_t* __restrict__ ia, const float* __restrict__ tb,
    int64_t n_tb, const int64_t* __restrict__ ib, int64_t n, int64_t h, float* __restrict__ out) {
  const int64_t r = warp_row();
  if (r >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t a = ia ? ia[r] : r;
  int64_t b = tb ? (ib ? ib[r] : r) : -1;
  if (a < 0 || a >= n_ta || (tb && (b < 0 || b >= n_tb))) { report(ERR_INDEX); return; }
  for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= h) continue;  // only the VEC == 1 path has a ragged tail
    float x[VEC], y[VEC];
    load_vec<VEC>(ta + a * h + col, x);
    if (tb) {
      load_vec<VEC>(tb + b * h + col, y);
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] += y[i];
    }
    store_vec<VEC>(out + r * h + col, x);
  }
}

template <int VEC>
__global__ void __launch_bounds__(kWarps * 32) cell_init_kernel(
    const int64_t* __restrict__ cov_ptr, const int64_t* __restrict__ nearest, const float* __restrict__ table,
    int64_t n_table, const float* __restrict__ covered_row, const float* __restrict__ covered_add, int64_t n_cells,
    int64_t h, float* __restrict__ out) {
  const int64_t r = warp_row();
  if (r >= n_cells) return;
  const int lane = threadIdx.x & 31;
  const bool covered = cov_ptr[r + 1] > cov_ptr[r];
  const int64_t k = nearest[r];
  if (!covered && (k < 0 || k >= n_table)) { report(ERR_INDEX); return; }
  for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= h) continue;  // only the VEC == 1 path has a ragged tail
    float x[VEC];
    if (covered) {
      load_vec<VEC>(covered_row + col, x);
      if (covered_add) {
        float y[VEC];
        load_vec<VEC>(covered_add + r * h + col, y);
#pragma unroll
        for (int i = 0; i < VEC; ++i) x[i] += y[i];
      }
    } else {
      load_vec<VEC>(table + k * h + col, x);
    }
    store_vec<VEC>(out + r * h + col, x);
  }
}

template <typename TX, typename TY, int VEC>
__global__ void __launch_bounds__(kWarps * 32) residual_add_kernel(
    TX* __restrict__ x, int64_t ldx, const int64_t* __restrict__ rows, const TY* __restrict__ y, int64_t ldy,
    int64_t n, int64_t h) {
  const int64_t r = warp_row();
  if (r >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t dst = rows ? rows[r] : r;
  for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= h) continue;  // only the VEC == 1 path has a ragged tail
    float a[VEC], b[VEC];
    load_vec<VEC>(x + dst * ldx + col, a);
    load_vec<VEC>(y + r * ldy + col, b);
#pragma unroll
    for (int i = 0; i < VEC; ++i) a[i] += b[i];
    store_vec<VEC>(x + dst * ldx + col, a);
  }
}

template <typename TX, typename TT, int VEC>
__global__ void __launch_bounds__(kWarps * 32) add_gather_kernel(
    TX* __restrict__ x, int64_t ldx, const TT* __restrict__ t, int64_t ldt, int64_t n_t,
    const int64_t* __restrict__ idx, int64_t n, int64_t h, int relu) {
  const int64_t r = warp_row();
  if (r >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t j = idx[r];
  if (j < 0 || j >= n_t) { report(ERR_INDEX); return; }
  for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
    const int64_t col = c0 + lane * VEC;
    if (col >= h) continue;  // only the VEC == 1 path has a ragged tail
    float a[VEC], b[VEC];
    load_vec<VEC>(x + r * ldx + col, a);
    load_vec<VEC>(t + j * ldt + col, b);
#pragma unroll
    for (int i = 0; i < VEC; ++i) a[i] = relu ? fmaxf(a[i] + b[i], 0.f) : a[i] + b[i];
    store_vec<VEC>(x + r * ldx + col, a);
  }
}

// Token row t of position p: latents first, then stones.
template <int VEC>
__global__ void __launch_bounds__(kWarps * 32) tokens_gather_kernel(
    const float* __restrict__ g, const float* __restrict__ s, const int64_t* __restrict__ stone_off,
    const int64_t* __restrict__ tok_off, int64_t n_pos, int64_t h, float* __restrict__ tok) {
  const int64_t p = blockIdx.y;
  const int64_t t0 = tok_off[p], n_t = tok_off[p + 1] - t0;
  const int lane = threadIdx.x & 31;
  for (int64_t t = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); t < n_t; t += (int64_t)gridDim.x * kWarps) {
    const float* src = t < 4 ? g + (p * 4 + t) * h : s + (stone_off[p] + t - 4) * h;
    for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
      if (c0 + lane * VEC >= h) continue;
      float a[VEC];
      load_vec<VEC>(src + c0 + lane * VEC, a);
      store_vec<VEC>(tok + (t0 + t) * h + c0 + lane * VEC, a);
    }
  }
}

template <typename TY, int VEC>
__global__ void __launch_bounds__(kWarps * 32) tokens_scatter_add_kernel(
    float* __restrict__ g, float* __restrict__ s, const int64_t* __restrict__ stone_off,
    const int64_t* __restrict__ tok_off, int64_t n_pos, int64_t h, const TY* __restrict__ tok, int update_stones) {
  const int64_t p = blockIdx.y;
  const int64_t t0 = tok_off[p], n_t = update_stones ? tok_off[p + 1] - t0 : 4;
  const int lane = threadIdx.x & 31;
  for (int64_t t = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); t < n_t; t += (int64_t)gridDim.x * kWarps) {
    float* dst = t < 4 ? g + (p * 4 + t) * h : s + (stone_off[p] + t - 4) * h;
    for (int64_t c0 = 0; c0 < h; c0 += 32 * VEC) {
      if (c0 + lane * VEC >= h) continue;
      float a[VEC], b[VEC];
      load_vec<VEC>(dst + c0 + lane * VEC, a);
      load_vec<VEC>(tok + (t0 + t) * h + c0 + lane * VEC, b);
#pragma unroll
      for (int i = 0; i < VEC; ++i) a[i] += b[i];
      store_vec<VEC>(dst + c0 + lane * VEC, a);
    }
  }
}

__global__ void latent_mean_kernel(const float* __restrict__ g, int64_t n_pos, int64_t h, float* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_pos * h) return;
  const int64_t p = i / h, c = i % h;
  const float* r = g + p * 4 * h + c;
  out[i] = (r[0] + r[h] + r[2 * h] + r[3 * h]) * 0.25f;
}

// Block per position: softmax of three logits per cell, then the position's
// maximum committed mass, floored.
__global__ void compose_q_kernel(const float* __restrict__ critic, int64_t ldc, const int64_t* __restrict__ offsets,
                                 int64_t n_pos, float floor_, float* __restrict__ q_score,
                                 float* __restrict__ q_values) {
  const int64_t p = blockIdx.x;
  const int64_t beg = offsets[p], end = offsets[p + 1];
  __shared__ float red[32];
  float mx = -3.402823466e38f;
  for (int64_t c = beg + threadIdx.x; c < end; c += blockDim.x) {
    const float* z = critic + c * ldc;
    const float m = fmaxf(z[0], fmaxf(z[1], z[2]));
    const float e0 = expf(z[0] - m), e1 = expf(z[1] - m), e2 = expf(z[2] - m);
    const float inv = 1.f / (e0 + e1 + e2);
    const float pp = e0 * inv, pn = e1 * inv;
    q_values[c] = pp - pn;
    mx = fmaxf(mx, pp + pn);
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -3.402823466e38f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = fmaxf(v, floor_);
  }
  __syncthreads();
  const float scale = red[0];
  for (int64_t c = beg + threadIdx.x; c < end; c += blockDim.x) q_score[c] = q_values[c] / scale;
}

static inline dim3 row_grid(int64_t n) { return dim3((unsigned)cdiv(n > 0 ? n : 1, kWarps)); }

}  // namespace mb

using namespace mb;

extern "C" {

int mb_run_reduce(const void* values, int values_dtype, int64_t ld_values, int64_t n_values, const int64_t* gather,
                  const int64_t* ptr, int64_t n_dest, int64_t width, const float* add, int64_t ld_add,
                  const int64_t* add_idx, int64_t n_add, void* out, int out_dtype, int64_t ld_out, void* stream) {
  MB_REQUIRE(valid_dtype(values_dtype) && valid_dtype(out_dtype), "run_reduce: bad dtype");
  MB_REQUIRE(n_dest >= 0 && width > 0, "run_reduce: bad sizes");
  if (n_dest == 0) return MB_OK;
  MB_REQUIRE(ptr && out && (values || n_values == 0), "run_reduce: null pointer");
  const int vec = row_vec(width);
  MB_REQUIRE(vec > 0, "run_reduce: bad width %lld", (long long)width);
  const int eb = vec * 4;
  MB_REQUIRE(aligned(out, vec * dtype_size(out_dtype)) && (ld_out * dtype_size(out_dtype)) % (vec * dtype_size(out_dtype)) == 0,
             "run_reduce: out misaligned");
  MB_REQUIRE(!values || (aligned(values, vec * dtype_size(values_dtype)) &&
                         (ld_values * dtype_size(values_dtype)) % (vec * dtype_size(values_dtype)) == 0),
             "run_reduce: values misaligned");
  MB_REQUIRE(!add || (aligned(add, eb) && (ld_add * 4) % eb == 0), "run_reduce: add misaligned");
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(values_dtype, TV, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        run_reduce_kernel<TV, TO, V><<<row_grid(n_dest), kWarps * 32, 0, s>>>(
            (const TV*)values, ld_values, n_values, gather, ptr, n_dest, width, add, ld_add, add_idx, n_add,
            (TO*)out, ld_out);
      });
    });
  });
  return launch_status("run_reduce");
}

int mb_row_encode(const void* pre, int pre_dtype, int64_t n_pre, const float* table, int64_t n_table,
                  const int64_t* edge_window, const int64_t* edge_class, const int64_t* cell_ptr, int64_t n_cells,
                  const int64_t* empty_counts, const float* empty_base, const int64_t* empty_cls, int n_empty,
                  int64_t h, void* out, int out_dtype, int64_t ld_out, void* stream) {
  MB_REQUIRE(valid_dtype(pre_dtype) && valid_dtype(out_dtype), "row_encode: bad dtype");
  if (n_cells == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0, "row_encode: bad width %lld", (long long)h);
  MB_REQUIRE(ld_out >= h && ld_out % vec == 0 && aligned(out, (size_t)vec * dtype_size(out_dtype)),
             "row_encode: output rows must hold h aligned columns (ld_out=%lld)", (long long)ld_out);
  MB_REQUIRE(table && cell_ptr && out, "row_encode: null pointer");
  MB_REQUIRE(!empty_counts || (empty_base && empty_cls && n_empty > 0), "row_encode: empty rows incomplete");
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(pre_dtype, TP, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        row_encode_kernel<TP, TO, V><<<row_grid(n_cells), kWarps * 32, 0, s>>>(
            (const TP*)pre, n_pre, table, n_table, edge_window, edge_class, cell_ptr, n_cells, empty_counts,
            empty_base, empty_cls, n_empty, h, (TO*)out, ld_out);
      });
    });
  });
  return launch_status("row_encode");
}

int mb_cell_pass(const void* x, int x_dtype, int64_t n_windows, const float* emb, int64_t n_cls,
                 const int64_t* cell_ptr, int64_t n_cov, const int64_t* edge_window, const int64_t* edge_class,
                 const int64_t* win_ptr, const int64_t* edge_wcell, int64_t h, float* scratch, void* out,
                 int out_dtype, void* stream) {
  MB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(out_dtype), "cell_pass: bad dtype");
  if (n_windows == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0, "cell_pass: bad width %lld", (long long)h);
  MB_REQUIRE(x && emb && cell_ptr && win_ptr && out && (n_cov == 0 || (scratch && edge_window && edge_class &&
                                                                          edge_wcell)),
             "cell_pass: null pointer");
  // the cell kernel reads x and emb and writes scratch in vec-wide vectors,
  // the window reduction reads scratch and writes out likewise
  MB_REQUIRE(aligned(x, (size_t)vec * dtype_size(x_dtype)) && aligned(emb, (size_t)vec * 4) &&
                 (n_cov == 0 || aligned(scratch, (size_t)vec * 4)) && aligned(out, (size_t)vec * dtype_size(out_dtype)),
             "cell_pass: x, emb, scratch and out must be aligned to %d elements", vec);
  cudaStream_t s = as_stream(stream);
  int st = MB_DISPATCH_T(x_dtype, TX, [&] {
    return MB_DISPATCH_VEC(vec, V, [&] {
      if (n_cov > 0)
        relay_cells_kernel<TX, V><<<row_grid(n_cov), kWarps * 32, 0, s>>>(
            (const TX*)x, n_windows, emb, n_cls, cell_ptr, n_cov, edge_window, edge_class, h, scratch);
      return launch_status("cell_pass.cells");
    });
  });
  if (st != MB_OK) return st;
  // window side: a run reduction of the cell values over the window-major view
  return mb_run_reduce(scratch, MB_F32, h, n_cov, edge_wcell, win_ptr, n_windows, h, nullptr, 0, nullptr, 0, out,
                       out_dtype, h, stream);
}

int mb_layer_norm(const void* x, int x_dtype, int64_t ldx, const int64_t* in_rows, int64_t n, int64_t h,
                  const float* gamma, const float* beta, float eps, void* out, int out_dtype, int64_t ldo,
                  void* stream) {
  MB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(out_dtype), "layer_norm: bad dtype");
  if (n == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && h <= 32 * vec * kMaxChunks, "layer_norm: unsupported width %lld", (long long)h);
  MB_REQUIRE(x && gamma && beta && out, "layer_norm: null pointer");
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(x_dtype, TX, [&] {
    MB_DISPATCH_T(out_dtype, TO, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        MB_DISPATCH_CH(row_chunks(h, vec), C, [&] {
          layer_norm_kernel<TX, TO, V, C><<<row_grid(n), kWarps * 32, 0, s>>>((const TX*)x, ldx, in_rows, n, h,
                                                                              gamma, beta, eps, (TO*)out, ldo);
        });
      });
    });
  });
  return launch_status("layer_norm");
}

int mb_add_ln(float* x, int64_t ldx, const void* y, int y_dtype, int64_t ldy, const float* y_bias, int64_t n,
              int64_t h, float eps, const float* g0, const float* b0, void* o0, int o0_dtype, int64_t ld0,
              const float* g1, const float* b1, void* o1, int o1_dtype, int64_t ld1, const float* g2,
              const float* b2, void* o2, int o2_dtype, int64_t ld2, void* stream) {
  if (n == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(x && vec > 0 && h <= 32 * vec * kMaxChunks, "add_ln: bad arguments (h=%lld)", (long long)h);
  MB_REQUIRE(!y || valid_dtype(y_dtype), "add_ln: bad y dtype");
  LnOut outs[3] = {{g0, b0, o0, o0_dtype, ld0}, {g1, b1, o1, o1_dtype, ld1}, {g2, b2, o2, o2_dtype, ld2}};
  int n_out = 0;
  for (int j = 0; j < 3; ++j) {
    if (!outs[j].out) break;
    MB_REQUIRE(outs[j].g && outs[j].b && valid_dtype(outs[j].dtype), "add_ln: output %d incomplete", j);
    n_out = j + 1;
  }
  for (int j = n_out; j < 3; ++j) MB_REQUIRE(!outs[j].out, "add_ln: outputs must be given in order");
  MB_REQUIRE(y || n_out > 0, "add_ln: nothing to do");
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(y ? y_dtype : MB_F32, TY, [&] {
    MB_DISPATCH_VEC(vec, V, [&] {
      MB_DISPATCH_CH(row_chunks(h, vec), C, [&] {
        add_ln_kernel<TY, V, C><<<row_grid(n), kWarps * 32, 0, s>>>(x, ldx, (const TY*)y, ldy, y_bias, n, h, eps,
                                                                    n_out, outs[0], outs[1], outs[2]);
      });
    });
  });
  return launch_status("add_ln");
}

int mb_embed(const float* ta, int64_t n_ta, const int64_t* ia, const float* tb, int64_t n_tb, const int64_t* ib,
             int64_t n, int64_t h, float* out, void* stream) {
  if (n == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && ta && out, "embed: bad arguments");
  MB_DISPATCH_VEC(vec, V, [&] {
    embed_kernel<V><<<row_grid(n), kWarps * 32, 0, as_stream(stream)>>>(ta, n_ta, ia, tb, n_tb, ib, n, h, out);
  });
  return launch_status("embed");
}

int mb_cell_init(const int64_t* cov_ptr, const int64_t* cell_nearest, const float* nearest_table, int64_t n_nearest,
                 const float* covered_row, const float* covered_add, int64_t n_cells, int64_t h, float* out,
                 void* stream) {
  if (n_cells == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && cov_ptr && cell_nearest && nearest_table && covered_row && out, "cell_init: bad arguments");
  MB_DISPATCH_VEC(vec, V, [&] {
    cell_init_kernel<V><<<row_grid(n_cells), kWarps * 32, 0, as_stream(stream)>>>(
        cov_ptr, cell_nearest, nearest_table, n_nearest, covered_row, covered_add, n_cells, h, out);
  });
  return launch_status("cell_init");
}

int mb_residual_add(void* x, int x_dtype, int64_t ldx, const int64_t* rows, const void* y, int y_dtype, int64_t ldy,
                    int64_t n, int64_t h, void* stream) {
  MB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(y_dtype), "residual_add: bad dtype");
  if (n == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && x && y, "residual_add: bad arguments");
  MB_DISPATCH_T(x_dtype, TX, [&] {
    MB_DISPATCH_T(y_dtype, TY, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        residual_add_kernel<TX, TY, V><<<row_grid(n), kWarps * 32, 0, as_stream(stream)>>>(
            (TX*)x, ldx, rows, (const TY*)y, ldy, n, h);
      });
    });
  });
  return launch_status("residual_add");
}

int mb_add_gather(void* x, int x_dtype, int64_t ldx, const void* t, int t_dtype, int64_t ldt, int64_t n_t,
                  const int64_t* idx, int64_t n, int64_t h, int relu, void* stream) {
  MB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(t_dtype), "add_gather: bad dtype");
  if (n == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && x && t && idx, "add_gather: bad arguments");
  MB_DISPATCH_T(x_dtype, TX, [&] {
    MB_DISPATCH_T(t_dtype, TT, [&] {
      MB_DISPATCH_VEC(vec, V, [&] {
        add_gather_kernel<TX, TT, V><<<row_grid(n), kWarps * 32, 0, as_stream(stream)>>>(
            (TX*)x, ldx, (const TT*)t, ldt, n_t, idx, n, h, relu);
      });
    });
  });
  return launch_status("add_gather");
}

int mb_tokens_gather(const float* g, const float* s, const int64_t* stone_off, const int64_t* tok_off, int64_t n_pos,
                     int64_t h, float* tok, void* stream) {
  if (n_pos == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && g && stone_off && tok_off && tok, "tokens_gather: bad arguments");
  MB_REQUIRE(n_pos <= 65535, "tokens_gather: at most 65535 positions per launch");
  MB_DISPATCH_VEC(vec, V, [&] {
    tokens_gather_kernel<V><<<dim3(4, (unsigned)n_pos), kWarps * 32, 0, as_stream(stream)>>>(g, s, stone_off, tok_off,
                                                                                             n_pos, h, tok);
  });
  return launch_status("tokens_gather");
}

int mb_tokens_scatter_add(float* g, float* s, const int64_t* stone_off, const int64_t* tok_off, int64_t n_pos,
                          int64_t h, const void* tok_out, int dtype, int update_stones, void* stream) {
  MB_REQUIRE(valid_dtype(dtype), "tokens_scatter_add: bad dtype");
  if (n_pos == 0) return MB_OK;
  const int vec = row_vec(h);
  MB_REQUIRE(vec > 0 && g && stone_off && tok_off && tok_out, "tokens_scatter_add: bad arguments");
  MB_REQUIRE(n_pos <= 65535, "tokens_scatter_add: at most 65535 positions per launch");
  MB_DISPATCH_T(dtype, TY, [&] {
    MB_DISPATCH_VEC(vec, V, [&] {
      tokens_scatter_add_kernel<TY, V><<<dim3(4, (unsigned)n_pos), kWarps * 32, 0, as_stream(stream)>>>(
          g, s, stone_off, tok_off, n_pos, h, (const TY*)tok_out, update_stones);
    });
  });
  return launch_status("tokens_scatter_add");
}

int mb_latent_mean(const float* g_ln, int64_t n_pos, int64_t h, float* out, void* stream) {
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(g_ln && out, "latent_mean: null pointer");
  latent_mean_kernel<<<(unsigned)cdiv(n_pos * h, 256), 256, 0, as_stream(stream)>>>(g_ln, n_pos, h, out);
  return launch_status("latent_mean");
}

int mb_compose_q(const float* critic, int64_t ld_critic, const int64_t* offsets, int64_t n_pos, float mass_floor,
                 float* q_score, float* q_values, void* stream) {
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(critic && offsets && q_score && q_values && ld_critic >= 3, "compose_q: bad arguments");
  compose_q_kernel<<<(unsigned)n_pos, 256, 0, as_stream(stream)>>>(critic, ld_critic, offsets, n_pos, mass_floor,
                                                                  q_score, q_values);
  return launch_status("compose_q");
}

}  // extern "C"
