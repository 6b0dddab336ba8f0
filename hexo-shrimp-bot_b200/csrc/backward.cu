// Backward kernels of the trunk's data-dependent ops, for the fit path
// (reference backward ops: attention.py:229-531 stone attention,
// cell_latents.py:287-543 typed segment attention, window_latents.py:270-473
// window-latent read / broadcast, row_encoder.py:114-207 action-row encoder).
//
// All fp32 math on f32 or bf16 inputs, fp32 gradients. Deterministic: no
// atomics; every sum runs in a fixed order. Scatters become gathers over
// stable permutations the host derives on the device (edges by source, by
// class, by window), and a class's edges, which can number millions, are
// split into a fixed set of contiguous parts summed in part order.
//
// Softmax backward, per query row i and head: with P_ij the forward
// probabilities and dP_ij = dO_i . V_j,
//   D_i = sum_j P_ij dP_ij (= dO_i . O_i),  dS_ij = P_ij (dP_ij - D_i),
//   dQ_i = scale sum_j dS_ij K_j,  dK_j = scale sum_i dS_ij Q_i,  dV_j = sum_i P_ij dO_i.
#include <math.h>

#include "common.cuh"

namespace mb {
namespace bwd {

constexpr int kClassWarps = 8;

// Sum over aligned groups of `group` lanes (a power of two up to 32).
__device__ __forceinline__ float gsum(float x, int group) {
  for (int o = group >> 1; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// ------------------------------------------------ typed segment attention
// Pass over a query row's edges (one warp per row, VEC columns per lane,
// lph lanes per head). Writes per (edge, head) alpha and dscore into the
// workspaces (the head's first lane), and dq.
template <typename T, typename TV, int VEC>
__global__ void __launch_bounds__(256) seg_bwd_rows_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ bias,
    int64_t n_cls, const TV* __restrict__ vcls, const int64_t* __restrict__ seg_ptr, const int64_t* __restrict__ src,
    const int64_t* __restrict__ cls, const float* __restrict__ m, const float* __restrict__ l,
    const float* __restrict__ go, int64_t n_q, int64_t n_src, int heads, int hd, float scale,
    float* __restrict__ alpha_ws, float* __restrict__ dscore_ws, float* __restrict__ dq) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= n_q) return;
  const int lane = threadIdx.x & 31;
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H, lead = live && lane % lph == 0;
  float qv[VEC], gv[VEC], acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) qv[i] = gv[i] = acc[i] = 0.f;
  float mh = 0.f, lh = 0.f;
  if (live) {
    load_vec<VEC>(q + row * H + col, qv);
    load_vec<VEC>(go + row * H + col, gv);
    mh = m[row * heads + head];
    lh = l[row * heads + head];
  }
  const float inv_l = lh > 0.f ? 1.f / lh : 0.f;
  const int64_t beg = seg_ptr[row], end = seg_ptr[row + 1];
  float delta = 0.f;
  for (int64_t e = beg; e < end; ++e) {
    const int64_t s = src[e], c = cls[e];
    const bool ok = s >= 0 && s < n_src && c >= 0 && c < n_cls;
    if (!ok && lane == 0) report(ERR_INDEX);
    float kv[VEC] = {}, vv[VEC] = {};
    if (ok && live) {
      load_vec<VEC>(k + s * H + col, kv);
      load_vec<VEC>(v + s * H + col, vv);
      if (vcls) {
        float a[VEC];
        load_vec<VEC>(vcls + c * H + col, a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) vv[i] += a[i];
      }
    }
    float d = 0.f, dp = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) { d += qv[i] * kv[i]; dp += gv[i] * vv[i]; }
    d = gsum(d, lph);
    dp = gsum(dp, lph);
    const float alpha = (ok && live) ? __expf(d * scale + bias[(int64_t)head * n_cls + c] - mh) * inv_l : 0.f;
    delta += alpha * dp;
    if (lead) {
      alpha_ws[e * heads + head] = alpha;
      dscore_ws[e * heads + head] = dp;
    }
  }
  __syncwarp();
  for (int64_t e = beg; e < end; ++e) {
    const int64_t s = src[e];  // warp-uniform
    const bool ok = s >= 0 && s < n_src && live;
    float ds = 0.f;
    if (ok) {
      const float alpha = alpha_ws[e * heads + head], dp = dscore_ws[e * heads + head];
      ds = alpha * (dp - delta);
      float kv[VEC];
      load_vec<VEC>(k + s * H + col, kv);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] += scale * ds * kv[i];
    }
    __syncwarp();  // every lane of the head has read dp before the head's first lane overwrites it
    if (lead) dscore_ws[e * heads + head] = ds;
  }
  if (live) store_vec<VEC>(dq + row * H + col, acc);
}

// dk, dv per source row over its edges (edge order by source, stable).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) seg_bwd_sources_kernel(
    const T* __restrict__ q, const float* __restrict__ go, const int64_t* __restrict__ qid,
    const int64_t* __restrict__ perm, const int64_t* __restrict__ ptr, int64_t n_src, int64_t n_q, int heads,
    int hd, float scale, const float* __restrict__ alpha_ws, const float* __restrict__ dscore_ws,
    float* __restrict__ dk, float* __restrict__ dv) {
  const int64_t s = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (s >= n_src) return;
  const int lane = threadIdx.x & 31;
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H;
  float ak[VEC] = {}, av[VEC] = {};
  for (int64_t i = ptr[s]; i < ptr[s + 1]; ++i) {
    const int64_t e = perm[i];
    const int64_t r = qid[e];
    if (r < 0 || r >= n_q) {
      if (lane == 0) report(ERR_INDEX);
      continue;
    }
    if (!live) continue;
    const float alpha = alpha_ws[e * heads + head], ds = dscore_ws[e * heads + head];
    float qv[VEC], gv[VEC];
    load_vec<VEC>(q + r * H + col, qv);
    load_vec<VEC>(go + r * H + col, gv);
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      ak[c] += scale * ds * qv[c];
      av[c] += alpha * gv[c];
    }
  }
  if (live) {
    store_vec<VEC>(dk + s * H + col, ak);
    store_vec<VEC>(dv + s * H + col, av);
  }
}

// dbias (heads, n_cls) and dvcls (n_cls, H) per class: a CTA per class, its
// edges (by class, stable) split in kClassWarps contiguous parts, the parts'
// sums added in part order.
template <int VEC>
__global__ void __launch_bounds__(kClassWarps * 32) seg_bwd_classes_kernel(
    const float* __restrict__ go, const int64_t* __restrict__ qid, const int64_t* __restrict__ perm,
    const int64_t* __restrict__ ptr, int64_t n_cls, int64_t n_q, int heads, int hd,
    const float* __restrict__ alpha_ws, const float* __restrict__ dscore_ws, float* __restrict__ dbias,
    float* __restrict__ dvcls) {
  __shared__ float part_b[kClassWarps][32];
  __shared__ float part_v[kClassWarps][32 * VEC];
  const int64_t c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H;
  const int64_t e0 = ptr[c], e1 = ptr[c + 1], n = e1 - e0;
  const int64_t lo = e0 + n * warp / kClassWarps, hi = e0 + n * (warp + 1) / kClassWarps;
  float sb = 0.f, sv[VEC] = {};
  for (int64_t i = lo; i < hi; ++i) {
    const int64_t e = perm[i];
    const int64_t r = qid[e];
    if (!live || r < 0 || r >= n_q) continue;
    sb += dscore_ws[e * heads + head];
    if (dvcls) {
      const float alpha = alpha_ws[e * heads + head];
      float gv[VEC];
      load_vec<VEC>(go + r * H + col, gv);
#pragma unroll
      for (int j = 0; j < VEC; ++j) sv[j] += alpha * gv[j];
    }
  }
  part_b[warp][lane] = sb;
#pragma unroll
  for (int j = 0; j < VEC; ++j) part_v[warp][lane * VEC + j] = sv[j];
  __syncthreads();
  if (warp == 0 && live) {
    float tb = 0.f, tv[VEC] = {};
    for (int w = 0; w < kClassWarps; ++w) {
      tb += part_b[w][lane];
#pragma unroll
      for (int j = 0; j < VEC; ++j) tv[j] += part_v[w][lane * VEC + j];
    }
    if (lane % lph == 0) dbias[(int64_t)head * n_cls + c] = tb;
    if (dvcls) store_vec<VEC>(dvcls + c * H + col, tv);
  }
}

// ------------------------------------------------------- stone attention
// Padded (P, A, T, D) layout, keys j < n_keys(p) live, query rows past it
// have zero gradients. lse from the forward (m + log l of the scaled scores).
constexpr int kStoneBwdThreads = 128;
constexpr int kStoneTile = 64;

template <typename T, int D>
__global__ void __launch_bounds__(kStoneBwdThreads) stone_bwd_dq_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ out,
    const T* __restrict__ go, int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* __restrict__ seq_lens,
    int64_t t_pad, int heads, const float* __restrict__ lse, float scale, float* __restrict__ dq,
    float* __restrict__ dsum) {
  __shared__ float ks[kStoneTile][D];
  __shared__ float vs[kStoneTile][D];
  const int64_t p = blockIdx.y;
  const int a = blockIdx.z;
  int64_t nk = seq_lens[p];
  if (nk > t_pad) nk = t_pad;
  const int64_t base = p * s_pos + a * s_head;
  const int64_t obase = ((p * heads) + a) * t_pad * D;  // dq is (P, A, T, D) contiguous fp32
  const int64_t i = (int64_t)blockIdx.x * kStoneBwdThreads + threadIdx.x;
  const bool active = i < nk;
  float qv[D], gv[D], acc[D];
  float Di = 0.f, li = 0.f;
#pragma unroll
  for (int c = 0; c < D; ++c) qv[c] = gv[c] = acc[c] = 0.f;
  if (active) {
    load_vec<D>(q + base + i * s_row, qv);
    load_vec<D>(go + base + i * s_row, gv);
    float ov[D];
    load_vec<D>(out + base + i * s_row, ov);
#pragma unroll
    for (int c = 0; c < D; ++c) Di += gv[c] * ov[c];
    li = lse[(p * heads + a) * t_pad + i];
  }
  for (int64_t j0 = 0; j0 < nk; j0 += kStoneTile) {
    const int n = (int)min((int64_t)kStoneTile, nk - j0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < n * D; idx += kStoneBwdThreads) {
      const int r = idx / D, c = idx % D;
      ks[r][c] = to_f(k[base + (j0 + r) * s_row + c]);
      vs[r][c] = to_f(v[base + (j0 + r) * s_row + c]);
    }
    __syncthreads();
    if (active) {
      for (int j = 0; j < n; ++j) {
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int c = 0; c < D; ++c) { s += qv[c] * ks[j][c]; dp += gv[c] * vs[j][c]; }
        const float pr = __expf(s * scale - li);
        const float ds = pr * (dp - Di);
#pragma unroll
        for (int c = 0; c < D; ++c) acc[c] += scale * ds * ks[j][c];
      }
    }
  }
  if (i < t_pad) {
    store_vec<D>(dq + obase + i * D, acc);
    dsum[(p * heads + a) * t_pad + i] = active ? Di : 0.f;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kStoneBwdThreads) stone_bwd_dkdv_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ go,
    int64_t s_pos, int64_t s_head, int64_t s_row, const int32_t* __restrict__ seq_lens, int64_t t_pad, int heads,
    const float* __restrict__ lse, const float* __restrict__ dsum, float scale, float* __restrict__ dk,
    float* __restrict__ dv) {
  __shared__ float qs[kStoneTile][D];
  __shared__ float gs[kStoneTile][D];
  __shared__ float ls[kStoneTile], dls[kStoneTile];
  const int64_t p = blockIdx.y;
  const int a = blockIdx.z;
  int64_t nk = seq_lens[p];
  if (nk > t_pad) nk = t_pad;
  const int64_t base = p * s_pos + a * s_head;
  const int64_t obase = ((p * heads) + a) * t_pad * D;
  const int64_t j = (int64_t)blockIdx.x * kStoneBwdThreads + threadIdx.x;
  const bool active = j < nk;
  float kv[D], vv[D], ak[D], av[D];
#pragma unroll
  for (int c = 0; c < D; ++c) kv[c] = vv[c] = ak[c] = av[c] = 0.f;
  if (active) {
    load_vec<D>(k + base + j * s_row, kv);
    load_vec<D>(v + base + j * s_row, vv);
  }
  for (int64_t i0 = 0; i0 < nk; i0 += kStoneTile) {  // live query rows are i < n_keys
    const int n = (int)min((int64_t)kStoneTile, nk - i0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < n * D; idx += kStoneBwdThreads) {
      const int r = idx / D, c = idx % D;
      qs[r][c] = to_f(q[base + (i0 + r) * s_row + c]);
      gs[r][c] = to_f(go[base + (i0 + r) * s_row + c]);
    }
    for (int r = threadIdx.x; r < n; r += kStoneBwdThreads) {
      ls[r] = lse[(p * heads + a) * t_pad + i0 + r];
      dls[r] = dsum[(p * heads + a) * t_pad + i0 + r];
    }
    __syncthreads();
    if (active) {
      for (int i = 0; i < n; ++i) {
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int c = 0; c < D; ++c) { s += qs[i][c] * kv[c]; dp += gs[i][c] * vv[c]; }
        const float pr = __expf(s * scale - ls[i]);
        const float ds = pr * (dp - dls[i]);
#pragma unroll
        for (int c = 0; c < D; ++c) {
          av[c] += pr * gs[i][c];
          ak[c] += scale * ds * qs[i][c];
        }
      }
    }
  }
  if (j < t_pad) {
    store_vec<D>(dk + obase + j * D, ak);
    store_vec<D>(dv + obase + j * D, av);
  }
}

// ------------------------------------------------------- window latents
// Read: four latent queries per position over its windows. Per window: its
// dk, dv from the position's four queries. Per position and query: dq over
// its windows (in the layout's order).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) read_bwd_windows_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ out,
    const float* __restrict__ m, const float* __restrict__ l, const float* __restrict__ go,
    const int64_t* __restrict__ window_pos, int64_t n_windows, int64_t n_pos, int heads, int hd, float scale,
    float* __restrict__ dk, float* __restrict__ dv) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= n_windows) return;
  const int lane = threadIdx.x & 31;
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H;
  const int64_t p = window_pos[w];
  float ak[VEC] = {}, av[VEC] = {};
  if (p < 0 || p >= n_pos) {
    if (lane == 0) report(ERR_INDEX);
  } else if (live) {
    float kv[VEC], vv[VEC];
    load_vec<VEC>(k + w * H + col, kv);
    load_vec<VEC>(v + w * H + col, vv);
    for (int i = 0; i < 4; ++i) {
      const int64_t r = p * 4 + i;
      float qv[VEC], gv[VEC], ov[VEC];
      load_vec<VEC>(q + r * H + col, qv);
      load_vec<VEC>(go + r * H + col, gv);
      load_vec<VEC>(out + r * H + col, ov);
      float s = 0.f, dp = 0.f, dd = 0.f;
#pragma unroll
      for (int c = 0; c < VEC; ++c) { s += qv[c] * kv[c]; dp += gv[c] * vv[c]; dd += gv[c] * ov[c]; }
      s = gsum(s, lph);
      dp = gsum(dp, lph);
      dd = gsum(dd, lph);
      const float lh = l[r * heads + head];
      const float pr = lh > 0.f ? __expf(s * scale - m[r * heads + head]) / lh : 0.f;
      const float ds = pr * (dp - dd);
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        ak[c] += scale * ds * qv[c];
        av[c] += pr * gv[c];
      }
    }
  }
  if (live) {
    store_vec<VEC>(dk + w * H + col, ak);
    store_vec<VEC>(dv + w * H + col, av);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(128) read_bwd_queries_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ out,
    const float* __restrict__ m, const float* __restrict__ l, const float* __restrict__ go,
    const int64_t* __restrict__ offsets, const int64_t* __restrict__ order, int64_t n_windows, int heads, int hd,
    float scale, float* __restrict__ dq) {
  const int64_t p = blockIdx.x;
  const int i = threadIdx.x >> 5, lane = threadIdx.x & 31;  // warp = latent query
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H;
  const int64_t r = p * 4 + i;
  float qv[VEC] = {}, gv[VEC] = {}, acc[VEC] = {};
  float dd = 0.f, mh = 0.f, lh = 0.f;
  if (live) {
    float ov[VEC];
    load_vec<VEC>(q + r * H + col, qv);
    load_vec<VEC>(go + r * H + col, gv);
    load_vec<VEC>(out + r * H + col, ov);
#pragma unroll
    for (int c = 0; c < VEC; ++c) dd += gv[c] * ov[c];
    mh = m[r * heads + head];
    lh = l[r * heads + head];
  }
  dd = gsum(dd, lph);
  const float inv_l = lh > 0.f ? 1.f / lh : 0.f;
  for (int64_t t = offsets[p]; t < offsets[p + 1]; ++t) {
    const int64_t w = order ? order[t] : t;
    if (w < 0 || w >= n_windows) {
      if (lane == 0) report(ERR_INDEX);
      continue;
    }
    float kv[VEC] = {}, vv[VEC] = {};
    if (live) {
      load_vec<VEC>(k + w * H + col, kv);
      load_vec<VEC>(v + w * H + col, vv);
    }
    float s = 0.f, dp = 0.f;
#pragma unroll
    for (int c = 0; c < VEC; ++c) { s += qv[c] * kv[c]; dp += gv[c] * vv[c]; }
    s = gsum(s, lph);
    dp = gsum(dp, lph);
    const float pr = __expf(s * scale - mh) * inv_l;
    const float ds = pr * (dp - dd);
#pragma unroll
    for (int c = 0; c < VEC; ++c) acc[c] += scale * ds * kv[c];
  }
  if (live) store_vec<VEC>(dq + r * H + col, acc);
}

// Broadcast: each window's query over its position's four latent keys. Per
// window: dq, and its per-(latent, head) P and dS into the workspaces. Per
// position and latent: dk, dv over the position's windows.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) bcast_bwd_windows_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ m,
    const float* __restrict__ l, const float* __restrict__ go, const int64_t* __restrict__ window_pos,
    int64_t n_windows, int64_t n_pos, int heads, int hd, float scale, float* __restrict__ dq,
    float* __restrict__ p_ws, float* __restrict__ ds_ws) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= n_windows) return;
  const int lane = threadIdx.x & 31;
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H, lead = live && lane % lph == 0;
  const int64_t p = window_pos[w];
  float acc[VEC] = {};
  if (p < 0 || p >= n_pos) {
    if (lane == 0) report(ERR_INDEX);
  } else if (live) {
    float qv[VEC], gv[VEC];
    load_vec<VEC>(q + w * H + col, qv);
    load_vec<VEC>(go + w * H + col, gv);
    const float mh = m[w * heads + head], lh = l[w * heads + head];
    const float inv_l = lh > 0.f ? 1.f / lh : 0.f;
    float pr[4], dp[4], kk[4][VEC];
    float dd = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float vv[VEC];
      load_vec<VEC>(k + (p * 4 + j) * H + col, kk[j]);
      load_vec<VEC>(v + (p * 4 + j) * H + col, vv);
      float s = 0.f, d = 0.f;
#pragma unroll
      for (int c = 0; c < VEC; ++c) { s += qv[c] * kk[j][c]; d += gv[c] * vv[c]; }
      s = gsum(s, lph);
      dp[j] = gsum(d, lph);
      pr[j] = __expf(s * scale - mh) * inv_l;
      dd += pr[j] * dp[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float ds = pr[j] * (dp[j] - dd);
#pragma unroll
      for (int c = 0; c < VEC; ++c) acc[c] += scale * ds * kk[j][c];
      if (lead) {
        p_ws[(w * 4 + j) * heads + head] = pr[j];
        ds_ws[(w * 4 + j) * heads + head] = ds;
      }
    }
  }
  if (live) store_vec<VEC>(dq + w * H + col, acc);
}

template <typename T, int VEC>
__global__ void __launch_bounds__(128) bcast_bwd_latents_kernel(
    const T* __restrict__ q, const float* __restrict__ go, const int64_t* __restrict__ offsets,
    const int64_t* __restrict__ order, int64_t n_windows, int heads, int hd, float scale,
    const float* __restrict__ p_ws, const float* __restrict__ ds_ws, float* __restrict__ dk,
    float* __restrict__ dv) {
  const int64_t p = blockIdx.x;
  const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;  // warp = latent key
  const int H = heads * hd, lph = hd / VEC, head = lane / lph, col = lane * VEC;
  const bool live = col < H;
  float ak[VEC] = {}, av[VEC] = {};
  for (int64_t t = offsets[p]; t < offsets[p + 1]; ++t) {
    const int64_t w = order ? order[t] : t;
    if (w < 0 || w >= n_windows) {
      if (lane == 0) report(ERR_INDEX);
      continue;
    }
    if (!live) continue;
    const float pr = p_ws[(w * 4 + j) * heads + head], ds = ds_ws[(w * 4 + j) * heads + head];
    float qv[VEC], gv[VEC];
    load_vec<VEC>(q + w * H + col, qv);
    load_vec<VEC>(go + w * H + col, gv);
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      ak[c] += scale * ds * qv[c];
      av[c] += pr * gv[c];
    }
  }
  if (live) {
    store_vec<VEC>(dk + (p * 4 + j) * H + col, ak);
    store_vec<VEC>(dv + (p * 4 + j) * H + col, av);
  }
}

// ------------------------------------------------------- action rows
// out[c] = sum_{e: cell e = c} relu(pre[win e] + table[cls e]). Gradients of
// pre per window (edges by window) and of table per class (edges by class,
// in kClassWarps parts): go[cell] where the pre-activation is positive.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) rows_bwd_pre_kernel(
    const T* __restrict__ pre, const float* __restrict__ table, const float* __restrict__ go,
    const int64_t* __restrict__ edge_class, const int64_t* __restrict__ edge_cell, const int64_t* __restrict__ perm,
    const int64_t* __restrict__ ptr, int64_t n_pre, int64_t n_table, int64_t n_cells, int h,
    float* __restrict__ grad) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= n_pre) return;
  const int lane = threadIdx.x & 31, col = lane * VEC;
  const bool live = col < h;
  float acc[VEC] = {}, pv[VEC] = {};
  if (live) load_vec<VEC>(pre + w * h + col, pv);
  for (int64_t i = ptr[w]; i < ptr[w + 1]; ++i) {
    const int64_t e = perm[i];
    const int64_t c = edge_class[e], cell = edge_cell[e];
    if (c < 0 || c >= n_table || cell < 0 || cell >= n_cells) {
      if (lane == 0) report(ERR_INDEX);
      continue;
    }
    if (!live) continue;
    float tv[VEC], gv[VEC];
    load_vec<VEC>(table + c * h + col, tv);
    load_vec<VEC>(go + cell * h + col, gv);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] += (pv[j] + tv[j] > 0.f) ? gv[j] : 0.f;
  }
  if (live) store_vec<VEC>(grad + w * h + col, acc);
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kClassWarps * 32) rows_bwd_table_kernel(
    const T* __restrict__ pre, const float* __restrict__ table, const float* __restrict__ go,
    const int64_t* __restrict__ edge_window, const int64_t* __restrict__ edge_cell, const int64_t* __restrict__ perm,
    const int64_t* __restrict__ ptr, int64_t n_pre, int64_t n_cells, int h, float* __restrict__ grad) {
  __shared__ float part[kClassWarps][32 * VEC];
  const int64_t c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, col = lane * VEC;
  const bool live = col < h;
  const int64_t e0 = ptr[c], e1 = ptr[c + 1], n = e1 - e0;
  const int64_t lo = e0 + n * warp / kClassWarps, hi = e0 + n * (warp + 1) / kClassWarps;
  float acc[VEC] = {}, tv[VEC] = {};
  if (live) load_vec<VEC>(table + c * h + col, tv);
  for (int64_t i = lo; i < hi; ++i) {
    const int64_t e = perm[i];
    const int64_t w = edge_window[e], cell = edge_cell[e];
    if (w < 0 || w >= n_pre || cell < 0 || cell >= n_cells || !live) continue;
    float pv[VEC], gv[VEC];
    load_vec<VEC>(pre + w * h + col, pv);
    load_vec<VEC>(go + cell * h + col, gv);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] += (pv[j] + tv[j] > 0.f) ? gv[j] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) part[warp][lane * VEC + j] = acc[j];
  __syncthreads();
  if (warp == 0 && live) {
    float t[VEC] = {};
    for (int p = 0; p < kClassWarps; ++p)
#pragma unroll
      for (int j = 0; j < VEC; ++j) t[j] += part[p][lane * VEC + j];
    store_vec<VEC>(grad + c * h + col, t);
  }
}

template <typename F>
int dispatch_vec(int64_t width, F&& f) {
  switch (width) {
    case 32: f(std::integral_constant<int, 1>{}); return MB_OK;
    case 64: f(std::integral_constant<int, 2>{}); return MB_OK;
    case 128: f(std::integral_constant<int, 4>{}); return MB_OK;
    case 256: f(std::integral_constant<int, 8>{}); return MB_OK;
    default: return fail(MB_UNSUPPORTED, "backward: width %lld unsupported (32, 64, 128 or 256)", (long long)width);
  }
}

}  // namespace bwd
}  // namespace mb

using namespace mb;

extern "C" {

int mb_segment_attention_backward(const void* q, const void* k, const void* v, int dtype, int64_t n_q, int64_t n_src,
                                  int heads, int head_dim, const float* bias, int64_t n_cls, const void* vcls,
                                  int vcls_dtype, const int64_t* seg_ptr, const int64_t* src, const int64_t* cls,
                                  const int64_t* qid, const float* m, const float* l, const float* grad_out,
                                  int64_t n_edges, const int64_t* src_perm, const int64_t* src_ptr,
                                  const int64_t* cls_perm, const int64_t* cls_ptr, float* alpha_ws, float* dscore_ws,
                                  float* dq, float* dk, float* dv, float* dbias, float* dvcls, void* stream) {
  MB_REQUIRE(valid_dtype(dtype) && valid_dtype(vcls_dtype), "segment_attention_backward: bad dtype");
  MB_REQUIRE(heads > 0 && head_dim > 0 && n_q >= 0 && n_src >= 0 && n_cls > 0 && n_edges >= 0,
             "segment_attention_backward: bad sizes");
  const int64_t H = (int64_t)heads * head_dim;
  MB_REQUIRE(H % 32 == 0 && H <= 256 && head_dim % (H / 32) == 0 && (head_dim / (H / 32)) <= 32,
             "segment_attention_backward: width %lld unsupported", (long long)H);
  MB_REQUIRE(q && k && v && bias && seg_ptr && src && cls && qid && m && l && grad_out && src_perm && src_ptr &&
                 cls_perm && cls_ptr && alpha_ws && dscore_ws && dq && dk && dv && dbias && (!vcls || dvcls),
             "segment_attention_backward: null pointer");
  cudaStream_t s = as_stream(stream);
  const float scale = 1.f / sqrtf((float)head_dim);
  int rc = MB_OK;
  MB_DISPATCH_T(dtype, T, [&] {
    MB_DISPATCH_T(vcls_dtype, TV, [&] {
      rc = bwd::dispatch_vec(H, [&](auto vec) {
        constexpr int VEC = decltype(vec)::value;
        if (n_q > 0)
          bwd::seg_bwd_rows_kernel<T, TV, VEC><<<(unsigned)cdiv(n_q, 8), 256, 0, s>>>(
              (const T*)q, (const T*)k, (const T*)v, bias, n_cls, (const TV*)vcls, seg_ptr, src, cls, m, l, grad_out,
              n_q, n_src, heads, head_dim, scale, alpha_ws, dscore_ws, dq);
        if (n_src > 0)
          bwd::seg_bwd_sources_kernel<T, VEC><<<(unsigned)cdiv(n_src, 8), 256, 0, s>>>(
              (const T*)q, grad_out, qid, src_perm, src_ptr, n_src, n_q, heads, head_dim, scale, alpha_ws, dscore_ws,
              dk, dv);
        bwd::seg_bwd_classes_kernel<VEC><<<(unsigned)n_cls, bwd::kClassWarps * 32, 0, s>>>(
            grad_out, qid, cls_perm, cls_ptr, n_cls, n_q, heads, head_dim, alpha_ws, dscore_ws, dbias,
            vcls ? dvcls : nullptr);
      });
    });
  });
  if (rc != MB_OK) return rc;
  return launch_status("segment_attention_backward");
}

int mb_stone_attention_backward(const void* q, const void* k, const void* v, const void* out, const void* grad_out,
                                int dtype, int64_t n_pos, int heads, int head_dim, int64_t s_pos, int64_t s_head,
                                int64_t s_row, const int32_t* seq_lens, int64_t t_pad, const float* lse,
                                float* dsum_ws, float* dq, float* dk, float* dv, void* stream) {
  MB_REQUIRE(valid_dtype(dtype), "stone_attention_backward: bad dtype");
  MB_REQUIRE(head_dim == 16 || head_dim == 32 || head_dim == 64, "stone_attention_backward: head_dim %d unsupported",
             head_dim);
  if (n_pos == 0 || t_pad == 0) return MB_OK;
  MB_REQUIRE(q && k && v && out && grad_out && seq_lens && lse && dsum_ws && dq && dk && dv,
             "stone_attention_backward: null pointer");
  MB_REQUIRE(n_pos <= 65535 && heads <= 65535, "stone_attention_backward: grid too large");
  dim3 grid((unsigned)cdiv(t_pad, bwd::kStoneBwdThreads), (unsigned)n_pos, (unsigned)heads);
  const float scale = 1.f / sqrtf((float)head_dim);
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_T(dtype, T, [&] {
    auto go = [&](auto dtag) {
      constexpr int D = decltype(dtag)::value;
      bwd::stone_bwd_dq_kernel<T, D><<<grid, bwd::kStoneBwdThreads, 0, s>>>(
          (const T*)q, (const T*)k, (const T*)v, (const T*)out, (const T*)grad_out, s_pos, s_head, s_row, seq_lens,
          t_pad, heads, lse, scale, dq, dsum_ws);
      bwd::stone_bwd_dkdv_kernel<T, D><<<grid, bwd::kStoneBwdThreads, 0, s>>>(
          (const T*)q, (const T*)k, (const T*)v, (const T*)grad_out, s_pos, s_head, s_row, seq_lens, t_pad, heads,
          lse, dsum_ws, scale, dk, dv);
    };
    if (head_dim == 16) go(std::integral_constant<int, 16>{});
    else if (head_dim == 32) go(std::integral_constant<int, 32>{});
    else go(std::integral_constant<int, 64>{});
  });
  return launch_status("stone_attention_backward");
}

int mb_window_latent_read_backward(const void* q, const void* k, const void* v, int dtype, const float* out,
                                   const float* m, const float* l, const float* grad_out, const int64_t* window_pos,
                                   const int64_t* offsets, const int64_t* order, int64_t n_pos, int64_t n_windows,
                                   int heads, int head_dim, float* dq, float* dk, float* dv, void* stream) {
  MB_REQUIRE(valid_dtype(dtype), "window_latent_read_backward: bad dtype");
  MB_REQUIRE(heads > 0 && head_dim > 0 && n_pos >= 0 && n_windows >= 0, "window_latent_read_backward: bad sizes");
  MB_REQUIRE(q && out && m && l && grad_out && offsets && dq && (n_windows == 0 || (k && v && window_pos && dk && dv)),
             "window_latent_read_backward: null pointer");
  const int64_t H = (int64_t)heads * head_dim;
  cudaStream_t s = as_stream(stream);
  const float scale = 1.f / sqrtf((float)head_dim);
  int rc = MB_OK;
  MB_DISPATCH_T(dtype, T, [&] {
    rc = bwd::dispatch_vec(H, [&](auto vec) {
      constexpr int VEC = decltype(vec)::value;
      if (n_windows > 0)
        bwd::read_bwd_windows_kernel<T, VEC><<<(unsigned)cdiv(n_windows, 8), 256, 0, s>>>(
            (const T*)q, (const T*)k, (const T*)v, out, m, l, grad_out, window_pos, n_windows, n_pos, heads,
            head_dim, scale, dk, dv);
      if (n_pos > 0)
        bwd::read_bwd_queries_kernel<T, VEC><<<(unsigned)n_pos, 128, 0, s>>>(
            (const T*)q, (const T*)k, (const T*)v, out, m, l, grad_out, offsets, order, n_windows, heads, head_dim,
            scale, dq);
    });
  });
  if (rc != MB_OK) return rc;
  return launch_status("window_latent_read_backward");
}

int mb_window_latent_broadcast_backward(const void* q, const void* k, const void* v, int dtype, const float* m,
                                        const float* l, const float* grad_out, const int64_t* window_pos,
                                        const int64_t* offsets, const int64_t* order, int64_t n_pos,
                                        int64_t n_windows, int heads, int head_dim, float* p_ws, float* ds_ws,
                                        float* dq, float* dk, float* dv, void* stream) {
  MB_REQUIRE(valid_dtype(dtype), "window_latent_broadcast_backward: bad dtype");
  MB_REQUIRE(heads > 0 && head_dim > 0 && n_pos >= 0 && n_windows >= 0,
             "window_latent_broadcast_backward: bad sizes");
  MB_REQUIRE(k && v && offsets && dk && dv && (n_windows == 0 || (q && m && l && grad_out && window_pos && p_ws &&
                                                                  ds_ws && dq)),
             "window_latent_broadcast_backward: null pointer");
  const int64_t H = (int64_t)heads * head_dim;
  cudaStream_t s = as_stream(stream);
  const float scale = 1.f / sqrtf((float)head_dim);
  int rc = MB_OK;
  MB_DISPATCH_T(dtype, T, [&] {
    rc = bwd::dispatch_vec(H, [&](auto vec) {
      constexpr int VEC = decltype(vec)::value;
      if (n_windows > 0)
        bwd::bcast_bwd_windows_kernel<T, VEC><<<(unsigned)cdiv(n_windows, 8), 256, 0, s>>>(
            (const T*)q, (const T*)k, (const T*)v, m, l, grad_out, window_pos, n_windows, n_pos, heads, head_dim,
            scale, dq, p_ws, ds_ws);
      if (n_pos > 0)
        bwd::bcast_bwd_latents_kernel<T, VEC><<<(unsigned)n_pos, 128, 0, s>>>(
            (const T*)q, grad_out, offsets, order, n_windows, heads, head_dim, scale, p_ws, ds_ws, dk, dv);
    });
  });
  if (rc != MB_OK) return rc;
  return launch_status("window_latent_broadcast_backward");
}

int mb_row_encode_backward(const void* pre, int pre_dtype, int64_t n_pre, const float* table, int64_t n_table,
                           const int64_t* edge_window, const int64_t* edge_class, const int64_t* edge_cell,
                           int64_t n_edges, const float* grad_out, int64_t n_cells, int64_t h,
                           const int64_t* win_perm, const int64_t* win_ptr, const int64_t* cls_perm,
                           const int64_t* cls_ptr, float* grad_pre, float* grad_table, void* stream) {
  MB_REQUIRE(valid_dtype(pre_dtype), "row_encode_backward: bad dtype");
  MB_REQUIRE(n_pre >= 0 && n_table >= 0 && n_edges >= 0 && n_cells >= 0, "row_encode_backward: bad sizes");
  MB_REQUIRE((n_edges == 0 || (pre && table && edge_window && edge_class && edge_cell && grad_out && win_perm &&
                               win_ptr && cls_perm && cls_ptr)) &&
                 grad_pre && grad_table,
             "row_encode_backward: null pointer");
  cudaStream_t s = as_stream(stream);
  int rc = MB_OK;
  MB_DISPATCH_T(pre_dtype, T, [&] {
    rc = bwd::dispatch_vec(h, [&](auto vec) {
      constexpr int VEC = decltype(vec)::value;
      if (n_pre > 0)
        bwd::rows_bwd_pre_kernel<T, VEC><<<(unsigned)cdiv(n_pre, 8), 256, 0, s>>>(
            (const T*)pre, table, grad_out, edge_class, edge_cell, win_perm, win_ptr, n_pre, n_table, n_cells, (int)h,
            grad_pre);
      if (n_table > 0)
        bwd::rows_bwd_table_kernel<T, VEC><<<(unsigned)n_table, bwd::kClassWarps * 32, 0, s>>>(
            (const T*)pre, table, grad_out, edge_window, edge_cell, cls_perm, cls_ptr, n_pre, n_cells, (int)h,
            grad_table);
    });
  });
  if (rc != MB_OK) return rc;
  return launch_status("row_encode_backward");
}

}  // extern "C"
