// Value head (reference model.py:1160-1183, the full forward's state-value
// readout): per position p, the rows [token g[p]; the position's windows],
// each LayerNorm'd (ln_value), are read by Q learned queries with one
// attention head of the full width (scale 1 / sqrt(h), slots that
// value_valid marks invalid masked out); the Q read rows, concatenated, go
// through Linear -> ReLU -> Linear to the value logits, whose fp32 softmax
// over the bins gives value_dist and its expectation over bin_centers the
// value.
//
// One CTA per position, eight warps. A warp takes the position's rows in
// turn (lane = h / 32 columns): LayerNorm with warp reductions, the Q scores,
// and an online softmax per query with the running read row in registers;
// the warps' states merge in shared memory. The two MLP layers run from
// shared memory (one output per thread, weights read through L1/L2), the bin
// softmax by one warp. Everything in fp32.
#include <math.h>

#include "common.cuh"

namespace mb {

constexpr int kValueWarps = 8;
constexpr int kValueMaxQ = 4;

template <typename TW, int VEC>
__global__ void __launch_bounds__(kValueWarps * 32) value_head_kernel(
    const float* __restrict__ g, const TW* __restrict__ w, int64_t ldw, const int64_t* __restrict__ win_off,
    const int64_t* __restrict__ win_order, const int64_t* __restrict__ window_slot, int64_t n_windows,
    const bool* __restrict__ value_valid, int64_t max_w, const float* __restrict__ ln_g,
    const float* __restrict__ ln_b, float eps, const float* __restrict__ queries, int nq,
    const float* __restrict__ w1, const float* __restrict__ b1, int vh, const float* __restrict__ w2,
    const float* __restrict__ b2, int bins, const float* __restrict__ centers, float* __restrict__ value,
    float* __restrict__ dist, float* __restrict__ logits) {
  constexpr int H = VEC * 32;
  extern __shared__ __align__(16) float vs[];
  float* qs = vs;                                   // [nq][H] queries
  float* st = qs + kValueMaxQ * H;                  // [warps][nq][H + 2]: acc, m, l
  float* r = st + kValueWarps * kValueMaxQ * (H + 2);  // [nq * H] read rows
  float* hid = r + kValueMaxQ * H;                  // [vh]
  float* lg = hid + 256;                            // [bins]
  const int64_t p = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < nq * H; i += blockDim.x) qs[i] = queries[i];
  __syncthreads();

  float gg[VEC], bb[VEC];
  load_vec<VEC>(ln_g + lane * VEC, gg);
  load_vec<VEC>(ln_b + lane * VEC, bb);
  const float scale = rsqrtf((float)H);
  float m[kValueMaxQ], l[kValueMaxQ], acc[kValueMaxQ][VEC];
#pragma unroll
  for (int j = 0; j < kValueMaxQ; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[j][i] = 0.f;
  }
  const int64_t w0 = win_off[p], w1e = win_off[p + 1];
  const int64_t n_rows = 1 + (w1e - w0);
  for (int64_t t = warp; t < n_rows; t += kValueWarps) {
    float x[VEC];
    int64_t slot;
    if (t == 0) {
      load_vec<VEC>(g + p * H + lane * VEC, x);
      slot = 0;
    } else {
      const int64_t wi = win_order ? win_order[w0 + t - 1] : w0 + t - 1;
      if (wi < 0 || wi >= n_windows) {
        report(ERR_INDEX);
        continue;
      }
      load_vec<VEC>(w + wi * ldw + lane * VEC, x);
      slot = window_slot[wi] - p * max_w;
      if (slot < 0 || slot >= max_w) {
        report(ERR_INDEX);
        continue;
      }
    }
    if (!value_valid[p * max_w + slot]) continue;
    // LayerNorm (two-pass fp32 statistics)
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) s += x[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / H;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const float d = x[i] - mean;
      sq += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq / H + eps);
#pragma unroll
    for (int i = 0; i < VEC; ++i) x[i] = (x[i] - mean) * rstd * gg[i] + bb[i];
#pragma unroll
    for (int j = 0; j < kValueMaxQ; ++j) {
      if (j >= nq) break;
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) d += qs[j * H + lane * VEC + i] * x[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      d *= scale;
      const float m_new = fmaxf(m[j], d);
      const float corr = __expf(m[j] - m_new), pw = __expf(d - m_new);
      l[j] = l[j] * corr + pw;
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[j][i] = acc[j][i] * corr + pw * x[i];
      m[j] = m_new;
    }
  }
  // merge the warps' softmax states
#pragma unroll
  for (int j = 0; j < kValueMaxQ; ++j) {
    if (j >= nq) break;
    float* sj = st + (warp * kValueMaxQ + j) * (H + 2);
#pragma unroll
    for (int i = 0; i < VEC; ++i) sj[lane * VEC + i] = acc[j][i];
    if (lane == 0) {
      sj[H] = m[j];
      sj[H + 1] = l[j];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < nq * H; idx += blockDim.x) {
    const int j = idx / H, c = idx % H;
    float mm = -INFINITY;
    for (int v = 0; v < kValueWarps; ++v) mm = fmaxf(mm, st[(v * kValueMaxQ + j) * (H + 2) + H]);
    float ll = 0.f, aa = 0.f;
    for (int v = 0; v < kValueWarps; ++v) {
      const float* sv = st + (v * kValueMaxQ + j) * (H + 2);
      if (sv[H] == -INFINITY) continue;
      const float f = __expf(sv[H] - mm);
      ll += sv[H + 1] * f;
      aa += sv[c] * f;
    }
    r[idx] = ll > 0.f ? aa / ll : 0.f;
  }
  __syncthreads();
  // Linear(nq * H -> vh) + ReLU
  const int din = nq * H;
  for (int o = tid; o < vh; o += blockDim.x) {
    const float* wr = w1 + (int64_t)o * din;
    float a = b1[o];
    for (int i = 0; i < din; i += 4) {
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(wr + i));
      a += w4.x * r[i] + w4.y * r[i + 1] + w4.z * r[i + 2] + w4.w * r[i + 3];
    }
    hid[o] = fmaxf(a, 0.f);
  }
  __syncthreads();
  for (int o = tid; o < bins; o += blockDim.x) {
    const float* wr = w2 + (int64_t)o * vh;
    float a = b2[o];
    for (int i = 0; i < vh; ++i) a += __ldg(wr + i) * hid[i];
    lg[o] = a;
  }
  __syncthreads();
  if (warp == 0) {
    float mm = -INFINITY;
    for (int o = lane; o < bins; o += 32) mm = fmaxf(mm, lg[o]);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, s));
    float z = 0.f;
    for (int o = lane; o < bins; o += 32) z += __expf(lg[o] - mm);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) z += __shfl_xor_sync(0xffffffffu, z, s);
    float ev = 0.f;
    for (int o = lane; o < bins; o += 32) {
      const float d = __expf(lg[o] - mm) / z;
      dist[p * bins + o] = d;
      logits[p * bins + o] = lg[o];
      ev += d * centers[o];
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) ev += __shfl_xor_sync(0xffffffffu, ev, s);
    if (lane == 0) value[p] = ev;
  }
}

}  // namespace mb

using namespace mb;

extern "C" int mb_value_head(const float* g, const void* w, int w_dtype, int64_t ldw, int64_t n_windows,
                             const int64_t* win_off, const int64_t* win_order, const int64_t* window_slot,
                             const uint8_t* value_valid, int64_t n_pos, int64_t max_w, int64_t h, const float* ln_g,
                             const float* ln_b, float eps, const float* queries, int nq, const float* w1,
                             const float* b1, int vh, const float* w2, const float* b2, int bins,
                             const float* centers, float* value, float* dist, float* logits, void* stream) {
  MB_REQUIRE(valid_dtype(w_dtype), "value_head: bad dtype");
  MB_REQUIRE(n_pos >= 0 && n_windows >= 0 && max_w >= 1, "value_head: bad sizes");
  MB_REQUIRE(h == 32 || h == 64 || h == 128 || h == 256 || h == 512, "value_head: width %lld unsupported", (long long)h);
  MB_REQUIRE(nq >= 1 && nq <= kValueMaxQ, "value_head: 1 to %d queries (got %d)", kValueMaxQ, nq);
  MB_REQUIRE(vh >= 1 && vh <= 256 && bins >= 1 && bins <= 256, "value_head: hidden width <= 256 and bins <= 256");
  MB_REQUIRE((nq * h) % 4 == 0, "value_head: the readout width must be a multiple of 4");
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(g && win_off && window_slot && value_valid && ln_g && ln_b && queries && w1 && b1 && w2 && b2 &&
                 centers && value && dist && logits && (n_windows == 0 || w),
             "value_head: null pointer");
  MB_REQUIRE(aligned(w1, 16) && aligned(g, 16) && (!w || aligned(w, 16)) && ldw % 8 == 0 && aligned(ln_g, 16) &&
                 aligned(ln_b, 16),
             "value_head: rows must be 16-byte aligned");
  MB_REQUIRE(n_pos <= INT32_MAX, "value_head: too many positions");
  const size_t smem = sizeof(float) * ((size_t)kValueMaxQ * h + (size_t)kValueWarps * kValueMaxQ * (h + 2) +
                                       (size_t)kValueMaxQ * h + 256 + 256);
  cudaStream_t s = as_stream(stream);
  int rc = MB_OK;
  MB_DISPATCH_T(w_dtype, TW, [&] {
    auto go = [&](auto vec) {
      constexpr int VEC = decltype(vec)::value;
      auto kern = value_head_kernel<TW, VEC>;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        rc = fail(MB_LAUNCH_FAILED, "value_head: %zu bytes of shared memory refused", smem);
        return;
      }
      kern<<<(unsigned)n_pos, kValueWarps * 32, smem, s>>>(
          g, (const TW*)w, ldw, win_off, win_order, window_slot, n_windows, (const bool*)value_valid, max_w, ln_g,
          ln_b, eps, queries, nq, w1, b1, vh, w2, b2, bins, centers, value, dist, logits);
    };
    switch (h) {
      case 32: go(std::integral_constant<int, 1>{}); break;
      case 64: go(std::integral_constant<int, 2>{}); break;
      case 128: go(std::integral_constant<int, 4>{}); break;
      case 256: go(std::integral_constant<int, 8>{}); break;
      default: go(std::integral_constant<int, 16>{}); break;
    }
  });
  if (rc != MB_OK) return rc;
  return launch_status("value_head");
}
