// KLENT policy improvement and the self-play move draw, on the device.
//
// Per position (one CTA per segment of legal cells):
//   log pi  = log-softmax(policy logits)
//   pi'     = softmax((q_score + tau log pi) / (tau + lam))
//   v_hat   = sum pi' q / sum pi'
//   kl      = sum pi' (log pi' - log pi) / sum pi'
//   entropy = sum -pi' log pi' / sum pi', normalised by log |A| (0 if |A| = 1)
// as python/mantisnet/mantisnet/klent/improve.py:27-69 defines them, and, when
// uniforms are given, the draw of python/mantisnet/mantisnet/klent/selfplay.py:180-190:
// pi' renormalised per position in float64, the rank of the first cell whose
// cumulative probability reaches the position's uniform (clipped to the
// segment), the stored float32 policy, the largest probability and the chosen
// one. The evaluator's outputs stay on the device, so the host receives one
// rank per position instead of three floats per legal cell.
//
// The element-wise terms are float32 as in the reference; the segment sums
// accumulate in float64. The draw's cumulative sums are per position (the
// reference accumulates over the whole batch), so a rank can differ from the
// reference's only when the uniform lies within float64 rounding of a
// cumulative boundary.
#include "common.cuh"

namespace mb {
namespace klent {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Block-wide reductions (every thread gets the result). `scratch` holds
// kWarps entries of the type; a barrier separates successive uses.
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  T r = scratch[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) r = op(r, scratch[w]);
  return r;
}

__global__ void __launch_bounds__(kThreads) improve_kernel(
    const float* __restrict__ logits, const float* __restrict__ score, const float* __restrict__ qv,
    const int64_t* __restrict__ offsets, int64_t n_pos, int64_t n, float tau, float lam, float* __restrict__ probs,
    float* __restrict__ v_hat, float* __restrict__ kl, float* __restrict__ norm_entropy,
    const double* __restrict__ uniforms, float* __restrict__ stored, int64_t* __restrict__ ranks,
    double* __restrict__ pi_top1, double* __restrict__ pi_chosen) {
  __shared__ float fs[kWarps];
  __shared__ double ds[kWarps];
  __shared__ long long rank_s;
  const int64_t p = blockIdx.x;
  const int64_t a = offsets[p], b = offsets[p + 1];
  if (a < 0 || b < a || b > n) {
    if (threadIdx.x == 0) report(ERR_RUN_BOUND);
    return;
  }
  const int64_t m = b - a;
  auto fmax_op = [](float x, float y) { return fmaxf(x, y); };
  auto dsum = [](double x, double y) { return x + y; };
  auto dmax = [](double x, double y) { return x > y ? x : y; };

  // log pi
  float mx = -INFINITY;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) mx = fmaxf(mx, logits[i]);
  mx = block_reduce(mx, fmax_op, fs);
  double s = 0.0;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) s += (double)expf(logits[i] - mx);
  const float lse1 = (float)log(block_reduce(s, dsum, ds));
  const float inv = 1.f / (tau + lam);
  auto log_pi = [&](int64_t i) { return (logits[i] - mx) - lse1; };
  auto zval = [&](int64_t i) { return (score[i] + tau * log_pi(i)) * inv; };

  // log pi'
  float mz = -INFINITY;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) mz = fmaxf(mz, zval(i));
  mz = block_reduce(mz, fmax_op, fs);
  s = 0.0;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) s += (double)expf(zval(i) - mz);
  const float lse2 = (float)log(block_reduce(s, dsum, ds));

  // pi' and its weighted means
  double mass = 0.0, sq = 0.0, skl = 0.0, sent = 0.0;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) {
    const float li = zval(i) - mz - lse2;
    const float pr = expf(li);
    probs[i] = pr;
    mass += pr;
    sq += (double)pr * qv[i];
    skl += (double)pr * (double)(li - log_pi(i));
    sent -= (double)pr * li;
  }
  mass = block_reduce(mass, dsum, ds);
  sq = block_reduce(sq, dsum, ds);
  skl = block_reduce(skl, dsum, ds);
  sent = block_reduce(sent, dsum, ds);
  if (threadIdx.x == 0) {
    v_hat[p] = (float)(sq / mass);
    kl[p] = (float)(skl / mass);
    const double ent = sent / mass;
    norm_entropy[p] = m > 1 ? (float)(ent / log((double)m)) : 0.f;
  }
  if (!uniforms) return;

  // The draw: float64 renormalisation of the float32 pi' (as stored), then the
  // first cell whose cumulative probability reaches the uniform. Each thread
  // owns a contiguous run of the segment, so the cumulative sum is a scan of
  // the run sums followed by one sequential walk inside the crossing run.
  __syncthreads();  // this block's probs writes are visible to its own reads
  double ps = 0.0;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) ps += (double)probs[i];
  const double total = block_reduce(ps, dsum, ds);
  const int64_t run = (m + kThreads - 1) / kThreads;
  const int64_t r0 = a + threadIdx.x * run, r1 = min(b, r0 + run);
  double own = 0.0, top = 0.0;
  for (int64_t i = r0; i < r1; ++i) {
    const double f = (double)probs[i] / total;
    own += f;
    top = fmax(top, f);
  }
  top = block_reduce(top, dmax, ds);
  // exclusive scan of the run sums, in thread order
  __shared__ double runs[kThreads];
  runs[threadIdx.x] = own;
  if (threadIdx.x == 0) rank_s = (long long)m - 1;
  __syncthreads();
  double before = 0.0;
  for (int t = 0; t < (int)threadIdx.x; ++t) before += runs[t];
  const double u = uniforms[p];
  if (r0 < r1 && before + own >= u) {
    double c = before;
    for (int64_t i = r0; i < r1; ++i) {
      c += (double)probs[i] / total;
      if (c >= u) {
        atomicMin(&rank_s, (long long)(i - a));
        break;
      }
    }
  }
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) stored[i] = (float)((double)probs[i] / total);
  __syncthreads();
  if (threadIdx.x == 0) {
    const int64_t r = m > 0 ? (int64_t)max(0LL, rank_s) : -1;
    ranks[p] = r;
    pi_top1[p] = top;
    pi_chosen[p] = m > 0 ? (double)probs[a + r] / total : 0.0;
  }
}

// Per segment, the rank of its largest value (the first one on ties), as
// torch.argmax over the segment; -1 for an empty segment.
__global__ void __launch_bounds__(kThreads) segment_argmax_kernel(const float* __restrict__ x,
                                                                  const int64_t* __restrict__ offsets, int64_t n_pos,
                                                                  int64_t n, int64_t* __restrict__ ranks) {
  __shared__ float vs[kWarps];
  __shared__ long long is[kWarps];
  const int64_t p = blockIdx.x;
  const int64_t a = offsets[p], b = offsets[p + 1];
  if (a < 0 || b < a || b > n) {
    if (threadIdx.x == 0) {
      report(ERR_RUN_BOUND);
      ranks[p] = -1;
    }
    return;
  }
  float best = -INFINITY;
  long long at = -1;
  for (int64_t i = a + threadIdx.x; i < b; i += kThreads) {
    const float v = x[i];
    if (at < 0 || v > best) {  // strided: the first index wins ties within a thread
      best = v;
      at = i - a;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const long long oi = __shfl_xor_sync(0xffffffffu, at, o);
    if (oi >= 0 && (at < 0 || ov > best || (ov == best && oi < at))) {
      best = ov;
      at = oi;
    }
  }
  if (lane == 0) {
    vs[warp] = best;
    is[warp] = at;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kWarps; ++w)
      if (is[w] >= 0 && (at < 0 || vs[w] > best || (vs[w] == best && is[w] < at))) {
        best = vs[w];
        at = is[w];
      }
    ranks[p] = at;
  }
}

}  // namespace klent
}  // namespace mb

extern "C" {

int mb_klent_improve(const float* policy_logits, const float* q_score, const float* q_values, const int64_t* offsets,
                     int64_t n_pos, int64_t n, float tau, float lam, float* probs, float* v_hat, float* kl,
                     float* norm_entropy, const double* uniforms, float* stored, int64_t* ranks, double* pi_top1,
                     double* pi_chosen, void* stream) {
  MB_REQUIRE(tau >= 0.f && lam >= 0.f && tau + lam > 0.f, "need tau, lam >= 0 with tau + lam > 0, got (%g, %g)",
             (double)tau, (double)lam);
  MB_REQUIRE(n_pos >= 0 && n >= 0, "klent_improve: negative size");
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(policy_logits && q_score && q_values && offsets && probs && v_hat && kl && norm_entropy,
             "klent_improve: null pointer");
  MB_REQUIRE(!uniforms || (stored && ranks && pi_top1 && pi_chosen),
             "klent_improve: a draw needs the stored, ranks, pi_top1 and pi_chosen outputs");
  MB_REQUIRE(n_pos <= 0x7fffffff, "klent_improve: too many positions");
  mb::klent::improve_kernel<<<(unsigned)n_pos, mb::klent::kThreads, 0, mb::as_stream(stream)>>>(
      policy_logits, q_score, q_values, offsets, n_pos, n, tau, lam, probs, v_hat, kl, norm_entropy, uniforms, stored,
      ranks, pi_top1, pi_chosen);
  return mb::launch_status("klent_improve");
}

}  // extern "C"

extern "C" int mb_segment_argmax(const float* x, const int64_t* offsets, int64_t n_pos, int64_t n, int64_t* ranks,
                                 void* stream) {
  MB_REQUIRE(n_pos >= 0 && n >= 0, "segment_argmax: negative size");
  if (n_pos == 0) return MB_OK;
  MB_REQUIRE(x && offsets && ranks, "segment_argmax: null pointer");
  MB_REQUIRE(n_pos <= INT32_MAX, "segment_argmax: too many segments");
  klent::segment_argmax_kernel<<<(unsigned)n_pos, klent::kThreads, 0, as_stream(stream)>>>(x, offsets, n_pos, n,
                                                                                         ranks);
  return launch_status("segment_argmax");
}
