// Hex message pass (the isolated-op workload of config 3) with its
// neighbour rows in shared memory:
//
//   y[r] = x[r] + (mean of x[nbr[r, j]] over the present slots j) @ W^T + b
//
// for contiguous bf16 rows x (n, 256), an int32 (n, 6) neighbour table (-1 =
// absent), W (256, 256) as mb_gemm_weight_image, bf16 y. The definition is
// the workload text (restated in oracle/isolated.py); the neighbour slots
// follow the reference adjacency walk (builder.py:458-471).
//
// A neighbour row lies within 64 rows of its own in the workload's token
// order, so a 128-row tile reads its neighbours from its rows +- 64. One
// persistent CTA per SM takes a contiguous range of tiles and keeps that
// window in shared memory as a ring of four 64-row segments (128 KB): moving
// to the next tile drops two segments and bulk-copies two new ones, so each
// x row crosses from DRAM once per CTA. Rows outside the window (other
// inputs) are read from global memory instead.
//
// Warp roles (12 warps): warp 0 lane 0 issues the MMAs, lane 1 streams W
// K-blocks (two 32 KB stages), lane 2 loads window segments; warps 1-7 form
// the mean A tile K-block by K-block (two 16 KB stages, 128-byte swizzled
// K-major, eight lanes per row reading one 128-byte piece of each neighbour
// row: conflict-free); warps 8-11 drain the two TMEM accumulators (256
// columns each), add bias and x[r] (read back through L2, where the window
// copy left it) and write y. Every mbarrier wait is bounded.
#include "common.cuh"

namespace mb {
namespace sm100 {

constexpr int HX_SEG = 64;                        // rows per window segment
constexpr int HX_SEG_BYTES = HX_SEG * KDIM * 2;   // 32 KB
constexpr int HX_NSEG = 4;                        // a tile's rows +- 64
constexpr int HX_PRODUCERS = 7;
constexpr int HX_EPI = 4;
constexpr int HX_THREADS = (1 + HX_PRODUCERS + HX_EPI) * 32;
constexpr int HX_WIN_OFF = 0;
constexpr int HX_A_OFF = HX_WIN_OFF + HX_NSEG * HX_SEG_BYTES;
constexpr int HX_W_OFF = HX_A_OFF + 2 * A_KB_BYTES;
constexpr int HX_BAR_OFF = HX_W_OFF + 2 * W_KB_BYTES;
constexpr int HX_BIAS_OFF = HX_BAR_OFF + 256;      // the bias (256 fp32)
constexpr int HX_ZERO_OFF = HX_BIAS_OFF + KDIM * 4;  // one zero row: absent neighbours read it
constexpr int HX_SMEM = HX_ZERO_OFF + KDIM * 2 + 1024;  // + alignment slack
static_assert(HX_SMEM <= 232448, "hex window plan exceeds 227 KB");
static_assert(BN == KDIM && BM == 2 * HX_SEG, "the window plan assumes 128-row tiles of 256 columns");

__global__ void __launch_bounds__(HX_THREADS, 1) hex_window_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t n, const int32_t* __restrict__ nbr,
    const __nv_bfloat16* __restrict__ w_img, const float* __restrict__ bias, __nv_bfloat16* __restrict__ out,
    int64_t ldo) {
  extern __shared__ uint8_t hx_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(hx_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* win = smem + HX_WIN_OFF;
  uint8_t* a_smem = smem + HX_A_OFF;
  uint8_t* w_smem = smem + HX_W_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + HX_BAR_OFF);
  float* bias_s = reinterpret_cast<float*>(smem + HX_BIAS_OFF);
  uint64_t* seg_full = bars;        // [4]
  uint64_t* mean_done = bars + 4;   // [1]
  uint64_t* a_full = bars + 5;      // [2]
  uint64_t* a_empty = bars + 7;     // [2]
  uint64_t* w_full = bars + 9;      // [2]
  uint64_t* w_empty = bars + 11;    // [2]
  uint64_t* t_full = bars + 13;     // [2]
  uint64_t* t_empty = bars + 15;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 18);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_tiles = (n + BM - 1) / BM;
  const int64_t t0 = n_tiles * blockIdx.x / gridDim.x, t1 = n_tiles * (blockIdx.x + 1) / gridDim.x;
  const int64_t my_tiles = t1 - t0;
  const int64_t s0 = 2 * t0 - 1;  // the first window segment (rows 64 s0 ...)

  if (threadIdx.x == 0) {
    for (int i = 0; i < HX_NSEG; ++i) mbar_init(smem_u32(&seg_full[i]), 1);
    mbar_init(smem_u32(&mean_done[0]), HX_PRODUCERS);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&a_full[i]), HX_PRODUCERS);
      mbar_init(smem_u32(&a_empty[i]), 1);
      mbar_init(smem_u32(&w_full[i]), 1);
      mbar_init(smem_u32(&w_empty[i]), 1);
      mbar_init(smem_u32(&t_full[i]), 1);
      mbar_init(smem_u32(&t_empty[i]), HX_EPI);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x < KDIM) {
    bias_s[threadIdx.x] = bias ? bias[threadIdx.x] : 0.f;
    reinterpret_cast<__nv_bfloat16*>(smem + HX_ZERO_OFF)[threadIdx.x] = __float2bfloat16(0.f);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int64_t n_kb = my_tiles * (KDIM / BK);  // K-blocks of the CTA, in MMA order

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      const uint32_t idesc = make_idesc(BN);
      bool ok = true;
      for (int64_t i = 0; ok && i < my_tiles && !*abort; ++i) {
        const uint32_t tb = i & 1, tph = (i >> 1) & 1;
        if (!mbar_wait(smem_u32(&t_empty[tb]), tph ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + tb * BN;
        for (int kb = 0; kb < KDIM / BK; ++kb) {
          const int64_t q = i * (KDIM / BK) + kb;
          const uint32_t s = q & 1, ph = (q >> 1) & 1;
          if (!mbar_wait(smem_u32(&a_full[s]), ph, abort) || !mbar_wait(smem_u32(&w_full[s]), ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(a_smem + s * A_KB_BYTES), b0 = smem_u32(w_smem + s * W_KB_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            umma(d, smem_desc(a0 + j * 32), smem_desc(b0 + j * 32), idesc, (kb | j) != 0);
          umma_commit(smem_u32(&a_empty[s]));
          umma_commit(smem_u32(&w_empty[s]));
        }
        if (!ok) break;
        umma_commit(smem_u32(&t_full[tb]));
      }
    } else if (lane == 1) {
      // ------------------------------------------- W K-blocks, two stages
      const uint8_t* wimg = reinterpret_cast<const uint8_t*>(w_img);
      for (int64_t q = 0; q < n_kb && !*abort; ++q) {
        const uint32_t s = q & 1, ph = (q >> 1) & 1;
        if (!mbar_wait(smem_u32(&w_empty[s]), ph ^ 1, abort)) break;
        mbar_expect_tx(smem_u32(&w_full[s]), W_KB_BYTES);
        bulk_g2s(smem_u32(w_smem + s * W_KB_BYTES), wimg + (size_t)(q % (KDIM / BK)) * W_KB_BYTES, W_KB_BYTES,
                 smem_u32(&w_full[s]));
      }
    } else if (lane == 2) {
      // ------------------------------------------------ window segments
      auto load_seg = [&](int64_t s) {
        const int slot = (int)((s - s0) & (HX_NSEG - 1));
        const int64_t r0 = s * HX_SEG;
        const int64_t lo = r0 < 0 ? 0 : r0, hi = r0 + HX_SEG < n ? r0 + HX_SEG : n;
        const uint32_t bar = smem_u32(&seg_full[slot]);
        if (hi > lo && lo == r0) {
          const uint32_t bytes = (uint32_t)(hi - lo) * KDIM * 2;
          mbar_expect_tx(bar, bytes);
          bulk_g2s(smem_u32(win + slot * HX_SEG_BYTES), x + lo * KDIM, bytes, bar);
        } else {
          mbar_arrive(bar);  // a segment before row 0 or past the last row: nothing to copy
        }
      };
      for (int64_t s = s0; s < s0 + HX_NSEG; ++s) load_seg(s);
      for (int64_t i = 0; i + 1 < my_tiles && !*abort; ++i) {
        // tile t0 + i no longer needs its first two segments once its mean is formed
        if (!mbar_wait(smem_u32(&mean_done[0]), i & 1, abort)) break;
        const int64_t t = t0 + i;
        load_seg(2 * t + 3);
        load_seg(2 * t + 4);
      }
    }
  } else if (warp <= HX_PRODUCERS) {
    // ------------------------------------------------- mean A tile (K-blocks)
    // A thread's rows of a tile are r = 4 g + sub for g = pw + 7 k. Their
    // neighbour indices are loaded a tile ahead and turned once per tile into
    // codes: >= 0 the byte offset of the neighbour row in shared memory (an
    // absent slot reads the zero row), <= -2 a row outside the window (-2 -
    // code, read from global memory). Unless some row of the warp has such a
    // neighbour, the four K-blocks of the tile read six shared-memory rows per
    // row with no branch.
    const int pw = warp - 1;
    const int sub = lane >> 3, c8 = lane & 7;  // 4 rows per warp step, 8 lanes (16 B each) per row
    constexpr int GROUPS = (BM / 4 + HX_PRODUCERS - 1) / HX_PRODUCERS;
    int raw[GROUPS][HEX_SLOTS];
    auto fetch = [&](int64_t t) {
#pragma unroll
      for (int k = 0; k < GROUPS; ++k) {
        const int g = pw + HX_PRODUCERS * k;
        const int64_t row = t * BM + g * 4 + sub;
        const bool live = g < BM / 4 && row < n;
#pragma unroll
        for (int j = 0; j < HEX_SLOTS; ++j) raw[k][j] = live ? __ldg(nbr + row * HEX_SLOTS + j) : -1;
      }
    };
    if (my_tiles > 0) fetch(t0);
    bool ok = true;
    for (int64_t i = 0; ok && i < my_tiles && !*abort; ++i) {
      const int64_t t = t0 + i, r0 = t * BM;
      const int64_t wbase = r0 - HX_SEG;  // first row of the window (segment 2t - 1)
      int code[GROUPS][HEX_SLOTS];
      float inv[GROUPS];
#pragma unroll
      for (int k = 0; k < GROUPS; ++k) {
        int present = 0;
#pragma unroll
        for (int j = 0; j < HEX_SLOTS; ++j) {
          const int64_t nb = raw[k][j];
          int c = HX_ZERO_OFF;
          if (nb >= n) {
            report(ERR_INDEX);
          } else if (nb >= 0) {
            const int64_t wr = nb - wbase;
            if (wr >= 0 && wr < HX_NSEG * HX_SEG) {
              const int slot = (int)((2 * t - 1 + wr / HX_SEG - s0) & (HX_NSEG - 1));
              c = slot * HX_SEG_BYTES + (int)(nb & (HX_SEG - 1)) * (KDIM * 2);
            } else {
              c = -2 - (int)nb;
            }
            ++present;
          }
          code[k][j] = c;
        }
        inv[k] = present ? 1.f / (float)present : 0.f;
      }
      bool far_row = false;
#pragma unroll
      for (int k = 0; k < GROUPS; ++k)
#pragma unroll
        for (int j = 0; j < HEX_SLOTS; ++j) far_row |= code[k][j] < 0;
      const bool far = __any_sync(0xffffffffu, far_row);
      if (i + 1 < my_tiles) fetch(t + 1);  // in flight during this tile
      // this tile's new segments (all four for the first tile)
      for (int64_t s = (i == 0 ? s0 : 2 * t + 1); s <= 2 * t + 2; ++s) {
        const int slot = (int)((s - s0) & (HX_NSEG - 1));
        if (!mbar_wait(smem_u32(&seg_full[slot]), ((s - s0) >> 2) & 1, abort)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      for (int kb = 0; ok && kb < KDIM / BK; ++kb) {
        const int64_t q = i * (KDIM / BK) + kb;
        const uint32_t s = q & 1, ph = (q >> 1) & 1;
        if (!mbar_wait(smem_u32(&a_empty[s]), ph ^ 1, abort)) {
          ok = false;
          break;
        }
        uint8_t* abuf = a_smem + s * A_KB_BYTES;
        const uint8_t* wk = win + kb * 128 + c8 * 16;
#pragma unroll
        for (int k = 0; k < GROUPS; ++k) {
          const int g = pw + HX_PRODUCERS * k;
          if (g >= BM / 4) break;
          const int r = g * 4 + sub;
          float acc[8] = {};
          uint4 raw16[HEX_SLOTS];
          if (!far) {
#pragma unroll
            for (int j = 0; j < HEX_SLOTS; ++j) raw16[j] = *reinterpret_cast<const uint4*>(wk + code[k][j]);
          } else {
#pragma unroll
            for (int j = 0; j < HEX_SLOTS; ++j) {
              const int c = code[k][j];
              raw16[j] = c >= 0 ? *reinterpret_cast<const uint4*>(wk + c)
                                : __ldg(reinterpret_cast<const uint4*>(x + (int64_t)(-2 - c) * KDIM + kb * BK) + c8);
            }
          }
#pragma unroll
          for (int j = 0; j < HEX_SLOTS; ++j) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw16[j]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              acc[2 * e] += f.x;
              acc[2 * e + 1] += f.y;
            }
          }
          uint4 w4;
          __nv_bfloat162* hw = reinterpret_cast<__nv_bfloat162*>(&w4);
#pragma unroll
          for (int e = 0; e < 4; ++e) hw[e] = __floats2bfloat162_rn(acc[2 * e] * inv[k], acc[2 * e + 1] * inv[k]);
          *reinterpret_cast<uint4*>(abuf + r * 128 + ((c8 ^ (r & 7)) << 4)) = w4;
        }
        fence_proxy_async();  // generic-proxy stores -> visible to the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&a_full[s]));
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(smem_u32(&mean_done[0]));
    }
  } else {
    // --------------------------------------------------------- epilogue
    const int qd = warp & 3;  // TMEM lane quadrant
    for (int64_t i = 0; i < my_tiles && !*abort; ++i) {
      const uint32_t tb = i & 1, tph = (i >> 1) & 1;
      if (!mbar_wait(smem_u32(&t_full[tb]), tph, abort)) break;
      tc_fence_after();
      const int64_t row = (t0 + i) * BM + qd * 32 + lane;
      const bool live = row < n;
      // x[r] is read back through L2 (the window slots may be refilled by
      // now), each 32-column chunk's 64 bytes requested two chunks ahead
      const uint4* xr = reinterpret_cast<const uint4*>(x + (live ? row : 0) * KDIM);
      constexpr int CH = BN / 32;
      uint4 xq[3][4];
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) xq[c][e] = live ? __ldg(xr + 4 * c + e) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        if (c + 2 < CH) {
#pragma unroll
          for (int e = 0; e < 4; ++e) xq[(c + 2) % 3][e] = live ? __ldg(xr + 4 * (c + 2) + e) : make_uint4(0, 0, 0, 0);
        }
        const int c0 = 32 * c;
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(qd * 32) << 16) + tb * BN + c0, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float4 bb = reinterpret_cast<const float4*>(bias_s + c0)[e];
          v[4 * e] += bb.x; v[4 * e + 1] += bb.y; v[4 * e + 2] += bb.z; v[4 * e + 3] += bb.w;
        }
        if (live) {
          uint4* orow = reinterpret_cast<uint4*>(out + row * ldo + c0);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&xq[c % 3][e]);
            uint4 w4;
            __nv_bfloat162* hw = reinterpret_cast<__nv_bfloat162*>(&w4);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 f = __bfloat1622float2(hx[u]);
              hw[u] = __floats2bfloat162_rn(v[8 * e + 2 * u] + f.x, v[8 * e + 2 * u + 1] + f.y);
            }
            orow[e] = w4;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&t_empty[tb]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// The window path of mb_hex_message_pass: contiguous rows (ldx == 256).
static int hex_window_launch(const void* x, int64_t n, const int32_t* nbr, const void* w_image, const float* bias,
                             void* out, int64_t ldo, cudaStream_t s) {
  if (cudaFuncSetAttribute(hex_window_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, HX_SMEM) != cudaSuccess)
    return ::mb::fail(MB_LAUNCH_FAILED, "hex_message_pass: %d bytes of shared memory refused", HX_SMEM);
  const int64_t tiles = (n + BM - 1) / BM;
  const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
  hex_window_kernel<<<grid, HX_THREADS, HX_SMEM, s>>>((const __nv_bfloat16*)x, n, nbr,
                                                      (const __nv_bfloat16*)w_image, bias, (__nv_bfloat16*)out, ldo);
  return launch_status("hex_message_pass");
}

}  // namespace sm100
}  // namespace mb
