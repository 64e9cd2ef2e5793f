// gemv.cu -- HBM-bound decode matvecs over repacked Q4 / Q8 weight tiles.
//
// Semantics restated from the reference shaders:
//   gemv_q4.wgsl:28-93      y[r] = sum_b d_rb * sum_i (q_i - 8) * x_{32b+i}      (the f16 `min` is ignored)
//   fused_qkv_q4.wgsl       q|k|v rows are one concatenated matrix here
//   fused_mlp_q4.wgsl:33-128 act[r] = gelu_tanh(Wg x)[r] * (Wu x)[r]             (gate/up rows interleaved per tile)
//   gemv_q8.wgsl            logits[r] = sum_b s_rb * sum_i q_i x_i               (int8, f32 scale)
//
// B200 design: each warp streams a contiguous range of 576-byte tiles with
// 1-D bulk copies (cp.async.bulk, mbarrier completion, SPW stages per warp) --
// the ranges are an even "stream-K" split of all tiles over every warp of a
// persistent grid.  With at least as many row tiles as CTAs, each CTA takes
// whole row tiles and splits their tiles evenly over its warps (cut row tiles
// are added in shared memory); otherwise the split is grid-wide and cut row
// tiles are combined through global memory by the last-arriving warp.  Both
// combines add in a fixed order.  The weights feed integer mma.sync (m16n8k32,
// s8): a Q4 nibble becomes 16 (q - 8) by one mask-and-xor and a Q8 byte q by one
// xor, against x as four s8 limbs per value under a power-of-two scale per
// 32-block (core.cuh: build_limbs / tile_i8), so every block dot product is an
// exact integer; the block scales are applied in f32.  The input prologue fuses the
// reference's rmsnorm / add_rmsnorm passes (add_rmsnorm.wgsl:15-51) so no
// separate norm kernel runs on the decode path.
#include <cmath>

#include <atomic>
#include <map>
#include <mutex>

#include "common.cuh"
#include "core.cuh"
#include "kernels.cuh"

namespace ch {

namespace {
#ifndef CH_GEMV_SPW
#define CH_GEMV_SPW 2
#endif
#ifndef CH_GEMV_CT
#define CH_GEMV_CT 8
#endif
constexpr int NW = 16;           // consumer warps per CTA (each self-feeds its own stages)
constexpr int SPW = CH_GEMV_SPW;  // stages per warp
constexpr int CT = CH_GEMV_CT;    // tiles per stage (8: 4608 B per bulk copy)
static_assert(CT % 2 == 0, "the unrolled stage loop consumes tiles in pairs");
constexpr int kStageBytes = CT * kTileBytes;
}  // namespace

int num_sms() {
  constexpr int kMaxDev = 64;
  static std::atomic<int> cache[kMaxDev];  // zero: not looked up yet
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  int n = (dev >= 0 && dev < kMaxDev) ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < kMaxDev) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}
cudaError_t ensure_smem_attr(const void *func, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, size_t> granted;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  size_t &g = granted[{dev, func}];
  if (smem <= g) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) g = smem;
  return e;
}
int gemv_default_grid() { return num_sms(); }
size_t gemv_partial_floats(int grid) { return (size_t)grid * NW * 2 * 16; }

// first tile of warp w's range
CH_DEV uint64_t range_begin(uint64_t T, uint64_t w, uint64_t GW) { return (T * w) / GW; }
// warp whose range contains tile t (T > 0)
CH_DEV uint64_t warp_of(uint64_t t, uint64_t T, uint64_t GW) {
  uint64_t w = ((t + 1) * GW + T - 1) / T - 1;
  return w;
}

template <int EPI>
CH_DEV void epilogue(float *y, uint32_t rt, int g, float v0, float v1) {
  if (EPI == EPI_STORE) {
    y[rt * 16 + g] = v0;
    y[rt * 16 + g + 8] = v1;
  } else {
    y[rt * 8 + g] = __fmul_rn(gelu_tanh(v0), v1);
  }
}

template <int PRO>
CH_DEV void prologue(const GemvArgs &a, float *vec, uint2 *xq, float *sxs, float *red) {
  const uint32_t K = a.K, nb = K / 32;
  if (PRO == PRO_NONE) {
    build_limbs(a.x, xq, sxs, K);
    return;
  }
  const bool writer = (blockIdx.x == 0);
  float ss = 0.0f;
  if (PRO == PRO_RMSNORM) {
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      float v[32];
      load32(a.x + b * 32, v);
#pragma unroll
      for (int e = 0; e < 32; e++) ss = __fmaf_rn(v[e], v[e], ss);
      store32(vec + b * 32, v);
    }
  } else {  // PRO_ADD_RMSNORM: r' = post_w ? rmsnorm(r) * post_w : r ; x = (x_in + r') * scalar
    float inv_r = 1.0f;
    if (a.post_w) {
      float sr = 0.0f;
      for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        float v[32];
        load32(a.r + b * 32, v);
#pragma unroll
        for (int e = 0; e < 32; e++) sr = __fmaf_rn(v[e], v[e], sr);
      }
      sr = block_sum(sr, red);
      inv_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sr, (float)K), a.eps)));
    }
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      float r[32], x[32], w[32];
      load32(a.r + b * 32, r);
      load32(a.x + b * 32, x);
      if (a.post_w) load32(a.post_w + b * 32, w);
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const float rr = a.post_w ? __fmul_rn(__fmul_rn(r[e], inv_r), w[e]) : r[e];
        x[e] = __fmul_rn(__fadd_rn(x[e], rr), a.scalar);
        ss = __fmaf_rn(x[e], x[e], ss);
      }
      store32(vec + b * 32, x);
      if (writer && a.x_out) store32(a.x_out + b * 32, x);
    }
  }
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
  for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(vec[i], inv), a.norm_w[i]);
    vec[i] = v;
    if (writer && a.normed_out) a.normed_out[i] = v;
  }
  __syncthreads();
  build_limbs(vec, xq, sxs, K);
}

template <int FMT, int EPI, int PRO>
__global__ void __launch_bounds__(NW * 32, 1) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *stages = smem;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + NW * SPW * kStageBytes);
  float *vec = reinterpret_cast<float *>(smem + NW * SPW * kStageBytes + NW * SPW * 8);  // norm prologues: K floats
  uint2 *xq = reinterpret_cast<uint2 *>(vec + (PRO == PRO_NONE ? 0u : a.K));              // input limbs
  float *sxs = reinterpret_cast<float *>(xq + (a.K / 32) * 16);                           // their block scales
  __shared__ float red[32];
  __shared__ float cpart[NW][2][16];  // CTA-local mode: partial row-tile sums, [warp][first/last segment][row]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint64_t GW = (uint64_t)gridDim.x * NW;
  const uint64_t gw = (uint64_t)blockIdx.x * NW + warp;
  const uint64_t KT = a.k_tiles;
  const uint64_t T = (uint64_t)a.row_tiles * KT;
  // Global stream-K: an even split of all tiles over every warp of the grid (a warp's
  // range may cut row tiles, whose partial sums the last contributor adds through
  // global memory).  CTA-local (a.cta_rows): each CTA takes whole row tiles and
  // splits their tiles evenly over its warps; cut row tiles are added up in shared
  // memory after one CTA barrier.
  const bool local = a.cta_rows != 0;
  const uint64_t cr0 = range_begin(a.row_tiles, blockIdx.x, gridDim.x) * KT;  // this CTA's tiles (local)
  const uint64_t CTn = range_begin(a.row_tiles, blockIdx.x + 1, gridDim.x) * KT - cr0;
  const uint64_t tb = local ? cr0 + range_begin(CTn, warp, NW) : range_begin(T, gw, GW);
  const uint64_t te = local ? cr0 + range_begin(CTn, warp + 1, NW) : range_begin(T, gw + 1, GW);
  const uint32_t nchunks = (uint32_t)((te - tb + CT - 1) / CT);
  uint8_t *my_stages = stages + (size_t)warp * SPW * kStageBytes;
  uint64_t *my_bars = bars + warp * SPW;

  // weights do not depend on the previous kernel: start streaming before the dependency wait
  if (lane == 0) {
    for (int s = 0; s < SPW; s++) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
    for (uint32_t j = 0; j < (uint32_t)SPW && j < nchunks; j++) {
      uint64_t t0 = tb + (uint64_t)j * CT;
      uint32_t bytes = (uint32_t)(min((uint64_t)CT, te - t0) * kTileBytes);
      mbar_arrive_expect_tx(&my_bars[j], bytes);
      bulk_g2s(my_stages + (size_t)j * kStageBytes, a.tiles + t0 * kTileBytes, bytes, &my_bars[j]);
    }
  }
  __syncwarp();

  grid_dep_wait();
  prologue<PRO>(a, vec, xq, sxs, red);
  __syncthreads();
  grid_dep_launch();

  const uint2 *xql = xq + t * 4 + (g & 3);
  uint64_t cur_rt = ~0ull, rt = 0;
  uint32_t kt_begin = 0, kt = 0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, accb[4] = {0.f, 0.f, 0.f, 0.f};  // two chains (even / odd tiles)
  bool first_seg = true;
  if (nchunks > 0) {
    rt = tb / KT;
    kt = (uint32_t)(tb - rt * KT);
  }

  auto flush = [&](uint64_t frt, uint32_t kb, uint32_t ke) {
    float acc0, acc1;
    limb_rows<FMT>(acc, accb, t, acc0, acc1);
    const bool full = (kb == 0 && ke == (uint32_t)KT);
    if (full) {
      if (t == 0) epilogue<EPI>(a.y, (uint32_t)frt, g, acc0, acc1);
    } else if (local) {
      if (t == 0) {
        cpart[warp][first_seg ? 0 : 1][g] = acc0;
        cpart[warp][first_seg ? 0 : 1][g + 8] = acc1;
      }
    } else {
      const int slot = first_seg ? 0 : 1;
      if (t == 0) {
        a.partial[(gw * 2 + slot) * 16 + g] = acc0;
        a.partial[(gw * 2 + slot) * 16 + g + 8] = acc1;
      }
      __threadfence();
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atomicAdd(&a.counters[frt], 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      const uint64_t w_first = warp_of(frt * KT, T, GW), w_last = warp_of((frt + 1) * KT - 1, T, GW);
      uint32_t ncontrib = 0;
      for (uint64_t w = w_first; w <= w_last; w++)
        if (range_begin(T, w + 1, GW) > range_begin(T, w, GW)) ncontrib++;
      if (old == ncontrib - 1) {
        __threadfence();
        float v0 = 0.f, v1 = 0.f;
        for (uint64_t w = w_first; w <= w_last; w++) {
          uint64_t b = range_begin(T, w, GW);
          if (range_begin(T, w + 1, GW) == b) continue;
          const int sl = (b / KT == frt) ? 0 : 1;
          v0 = __fadd_rn(v0, __ldcg(&a.partial[(w * 2 + sl) * 16 + g]));
          v1 = __fadd_rn(v1, __ldcg(&a.partial[(w * 2 + sl) * 16 + g + 8]));
        }
        if (t == 0) epilogue<EPI>(a.y, (uint32_t)frt, g, v0, v1);
        if (lane == 0) a.counters[frt] = 0u;
      }
    }
    first_seg = false;
  };

  uint32_t failed_at = 0;
  bool ok = true;
  for (uint32_t j = 0; j < nchunks; j++) {
    const int s = j % SPW;
    if (!mbar_wait_bounded(&my_bars[s], (j / SPW) & 1, a.err)) {
      ok = false;
      failed_at = j;
      break;
    }
    const uint8_t *st = my_stages + (size_t)s * kStageBytes;
    const uint64_t t0 = tb + (uint64_t)j * CT;
    const uint32_t nt = (uint32_t)min((uint64_t)CT, te - t0);
    uint32_t i = 0;
    while (i < nt) {
      if (rt != cur_rt) {
        if (cur_rt != ~0ull) flush(cur_rt, kt_begin, (uint32_t)KT);
        cur_rt = rt;
        kt_begin = kt;
#pragma unroll
        for (int c = 0; c < 4; c++) acc[c] = accb[c] = 0.f;
      }
      // a run of tiles inside one row tile: no per-tile boundary checks
      const uint32_t run = min(nt - i, (uint32_t)KT - kt);
      const uint8_t *p = st + (size_t)i * kTileBytes;
      uint32_t r = 0;
      if (run == CT) {
#pragma unroll
        for (int q = 0; q < CT; q += 2) {
          tile_i8<FMT>(p + q * kTileBytes, kt + q, xql, sxs, lane, acc);
          tile_i8<FMT>(p + (q + 1) * kTileBytes, kt + q + 1, xql, sxs, lane, accb);
        }
        r = CT;
      } else {
        for (; r + 2 <= run; r += 2) {
          tile_i8<FMT>(p + r * kTileBytes, kt + r, xql, sxs, lane, acc);
          tile_i8<FMT>(p + (r + 1) * kTileBytes, kt + r + 1, xql, sxs, lane, accb);
        }
        if (r < run) {
          tile_i8<FMT>(p + r * kTileBytes, kt + r, xql, sxs, lane, acc);
          r++;
        }
      }
      i += run;
      kt += run;
      if (kt == (uint32_t)KT) {
        kt = 0;
        rt++;
      }
    }
    __syncwarp();
    if (lane == 0 && j + SPW < nchunks) {
      fence_proxy_async();
      const uint64_t tn = tb + (uint64_t)(j + SPW) * CT;
      const uint32_t bytes = (uint32_t)(min((uint64_t)CT, te - tn) * kTileBytes);
      mbar_arrive_expect_tx(&my_bars[s], bytes);
      bulk_g2s(my_stages + (size_t)s * kStageBytes, a.tiles + tn * kTileBytes, bytes, &my_bars[s]);
    }
  }
  if (!ok) {
    // drain the copies this warp still has in flight (chunks failed_at .. +SPW-1), bounded
    for (uint32_t j = failed_at + 1; j < nchunks && j < failed_at + SPW; j++)
      mbar_wait_bounded(&my_bars[j % SPW], (j / SPW) & 1, nullptr, 100000000ull);
  } else if (cur_rt != ~0ull) {
    const uint32_t ke = (uint32_t)(te - cur_rt * KT);
    flush(cur_rt, kt_begin, ke);
  }
  if (!local) return;
  __syncthreads();
  if (!__all_sync(0xffffffffu, ok)) return;  // the device error word already records the failure
  // The warp whose range holds the last tile of a cut row tile adds the partials of
  // every warp that touched it, in warp order (slot 0 = that warp's first segment,
  // slot 1 = its last).  Only a warp's first segment can start inside a row tile, so
  // the combiner is the warp whose range starts inside row tile r and reaches its end.
  if (te == tb || tb % KT == 0 || te < (tb / KT + 1) * KT) return;
  const uint64_t frt = tb / KT, lo = frt * KT - cr0;
  const uint32_t w_first = (uint32_t)warp_of(lo, CTn, NW);
  float v0 = 0.f, v1 = 0.f;
  for (uint32_t w = w_first; w <= (uint32_t)warp; w++) {
    const uint64_t b = range_begin(CTn, w, NW);
    if (range_begin(CTn, w + 1, NW) == b) continue;
    const int sl = (b >= lo) ? 0 : 1;
    v0 = __fadd_rn(v0, cpart[w][sl][g]);
    v1 = __fadd_rn(v1, cpart[w][sl][g + 8]);
  }
  if (t == 0) epilogue<EPI>(a.y, (uint32_t)frt, g, v0, v1);
}

template <int FMT, int EPI, int PRO>
static cudaError_t launch_gemv_t(const GemvArgs &a, int grid, cudaStream_t s, bool pdl) {
  size_t smem = (size_t)NW * SPW * kStageBytes + NW * SPW * 8 + (size_t)(a.K / 32) * (128 + 4);
  if (PRO != PRO_NONE) smem += (size_t)a.K * 4;
  {
    const cudaError_t e = ensure_smem_attr((const void *)gemv_kernel<FMT, EPI, PRO>, smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, EPI, PRO>, a);
}

cudaError_t launch_gemv(const GemvPlan &p, const GemvArgs &a0, cudaStream_t s, bool pdl) {
  if (a0.K % 64 != 0 && p.fmt == FMT_Q4) return cudaErrorInvalidValue;
  if (a0.K % 32 != 0) return cudaErrorInvalidValue;
  int grid = p.grid > 0 ? p.grid : gemv_default_grid();
  // Whole row tiles per CTA (stream-K over its warps, cut rows added in shared memory)
  // whenever every CTA gets at least one: even an uneven share (240 row tiles on 148
  // CTAs) beats the grid-wide split, whose cross-CTA combine (fences, counters, a
  // second pass over global partials) costs several microseconds per launch.
  GemvArgs a = a0;
  a.cta_rows = a.row_tiles >= (uint32_t)grid;
#define CH_GEMV_CASE(F, E, P) \
  if (p.fmt == F && p.epi == E && p.pro == P) return launch_gemv_t<F, E, P>(a, grid, s, pdl);
  CH_GEMV_CASE(FMT_Q4, EPI_STORE, PRO_NONE)
  CH_GEMV_CASE(FMT_Q4, EPI_STORE, PRO_RMSNORM)
  CH_GEMV_CASE(FMT_Q4, EPI_STORE, PRO_ADD_RMSNORM)
  CH_GEMV_CASE(FMT_Q4, EPI_GELU_MUL, PRO_NONE)
  CH_GEMV_CASE(FMT_Q4, EPI_GELU_MUL, PRO_RMSNORM)
  CH_GEMV_CASE(FMT_Q4, EPI_GELU_MUL, PRO_ADD_RMSNORM)
  CH_GEMV_CASE(FMT_Q8, EPI_STORE, PRO_NONE)
  CH_GEMV_CASE(FMT_Q8, EPI_STORE, PRO_RMSNORM)
  CH_GEMV_CASE(FMT_Q8, EPI_STORE, PRO_ADD_RMSNORM)
#undef CH_GEMV_CASE
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// repack: quant.zig blocks (5 words / 32 weights, src/quant.zig:54-98) -> tiles.
// One thread per (tile, lane).  rowmap MAP_GATEUP interleaves two matrices:
// tile rows 0..7 come from `src` rows rt*8.., rows 8..15 from `src_b`.
CH_DEV uint32_t q4_nib(const uint32_t *src, uint32_t nb, uint32_t row, uint32_t k) {
  uint32_t b = k >> 5, n = k & 31;
  return (src[((size_t)row * nb + b) * 5 + 1 + (n >> 3)] >> (4 * (n & 7))) & 0xFu;
}
__global__ void repack_q4_kernel(const uint32_t *src, const uint32_t *src_b, uint32_t rows_out, uint32_t cols, int rowmap,
                                 uint8_t *dst) {
  const uint32_t KT = cols / kQ4TileK, nb = cols / 32;
  const uint64_t total = (uint64_t)(rows_out / 16) * KT * 32;
  for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t lane = idx & 31;
    const uint64_t tile = idx >> 5;
    const uint32_t rt = (uint32_t)(tile / KT), kt = (uint32_t)(tile % KT);
    const uint32_t g = lane >> 2, t = lane & 3;
    const uint32_t *sa, *sb;
    uint32_t ra, rb;
    if (rowmap == MAP_GATEUP) {
      sa = src;
      sb = src_b;
      ra = rt * 8 + g;
      rb = rt * 8 + g;
    } else {
      sa = src;
      sb = src;
      ra = rt * 16 + g;
      rb = rt * 16 + g + 8;
    }
    uint32_t out[4];
#pragma unroll
    for (int blk = 0; blk < 2; blk++)
#pragma unroll
      for (int ch = 0; ch < 2; ch++) {
        const uint32_t kb = kt * 64 + blk * 32 + ch * 16;
        uint32_t w = 0;
        w |= q4_nib(sa, nb, ra, kb + 2 * t) << 0;
        w |= q4_nib(sa, nb, ra, kb + 2 * t + 1) << 16;
        w |= q4_nib(sb, nb, rb, kb + 2 * t) << 4;
        w |= q4_nib(sb, nb, rb, kb + 2 * t + 1) << 20;
        w |= q4_nib(sa, nb, ra, kb + 2 * t + 8) << 8;
        w |= q4_nib(sa, nb, ra, kb + 2 * t + 9) << 24;
        w |= q4_nib(sb, nb, rb, kb + 2 * t + 8) << 12;
        w |= q4_nib(sb, nb, rb, kb + 2 * t + 9) << 28;
        out[blk * 2 + ch] = w;
      }
    uint8_t *tp = dst + tile * kTileBytes;
    *reinterpret_cast<uint4 *>(tp + lane * 16) = make_uint4(out[0], out[1], out[2], out[3]);
    if (t == 0) {
      const uint32_t b0 = kt * 2, b1 = kt * 2 + 1;
      uint32_t sa0 = sa[((size_t)ra * nb + b0) * 5] & 0xFFFFu, sa1 = sa[((size_t)ra * nb + b1) * 5] & 0xFFFFu;
      uint32_t sb0 = sb[((size_t)rb * nb + b0) * 5] & 0xFFFFu, sb1 = sb[((size_t)rb * nb + b1) * 5] & 0xFFFFu;
      *reinterpret_cast<uint2 *>(tp + 512 + g * 8) = make_uint2(sa0 | (sa1 << 16), sb0 | (sb1 << 16));
    }
  }
}
// Q8_0 blocks (9 words / 32, src/quant.zig:19-52) -> tiles; bytes stored as q ^ 0x80
CH_DEV uint32_t q8_byte(const uint32_t *src, uint32_t nb, uint32_t row, uint32_t k) {
  uint32_t b = k >> 5, n = k & 31;
  return ((src[((size_t)row * nb + b) * 9 + 1 + (n >> 2)] >> (8 * (n & 3))) & 0xFFu) ^ 0x80u;
}
__global__ void repack_q8_kernel(const uint32_t *src, uint32_t rows, uint32_t cols, uint8_t *dst) {
  const uint32_t KT = cols / kQ8TileK, nb = cols / 32;
  const uint64_t total = (uint64_t)(rows / 16) * KT * 32;
  for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t lane = idx & 31;
    const uint64_t tile = idx >> 5;
    const uint32_t rt = (uint32_t)(tile / KT), kt = (uint32_t)(tile % KT);
    const uint32_t g = lane >> 2, t = lane & 3;
    const uint32_t ra = rt * 16 + g, rb = ra + 8;
    uint32_t out[4];
#pragma unroll
    for (int ch = 0; ch < 2; ch++) {
      const uint32_t kb = kt * 32 + ch * 16;
      out[ch * 2 + 0] = q8_byte(src, nb, ra, kb + 2 * t) | (q8_byte(src, nb, ra, kb + 2 * t + 1) << 8) |
                        (q8_byte(src, nb, rb, kb + 2 * t) << 16) | (q8_byte(src, nb, rb, kb + 2 * t + 1) << 24);
      out[ch * 2 + 1] = q8_byte(src, nb, ra, kb + 2 * t + 8) | (q8_byte(src, nb, ra, kb + 2 * t + 9) << 8) |
                        (q8_byte(src, nb, rb, kb + 2 * t + 8) << 16) | (q8_byte(src, nb, rb, kb + 2 * t + 9) << 24);
    }
    uint8_t *tp = dst + tile * kTileBytes;
    *reinterpret_cast<uint4 *>(tp + lane * 16) = make_uint4(out[0], out[1], out[2], out[3]);
    if (t == 0) {
      uint32_t da = src[((size_t)ra * nb + kt) * 9], db = src[((size_t)rb * nb + kt) * 9];
      *reinterpret_cast<uint2 *>(tp + 512 + g * 8) = make_uint2(da, db);
    }
  }
}

static int grid_for(uint64_t n, int block) {
  uint64_t g = (n + block - 1) / block;
  uint64_t cap = (uint64_t)num_sms() * 16;
  return (int)(g < cap ? (g > 0 ? g : 1) : cap);
}

cudaError_t launch_repack_q4(const uint32_t *src, const uint32_t *src_b, uint32_t rows_out, uint32_t cols, int rowmap,
                             uint8_t *dst, cudaStream_t s) {
  if (rows_out % 16 || cols % 64) return cudaErrorInvalidValue;
  uint64_t n = (uint64_t)(rows_out / 16) * (cols / 64) * 32;
  repack_q4_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, src_b ? src_b : src, rows_out, cols, rowmap, dst);
  return cudaGetLastError();
}
cudaError_t launch_repack_q8(const uint32_t *src, uint32_t rows, uint32_t cols, uint8_t *dst, cudaStream_t s) {
  if (rows % 16 || cols % 32) return cudaErrorInvalidValue;
  uint64_t n = (uint64_t)(rows / 16) * (cols / 32) * 32;
  repack_q8_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, rows, cols, dst);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// seeded synthetic tensors (same spec as the oracle's or_gen_*)
// blocks [blk0, blk0 + nblocks) of a tensor's block stream (a row range of the matrix)
// block i of the output is global block blk0 + i, or with a column range (nbl > 0)
// global block (i / nbl) * nbf + cb0 + i % nbl: blocks cb0 .. cb0+nbl of rows of nbf
__global__ void gen_q4_kernel(uint32_t *dst, uint64_t blk0, uint64_t nblocks, uint64_t tseed, float scale_std,
                              uint64_t nbf = 0, uint64_t cb0 = 0, uint64_t nbl = 0) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nblocks;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t blk = nbl ? (i / nbl) * nbf + cb0 + i % nbl : blk0 + i;
    uint64_t ha = hash3(tseed, 0, blk * 2), hb = hash3(tseed, 0, blk * 2 + 1);
    float z = gen_normal(tseed, 1, blk);
    float d = __fmul_rn(fabsf(z), scale_std);
    __half d16 = __float2half_rn(d);
    __half m16 = __float2half_rn(__fmul_rn(-8.0f, __half2float(d16)));
    uint32_t *o = dst + i * 5;
    o[0] = (uint32_t)__half_as_ushort(d16) | ((uint32_t)__half_as_ushort(m16) << 16);
    o[1] = (uint32_t)ha;
    o[2] = (uint32_t)(ha >> 32);
    o[3] = (uint32_t)hb;
    o[4] = (uint32_t)(hb >> 32);
  }
}
__global__ void gen_bf16_kernel(uint16_t *dst, uint64_t n, uint64_t tseed, float mean, float std) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float z = gen_normal(tseed, 2, i);
    dst[i] = bf16_rne(__fadd_rn(mean, __fmul_rn(z, std)));
  }
}
__global__ void gen_f32_kernel(float *dst, uint64_t n, uint64_t tseed, float mean, float std) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float z = gen_normal(tseed, 3, i);
    dst[i] = __fadd_rn(mean, __fmul_rn(z, std));
  }
}
__global__ void bf16_to_f32_kernel(const uint16_t *src, float *dst, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = bf16_to_f32(src[i]);
}
// quantizeRowQ8_0 (src/quant.zig:21-52), one warp per 32-element block
__global__ void quantize_q8_kernel(const uint16_t *src, uint64_t nblocks, uint32_t *dst) {
  const int lane = threadIdx.x & 31;
  for (uint64_t blk = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5; blk < nblocks;
       blk += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
    float v = bf16_to_f32(src[blk * 32 + lane]);
    float amax = warp_max(fabsf(v));
    float d = __fdiv_rn(amax, 127.0f);
    float id = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    int q = (int)roundf(__fmul_rn(v, id));
    q = max(-128, min(127, q));
    uint32_t byte = (uint32_t)(q & 0xFF) << (8 * (lane & 3));
    byte |= __shfl_xor_sync(0xffffffffu, byte, 1);
    byte |= __shfl_xor_sync(0xffffffffu, byte, 2);
    uint32_t *o = dst + blk * 9;
    if (lane == 0) o[0] = __float_as_uint(d);
    if ((lane & 3) == 0) o[1 + (lane >> 2)] = byte;
  }
}
// quantizeRowQ4_0 (src/quant.zig:58-98), one warp per block
__global__ void quantize_q4_kernel(const uint16_t *src, uint64_t nblocks, uint32_t *dst) {
  const int lane = threadIdx.x & 31;
  for (uint64_t blk = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5; blk < nblocks;
       blk += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
    float v = bf16_to_f32(src[blk * 32 + lane]);
    float amax = warp_max(fabsf(v));
    float d = __fdiv_rn(amax, 8.0f);
    float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = (int)roundf(__fadd_rn(__fmul_rn(v, id), 8.0f));
    q = max(0, min(15, q));
    uint32_t nib = (uint32_t)q << (4 * (lane & 7));
    nib |= __shfl_xor_sync(0xffffffffu, nib, 1);
    nib |= __shfl_xor_sync(0xffffffffu, nib, 2);
    nib |= __shfl_xor_sync(0xffffffffu, nib, 4);
    uint32_t *o = dst + blk * 5;
    if (lane == 0) {
      __half s = __float2half_rn(d), m = __float2half_rn(__fmul_rn(-8.0f, d));
      o[0] = (uint32_t)__half_as_ushort(s) | ((uint32_t)__half_as_ushort(m) << 16);
    }
    if ((lane & 7) == 0) o[1 + (lane >> 3)] = nib;
  }
}

cudaError_t launch_gen_q4_blocks(uint32_t *dst, uint32_t rows, uint32_t cols, uint64_t tseed, float scale_std,
                                 cudaStream_t s) {
  return launch_gen_q4_rows(dst, 0, rows, cols, tseed, scale_std, s);
}
cudaError_t launch_gen_q4_rows(uint32_t *dst, uint32_t row0, uint32_t rows, uint32_t cols, uint64_t tseed,
                               float scale_std, cudaStream_t s) {
  const uint64_t nb = (uint64_t)rows * (cols / 32), b0 = (uint64_t)row0 * (cols / 32);
  gen_q4_kernel<<<grid_for(nb, 256), 256, 0, s>>>(dst, b0, nb, tseed, scale_std);
  return cudaGetLastError();
}
cudaError_t launch_gen_q4_cols(uint32_t *dst, uint32_t rows, uint32_t cols, uint32_t col0, uint32_t ncols,
                               uint64_t tseed, float scale_std, cudaStream_t s) {
  if (col0 % 32 || ncols % 32 || col0 + ncols > cols) return cudaErrorInvalidValue;
  const uint64_t nbl = ncols / 32, nb = (uint64_t)rows * nbl;
  gen_q4_kernel<<<grid_for(nb, 256), 256, 0, s>>>(dst, 0, nb, tseed, scale_std, cols / 32, col0 / 32, nbl);
  return cudaGetLastError();
}
cudaError_t launch_gen_bf16(uint16_t *dst, size_t n, uint64_t tseed, float mean, float std, cudaStream_t s) {
  gen_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, n, tseed, mean, std);
  return cudaGetLastError();
}
cudaError_t launch_gen_f32(float *dst, size_t n, uint64_t tseed, float mean, float std, cudaStream_t s) {
  gen_f32_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, n, tseed, mean, std);
  return cudaGetLastError();
}
cudaError_t launch_bf16_to_f32(const uint16_t *src, float *dst, size_t n, cudaStream_t s) {
  bf16_to_f32_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, dst, n);
  return cudaGetLastError();
}
cudaError_t launch_quantize_q8_rows(const uint16_t *src, uint32_t rows, uint32_t cols, uint32_t *dst, cudaStream_t s) {
  uint64_t nb = (uint64_t)rows * (cols / 32);
  quantize_q8_kernel<<<grid_for(nb * 32, 256), 256, 0, s>>>(src, nb, dst);
  return cudaGetLastError();
}
cudaError_t launch_quantize_q4_rows(const uint16_t *src, uint32_t rows, uint32_t cols, uint32_t *dst, cudaStream_t s) {
  uint64_t nb = (uint64_t)rows * (cols / 32);
  quantize_q4_kernel<<<grid_for(nb * 32, 256), 256, 0, s>>>(src, nb, dst);
  return cudaGetLastError();
}

}  // namespace ch
