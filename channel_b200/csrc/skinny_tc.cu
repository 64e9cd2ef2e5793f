// skinny_tc.cu -- the Q4 projections of the multi-stream decode step (q|k|v, o,
// gate|up, down) for 17 to 64 tokens on the 5th-generation tensor cores.
//
// Restated reference shader: batch_gemm_q4.wgsl:26-160,
//   Y[t][r] = sum_b d_rb sum_i (q_rbi - 8) X[t][32b + i],
// for one decode token per stream (the reference decodes one stream; the batch is new).
//
// Shape.  A tcgen05 MMA instruction costs about the same time (~128 cycles) at any
// shape up to M256 x N256, so a batch of at most 64 tokens goes on the M side with its
// f16 hi and lo halves stacked: the A operand is the 128 x 16 block
// [X_hi (tokens 0-63) ; X_lo 2^8 (tokens 0-63)] and the B operand 256 weight rows (16 Q4
// row tiles) of one CTA; D is 128 lanes x 256 f32 columns of tensor memory.  Per 16-wide
// k step two MMAs (cta_group::1, kind::f16):
//   D1 += X . W_hi^T,  D2 += X . W_lo^T,
// with the exact weight halves of the prefill GEMM (prefill_tc.cu): W_hi = (q-8) d_hi 2^8,
// W_lo = (q-8) d_lo 2^16.  Then y[t][r] = 2^-8 D1[t][r] + 2^-16 (D1[64+t][r] + D2[t][r]);
// D2[64+t] (X_lo W_lo, below 2^-18 of a product) is not read.  That is two MMAs per
// 4096 weights, where the prefill GEMM's pair shape at 64 tokens takes six.
//
// Data movement per 64-wide k tile: one 3-D TMA box of the CTA's 16 Q4 tiles (9 KB,
// 4-deep ring), one 16 KB bulk copy of the pre-split, pre-swizzled activation block
// (3-deep ring; written by skinny_tc_x_kernel), and the dequantised W_hi | W_lo (2 x 32 KB,
// 2 stages) that the 16 dequant warps write with stmatrix from the tiles' mma fragment
// layout.  K is split over gridDim.y so that every GEMM covers the SMs; each split writes
// partial[split][token][row] and skinny_reduce_kernel (lmhead.cu) adds the splits in
// order and applies the epilogue.
//
// Warp roles (19 warps): 0-15 dequant (warp j: Q4 row tile j of every k tile), then the
// epilogue; 16 TMEM allocation and the activation copies (lane 0); 17 MMA issue (lane 0);
// 18 the weight boxes (lane 0).  Every mbarrier wait is bounded; a wait that gives up
// sets the device error word and the abort flag, the roles leave their loops, the MMA
// warp commits what it issued, and the epilogue waits for that commit before TMEM is
// released.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace ch {

namespace {
constexpr int kSkRows = 256;                            // weight rows per CTA at most: the MMA's N
constexpr int kSkTiles = kSkRows / 16;                  // Q4 row tiles per CTA at most
constexpr int kSkTok = 64;                              // tokens per launch at most (M = 2 x 64)
constexpr uint32_t kSkXBytes = 2 * kSkTok * 128;        // 16 KB: 128 rows (hi | lo) x 64 k f16
constexpr uint32_t kSkWBytes = kSkRows * 128;           // 32 KB: one of W_hi, W_lo
constexpr uint32_t kSkRawBytes = kSkTiles * kTileBytes; // 9 KB: one TMA box of Q4 tiles
constexpr int kSkWSt = 2, kSkXSt = 3, kSkRaw = 4;       // ring depths
constexpr int kSkEpiWarps = 16, kSkProd = 16, kSkMma = 17, kSkBox = 18;
constexpr int kSkThreads = 19 * 32;
constexpr uint32_t kSkTmemCols = 512;                   // D1: columns 0-255, D2: 256-511
// shared-memory map from a 1024-byte aligned base
constexpr uint32_t kSkOffW = 0;
constexpr uint32_t kSkOffX = kSkOffW + kSkWSt * 2 * kSkWBytes;
constexpr uint32_t kSkOffRaw = kSkOffX + kSkXSt * kSkXBytes;
constexpr uint32_t kSkOffBars = kSkOffRaw + kSkRaw * kSkRawBytes;
constexpr uint32_t kSkNumBars = 2 * kSkWSt + 2 * kSkXSt + 2 * kSkRaw + 1;
constexpr uint32_t kSkOffMisc = kSkOffBars + kSkNumBars * 8;
constexpr size_t kSkSmemBytes = kSkOffMisc + 16 + 1024;  // + alignment slack
static_assert(kSkSmemBytes <= 232448, "shared memory per CTA");
// epilogue exchange of the D1 lo rows, over the W stages once the MMAs are done:
// [4 column groups][2 chunks][64 tokens][33] f32 (row pitch 33: no bank conflicts)
constexpr uint32_t kSkExPitch = 33;
static_assert(4 * 2 * kSkTok * kSkExPitch * 4 <= kSkWSt * 2 * kSkWBytes, "exchange fits the W stages");
// instruction descriptor, kind::f16: D f32, A and B f16, both K-major, N = the CTA's
// weight rows (a multiple of 16, at most 256), M = 128
constexpr uint32_t sk_idesc(uint32_t n_rows) {
  return (1u << 4) | ((n_rows >> 3) << 17) | ((uint32_t)((2 * kSkTok) >> 4) << 24);
}
}  // namespace

CH_DEV void sk_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued so far is complete
CH_DEV void sk_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// the 16 dequant / epilogue warps' own barrier (named barrier 1)
CH_DEV void sk_epi_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kSkEpiWarps * 32) : "memory"); }

struct SkTcArgs {
  const uint8_t *xs;  // [K/64][16 KB] activation blocks (skinny_tc_x_kernel)
  float *partial;     // [splits][B][row_tiles * 16]
  uint32_t row_tiles, K, B, splits;
  uint32_t tpc;       // Q4 row tiles per CTA (the MMA's N / 16, <= 16)
  uint32_t idesc;     // sk_idesc(16 tpc)
  uint32_t *err;
};

// X [B][K] f32 (row stride ldx) -> per k tile a 16 KB block of 128 rows x 64 k f16 in the
// 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)): row t < 64 is token
// t's hi part, row 64 + t its (lo 2^8) part; tokens >= B are zero.
__global__ void skinny_tc_x_kernel(const float *x, uint32_t ldx, uint32_t B, uint32_t K, uint8_t *xs) {
  const uint32_t c8n = K / 8, total = kSkTok * c8n;
  for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const uint32_t n = idx / c8n, c8 = idx % c8n, kt = c8 >> 3, c = c8 & 7;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (n < B) {
      const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)n * ldx + (size_t)c8 * 8);
      const float4 x0 = src[0], x1 = src[1];
      v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w, v[4] = x1.x, v[5] = x1.y, v[6] = x1.z, v[7] = x1.w;
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const __half h0 = __float2half_rn(v[2 * e]), h1 = __float2half_rn(v[2 * e + 1]);
      const __half l0 = __float2half_rn(__fmul_rn(__fsub_rn(v[2 * e], __half2float(h0)), 256.f));
      const __half l1 = __float2half_rn(__fmul_rn(__fsub_rn(v[2 * e + 1], __half2float(h1)), 256.f));
      hi[e] = pack_half2(h0, h1);
      lo[e] = pack_half2(l0, l1);
    }
    uint8_t *blk = xs + (size_t)kt * kSkXBytes;
    const uint32_t rh = n, rl = kSkTok + n;  // rl % 8 == rh % 8
    const uint32_t sw = (c ^ (n & 7)) << 4;
    *reinterpret_cast<uint4 *>(blk + (rh >> 3) * 1024 + (rh & 7) * 128 + sw) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(blk + (rl >> 3) * 1024 + (rl & 7) * 128 + sw) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// grid (row-tile groups of 16, K splits); 19 warps
__global__ void __launch_bounds__(kSkThreads, 1)
    skinny_tc_kernel(const SkTcArgs a, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ uint8_t smem_dyn[];
  const uint32_t dyn = smem_u32(smem_dyn);
  uint8_t *sm = smem_dyn + (((dyn + 1023u) & ~1023u) - dyn);
  const uint32_t sbase = smem_u32(sm);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kSkOffBars);
  uint64_t *wready = bars, *wempty = wready + kSkWSt, *xfull = wempty + kSkWSt, *xempty = xfull + kSkXSt;
  uint64_t *rfull = xempty + kSkXSt, *rempty = rfull + kSkRaw, *dfull = rempty + kSkRaw;
  uint32_t *misc = reinterpret_cast<uint32_t *>(sm + kSkOffMisc);
  uint32_t *tmem_slot = misc;
  volatile uint32_t *abort = misc + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t KT = a.K / 64, split = blockIdx.y;
  const uint32_t k0 = split * KT / a.splits, k1 = (split + 1) * KT / a.splits, nk = k1 - k0;
  const uint32_t rt0 = blockIdx.x * a.tpc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSkWSt; s++) {
      mbar_init(&wready[s], kSkEpiWarps);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < kSkXSt; s++) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int r = 0; r < kSkRaw; r++) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], kSkEpiWarps);
    }
    mbar_init(dfull, 1);
    *abort = 0u;
    fence_mbar_init();
  }
  if (warp == kSkProd) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kSkTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();  // barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kSkProd) {
    if (lane == 0) {
      uint32_t i = 0;
      for (; i < nk; i++) {
        const int s = i % kSkXSt;
        if (i >= (uint32_t)kSkXSt && !tc_wait(&xempty[s], ((i / kSkXSt) - 1) & 1, abort, a.err)) break;
        mbar_arrive_expect_tx(&xfull[s], kSkXBytes);
        bulk_g2s(sm + kSkOffX + s * kSkXBytes, a.xs + (size_t)(k0 + i) * kSkXBytes, kSkXBytes, &xfull[s]);
      }
      // the last copies land before the CTA may leave (normally long done)
      for (uint32_t j = i > (uint32_t)kSkXSt ? i - kSkXSt : 0; j < i; j++)
        tc_wait(&xfull[j % kSkXSt], (j / kSkXSt) & 1, nullptr, a.err);
    }
  } else if (warp == kSkBox) {
    if (lane == 0) {
      uint32_t i = 0;
      for (; i < nk; i++) {
        const int r = i % kSkRaw;
        if (i >= (uint32_t)kSkRaw && !tc_wait(&rempty[r], ((i / kSkRaw) - 1) & 1, abort, a.err)) break;
        // the box always lands whole (row tiles past the matrix read as zeros)
        mbar_arrive_expect_tx(&rfull[r], a.tpc * kTileBytes);
        tma_load_3d(sm + kSkOffRaw + r * kSkRawBytes, &wmap, 0, (int)(k0 + i), (int)rt0, &rfull[r]);
      }
      for (uint32_t j = i > (uint32_t)kSkRaw ? i - kSkRaw : 0; j < i; j++)
        tc_wait(&rfull[j % kSkRaw], (j / kSkRaw) & 1, nullptr, a.err);
    }
  } else if (warp == kSkMma) {
    if (lane == 0) {
      for (uint32_t i = 0; i < nk; i++) {
        const int s = i % kSkWSt, xsl = i % kSkXSt;
        if (!tc_wait(&wready[s], (i / kSkWSt) & 1, abort, a.err)) break;
        if (!tc_wait(&xfull[xsl], (i / kSkXSt) & 1, abort, a.err)) break;
        tc_fence_after();
        const uint64_t xd = umma_desc_sw128(sbase + kSkOffX + xsl * kSkXBytes);
        const uint64_t wh = umma_desc_sw128(sbase + kSkOffW + s * 2 * kSkWBytes);
        const uint64_t wl = umma_desc_sw128(sbase + kSkOffW + s * 2 * kSkWBytes + kSkWBytes);
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ko = (uint64_t)(ks * 2);  // 32 B per 16-wide k step, in 16-byte units
          const uint32_t acc = (i | ks) != 0;
          sk_mma(tmem, xd + ko, wh + ko, a.idesc, acc);                 // D1 += X W_hi^T
          sk_mma(tmem + (uint32_t)kSkRows, xd + ko, wl + ko, a.idesc, acc);  // D2 += X W_lo^T
        }
        sk_commit(&wempty[s]);
        sk_commit(&xempty[xsl]);
      }
      sk_commit(dfull);  // every MMA issued (all of them, or those before an abort) is complete
    }
  } else {
    // dequant: warp j expands Q4 row tile j of each k tile into W_hi and W_lo (rows
    // 16j..16j+15), one stmatrix.x4 per operand and word, as in prefill_tc.cu
    const uint32_t j = warp, g = lane >> 2, mi = lane >> 3, rr = lane & 7;
    for (uint32_t i = 0; i < nk; i++) {
      const int s = i % kSkWSt, r = i % kSkRaw;
      if (!__all_sync(0xFFFFFFFFu, tc_wait(&rfull[r], (i / kSkRaw) & 1, abort, a.err))) break;
      if (i >= (uint32_t)kSkWSt &&
          !__all_sync(0xFFFFFFFFu, tc_wait(&wempty[s], ((i / kSkWSt) - 1) & 1, abort, a.err)))
        break;
      const uint32_t Wh = sbase + kSkOffW + s * 2 * kSkWBytes, Wl = Wh + kSkWBytes;
      if (j < a.tpc) {  // warps past the CTA's row tiles only take part in the barriers
        const uint8_t *raw = sm + kSkOffRaw + r * kSkRawBytes + j * kTileBytes;
        const uint4 w = *reinterpret_cast<const uint4 *>(raw + lane * 16);
        const uint2 sc = *reinterpret_cast<const uint2 *>(raw + 512 + g * 8);  // rows g, g+8: (blk0 | blk1 << 16)
        uint32_t hs[2][2], ls[2][2];                                          // [row g / g+8][blk]
        bool ok = split_scale(sc.x & 0xFFFFu, hs[0][0], ls[0][0]);
        ok &= split_scale(sc.x >> 16, hs[0][1], ls[0][1]);
        ok &= split_scale(sc.y & 0xFFFFu, hs[1][0], ls[1][0]);
        ok &= split_scale(sc.y >> 16, hs[1][1], ls[1][1]);
        if (!ok) atomicOr(a.err, DEV_ERR_SCALE_RANGE);
        const uint32_t rbase = (2 * j + (mi & 1)) * 1024 + rr * 128;
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};  // (blk, ch) = (0,0) (0,1) (1,0) (1,1)
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
          const int blk = wi >> 1;
          uint32_t f[4];
          dequant_q4_word(ws[wi], f);
          const uint32_t chunk = blk * 4 + (wi & 1) * 2 + (mi >> 1);
          const uint32_t off = rbase + ((chunk ^ rr) << 4);
          stmatrix_x4(Wh + off, hmul2_u32(f[0], hs[0][blk]), hmul2_u32(f[1], hs[1][blk]), hmul2_u32(f[2], hs[0][blk]),
                      hmul2_u32(f[3], hs[1][blk]));
          stmatrix_x4(Wl + off, hmul2_u32(f[0], ls[0][blk]), hmul2_u32(f[1], ls[1][blk]), hmul2_u32(f[2], ls[0][blk]),
                      hmul2_u32(f[3], ls[1][blk]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[r]);  // the box is read
      fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&wready[s]);
    }

    // epilogue: quads 2-3 (TMEM lanes 64-127: the lo rows) hand D1's lo rows over through
    // shared memory; quads 0-1 (lanes 0-63: the hi rows) combine and store.  Column
    // group cg = warp / 4 covers weight rows 64 cg .. 64 cg + 63 in two chunks of 32.
    const uint32_t quad = warp & 3, cg = warp >> 2, t = (quad & 1) * 32 + lane;
    const bool done = __all_sync(0xFFFFFFFFu, tc_wait(dfull, 0, nullptr, a.err));
    tc_fence_after();
    const bool ok = __all_sync(0xFFFFFFFFu, done && !*abort);
    float *ex = reinterpret_cast<float *>(sm + kSkOffW);
    if (ok && quad >= 2) {
#pragma unroll 1
      for (int ch = 0; ch < 2; ch++) {
        uint32_t v[32];
        tc_ld32(tmem + ((quad * 32u) << 16) + cg * 64 + ch * 32, v);
        tc_wait_ld();
        float *row = ex + ((size_t)(cg * 2 + ch) * kSkTok + t) * kSkExPitch;
#pragma unroll
        for (int i = 0; i < 32; i++) row[i] = __uint_as_float(v[i]);
      }
    }
    sk_epi_sync();
    if (ok && quad < 2) {
      const size_t R16 = (size_t)a.row_tiles * 16;
      float *pr = a.partial + ((size_t)split * a.B + t) * R16;
#pragma unroll 1
      for (int ch = 0; ch < 2; ch++) {
        const uint32_t col = cg * 64 + ch * 32;
        uint32_t v1[32], v2[32];
        tc_ld32(tmem + ((quad * 32u) << 16) + col, v1);
        tc_ld32(tmem + ((quad * 32u) << 16) + (uint32_t)kSkRows + col, v2);
        tc_wait_ld();
        const float *row = ex + ((size_t)(cg * 2 + ch) * kSkTok + t) * kSkExPitch;
        const uint32_t r0 = rt0 * 16 + col;
        const uint32_t rend = min((uint32_t)R16, (rt0 + a.tpc) * 16);  // this CTA's rows
        if (t < a.B) {
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const float corr = __fadd_rn(row[i], __uint_as_float(v2[i]));
            y[i] = __fmaf_rn(corr, 1.0f / 65536.f, __fmul_rn(__uint_as_float(v1[i]), 1.0f / 256.f));
          }
          if (r0 + 32 <= rend) {  // whole chunk: 16-byte stores (rend and r0 are multiples of 16)
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4 *>(pr + r0 + i) = make_float4(y[i], y[i + 1], y[i + 2], y[i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (r0 + i < rend) pr[r0 + i] = y[i];
          }
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();  // every role done with TMEM
  if (warp == kSkProd) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kSkTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// The end of a row-parallel projection (o, down) of the multi-stream step, one token per
// CTA: v = the K splits' partials added in split order (as skinny_reduce_kernel), then
// with the operations and order of rmsnorm_rows_vec_kernel and add_rmsnorm_rows_vec_kernel
// (prefill.cu): v = rmsnorm(v) * post_w (when given), x = (x + v) * scalar,
// y = rmsnorm(x) * next_w; and, when xs is given, y's hi / lo blocks for the next skinny
// GEMM (as skinny_tc_x_kernel).  Rows of H <= 4096 floats, H % 64 == 0.
constexpr int kTailThreads = 256, kTailVec = 4;
__global__ void __launch_bounds__(kTailThreads)
    skinny_tail_kernel(const float *partial, uint32_t splits, uint32_t B, uint32_t H, const float *post_w, float *x,
                       const float *next_w, float *y, float eps, float scalar, uint8_t *xs) {
  __shared__ float red[32];
  const uint32_t t = blockIdx.x, n4 = H / 4, tid = threadIdx.x;
  float4 v[kTailVec];
  auto part = [&](uint32_t sp, int k) {  // split sp's float4 k of this thread (zeros past the row)
    const uint32_t j = tid + k * kTailThreads;
    return j < n4 ? *(reinterpret_cast<const float4 *>(partial + ((size_t)sp * B + t) * H) + j)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
  };
#pragma unroll
  for (int k = 0; k < kTailVec; k++) v[k] = part(0, k);
  // splits in order; the loads of several splits are in flight before their additions
#pragma unroll 3
  for (uint32_t sp = 1; sp < splits; sp++) {
    float4 b[kTailVec];
#pragma unroll
    for (int k = 0; k < kTailVec; k++) b[k] = part(sp, k);
#pragma unroll
    for (int k = 0; k < kTailVec; k++)
      v[k] = make_float4(__fadd_rn(v[k].x, b[k].x), __fadd_rn(v[k].y, b[k].y), __fadd_rn(v[k].z, b[k].z),
                         __fadd_rn(v[k].w, b[k].w));
  }
  auto sumsq = [&](const float4 (&u)[kTailVec]) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kTailVec; k++) {
      ss = __fmaf_rn(u[k].x, u[k].x, ss);
      ss = __fmaf_rn(u[k].y, u[k].y, ss);
      ss = __fmaf_rn(u[k].z, u[k].z, ss);
      ss = __fmaf_rn(u[k].w, u[k].w, ss);
    }
    const float tot = block_sum(ss, red);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
  };
  if (post_w) {
    const float inv = sumsq(v);
#pragma unroll
    for (int k = 0; k < kTailVec; k++) {
      const uint32_t j = tid + k * kTailThreads;
      if (j < n4) {
        const float4 g = reinterpret_cast<const float4 *>(post_w)[j];
        v[k] = make_float4(__fmul_rn(__fmul_rn(v[k].x, inv), g.x), __fmul_rn(__fmul_rn(v[k].y, inv), g.y),
                           __fmul_rn(__fmul_rn(v[k].z, inv), g.z), __fmul_rn(__fmul_rn(v[k].w, inv), g.w));
      }
    }
  }
  float4 *xr = reinterpret_cast<float4 *>(x + (size_t)t * H);
#pragma unroll
  for (int k = 0; k < kTailVec; k++) {
    const uint32_t j = tid + k * kTailThreads;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (j < n4) a = xr[j], b = v[k];
    v[k] = make_float4(__fmul_rn(__fadd_rn(a.x, b.x), scalar), __fmul_rn(__fadd_rn(a.y, b.y), scalar),
                       __fmul_rn(__fadd_rn(a.z, b.z), scalar), __fmul_rn(__fadd_rn(a.w, b.w), scalar));
    if (j < n4) xr[j] = v[k];
  }
  const float inv = sumsq(v);
  float4 *yr = reinterpret_cast<float4 *>(y + (size_t)t * H);
#pragma unroll
  for (int k = 0; k < kTailVec; k++) {
    const uint32_t j = tid + k * kTailThreads;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < n4) {
      const float4 g = reinterpret_cast<const float4 *>(next_w)[j];
      o = make_float4(__fmul_rn(__fmul_rn(v[k].x, inv), g.x), __fmul_rn(__fmul_rn(v[k].y, inv), g.y),
                      __fmul_rn(__fmul_rn(v[k].z, inv), g.z), __fmul_rn(__fmul_rn(v[k].w, inv), g.w));
      yr[j] = o;
    }
    if (xs) {  // even thread: its float4 and its neighbour's are one 8-wide chunk (n4 is even)
      const float4 nb = make_float4(__shfl_down_sync(0xFFFFFFFFu, o.x, 1), __shfl_down_sync(0xFFFFFFFFu, o.y, 1),
                                    __shfl_down_sync(0xFFFFFFFFu, o.z, 1), __shfl_down_sync(0xFFFFFFFFu, o.w, 1));
      if (!(tid & 1) && j < n4) {
        const float e8[8] = {o.x, o.y, o.z, o.w, nb.x, nb.y, nb.z, nb.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const __half h0 = __float2half_rn(e8[2 * e]), h1 = __float2half_rn(e8[2 * e + 1]);
          const __half l0 = __float2half_rn(__fmul_rn(__fsub_rn(e8[2 * e], __half2float(h0)), 256.f));
          const __half l1 = __float2half_rn(__fmul_rn(__fsub_rn(e8[2 * e + 1], __half2float(h1)), 256.f));
          hi[e] = pack_half2(h0, h1);
          lo[e] = pack_half2(l0, l1);
        }
        const uint32_t c8 = j >> 1, kt = c8 >> 3, c = c8 & 7;
        uint8_t *blk = xs + (size_t)kt * kSkXBytes;
        const uint32_t rh = t, rl = kSkTok + t, sw = (c ^ (t & 7)) << 4;
        *reinterpret_cast<uint4 *>(blk + (rh >> 3) * 1024 + (rh & 7) * 128 + sw) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(blk + (rl >> 3) * 1024 + (rl & 7) * 128 + sw) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
  }
}

cudaError_t launch_skinny_tail(const float *partial, uint32_t splits, uint32_t B, uint32_t H, const float *post_w,
                               float *x, const float *next_w, float *y, float eps, float scalar, uint8_t *xs,
                               cudaStream_t s) {
  if (B == 0 || B > (uint32_t)kSkTok || splits == 0 || H % 64 || H > 4u * kTailVec * kTailThreads)
    return cudaErrorInvalidValue;
  if (((uintptr_t)partial | (uintptr_t)x | (uintptr_t)next_w | (uintptr_t)y | (uintptr_t)post_w | (uintptr_t)xs) & 15)
    return cudaErrorInvalidValue;
  skinny_tail_kernel<<<B, kTailThreads, 0, s>>>(partial, splits, B, H, post_w, x, next_w, y, eps, scalar, xs);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Row tiles per CTA: 16 (N = 256), or fewer when 12-15 per SM cover the rows in one wave
// (an MMA costs about the same at N = 208 as at 256, so the idle SMs of 16-tile groups
// would be lost: 1,920 row tiles make 148 CTAs of 13 instead of 120 of 16).  K splits:
// as many CTAs as fit the SMs in one wave (the rows alone give too few for o and down),
// at most one per k tile.
static uint32_t skinny_tc_tpc(uint32_t row_tiles) {
  const uint32_t sms = (uint32_t)num_sms(), per_sm = (row_tiles + sms - 1) / sms;
  return per_sm >= 12 && per_sm < (uint32_t)kSkTiles ? per_sm : (uint32_t)kSkTiles;
}
uint32_t skinny_tc_splits(uint32_t row_tiles, uint32_t K) {
  const uint32_t tpc = skinny_tc_tpc(row_tiles), ctas = (row_tiles + tpc - 1) / tpc;
  return std::max(1u, std::min((uint32_t)num_sms() / std::max(1u, ctas), K / 64));
}
size_t skinny_tc_x_bytes(uint32_t K) { return (size_t)(K / 64) * kSkXBytes; }
size_t skinny_tc_partial_floats(uint32_t B, uint32_t row_tiles, uint32_t K) {
  return (size_t)skinny_tc_splits(row_tiles, K) * B * row_tiles * 16;
}

// tensor maps of the weight matrices, encoded once per (tiles, rows, K, box rows)
static cudaError_t tile_map_cached(const uint8_t *tiles, uint32_t M, uint32_t K, uint32_t box, CUtensorMap *out) {
  struct Key {
    const uint8_t *p;
    uint32_t M, K, box;
    bool operator==(const Key &o) const { return p == o.p && M == o.M && K == o.K && box == o.box; }
  };
  struct Hash {
    size_t operator()(const Key &k) const {
      return std::hash<const void *>()(k.p) ^ ((size_t)k.M * 0x9E3779B97F4A7C15ull) ^ ((size_t)k.K << 1) ^
             ((size_t)k.box << 40);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  std::lock_guard<std::mutex> lock(mu);
  const Key key{tiles, M, K, box};
  auto it = cache.find(key);
  if (it != cache.end()) {
    std::memcpy(out, &it->second, sizeof(CUtensorMap));
    return cudaSuccess;
  }
  alignas(64) CUtensorMap m;
  cudaError_t e = encode_tile_map(&m, tiles, M, K, box);
  if (e != cudaSuccess) return e;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  std::memcpy(out, &m, sizeof(CUtensorMap));
  return cudaSuccess;
}

// partial[split][B][row_tiles * 16] = the K split's share of W x for B <= 64 tokens;
// xs scratch: skinny_tc_x_bytes(K), 16-byte aligned.  x_ready: xs already holds x's
// blocks (written by skinny_tail_kernel), x is not read.
cudaError_t launch_skinny_q4_tc(const uint8_t *tiles, uint32_t row_tiles, uint32_t K, const float *x, uint32_t ldx,
                                uint32_t B, uint8_t *xs, float *partial, uint32_t *err, uint32_t *splits,
                                cudaStream_t s, bool x_ready) {
  if (B == 0 || B > (uint32_t)kSkTok || K % 64 || row_tiles == 0 || ((uintptr_t)xs & 15) || ((uintptr_t)tiles & 15))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  if (!x_ready) {
    if (ldx % 4 || ((uintptr_t)x & 15)) return cudaErrorInvalidValue;
    const uint32_t total = kSkTok * (K / 8);
    skinny_tc_x_kernel<<<std::min<uint32_t>((total + 255) / 256, (uint32_t)num_sms() * 8), 256, 0, s>>>(x, ldx, B,
                                                                                                          K, xs);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const uint32_t tpc = skinny_tc_tpc(row_tiles);
  alignas(64) CUtensorMap wmap;
  e = tile_map_cached(tiles, row_tiles * 16, K, tpc, &wmap);
  if (e != cudaSuccess) return e;
  SkTcArgs a{};
  a.tpc = tpc;
  a.idesc = sk_idesc(16 * tpc);
  a.xs = xs;
  a.partial = partial;
  a.row_tiles = row_tiles;
  a.K = K;
  a.B = B;
  a.splits = skinny_tc_splits(row_tiles, K);
  a.err = err;
  *splits = a.splits;
  e = cudaFuncSetAttribute(skinny_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSkSmemBytes);
  if (e != cudaSuccess) return e;
  const dim3 grid((row_tiles + tpc - 1) / tpc, a.splits);
  skinny_tc_kernel<<<grid, kSkThreads, kSkSmemBytes, s>>>(a, wmap);
  return cudaGetLastError();
}

}  // namespace ch
