// prefill_tc.cu -- the batched prefill GEMM on the 5th-generation tensor cores.
//
// Restated reference shaders:
//   batch_gemm_q4.wgsl:26-160       Y[t*M + r] = sum_b d_rb sum_i (q_rbi - 8) X[t][32b+i]
//   batch_fused_mlp_q4.wgsl:33-196  Y[t*M/2 + r] = gelu_tanh(gate_r . x_t) * (up_r . x_t)
//
// A pair of CTAs (a cluster of 2 on two SMs) computes a tile of 256 weight rows x
// 256 tokens with tcgen05.mma.cta_group::2 (kind::f16, M=256, N=256, f32
// accumulators in tensor memory): each CTA holds 128 rows of the weight operand and
// 128 tokens of the activation operand and receives the 128 x 256 accumulators of
// its own rows.  M=256 x N=256 is the largest tcgen05 shape: an MMA instruction
// takes about the same time at any smaller shape.
//
// Numerics (fp32-faithful; the shaders' up to the order of the additions):
//   * the weight w = (q-8) d of a 32-block enters as two exact f16 operands:
//     d = d_hi + d_lo with d_hi = d's top 8 significant bits and d_lo the rest
//     (at most 3 bits), A_hi = (q-8) d_hi 2^8 and A_lo = (q-8) d_lo 2^16 -- both
//     products fit an f16 significand, so the dequantised weights are exact;
//   * the activation enters as an f16 pair hi + lo (x = hi + lo to 2^-22), the lo
//     part stored as lo 2^8;
//   * per 16-wide k step three MMAs: D1 += A_hi X_hi (scale 2^-8) and the two
//     correction terms D2 += A_hi (X_lo 2^8), D2 += A_lo X_hi (scale 2^-16), so
//     that the small terms are summed among themselves and not rounded away
//     against the main sum; Y = 2^-8 D1 + 2^-16 D2.  The one term left out,
//     A_lo X_lo, is below 2^-18 of each product.
//   Scales are assumed |d| < 16 (checked; the device error word flags others).
//
// Per 64-wide k tile each CTA takes two copy requests -- one 3-D TMA box of its 8
// Q4 tiles (576 B each, at a stride of K/64 tiles in the row-tile-major layout)
// and one 32 KB bulk copy of its activation share, pre-split and pre-swizzled by
// tc_split_x_kernel -- because the copy engine takes tens of cycles per request.
//
// Warp roles (19 warps per CTA):
//   0-15  during the k loop, dequant: warp w expands Q4 tile w % 8 of the even
//         (w < 8) or odd k tiles -- nibbles and scales (staged by TMA) -> A_hi,
//         A_lo, stored by stmatrix straight from the mma fragment layout of the Q4
//         tiles; two k tiles are dequantised at a time.  After the k loop, the
//         epilogue: warp w reads TMEM lanes 32*(w%4).. (a warp may touch only its
//         quarter of the lanes) and token columns 64*(w/4)..+63 of both
//         accumulators, and stores Y (or a split-K partial)
//   16    producer: TMEM allocation (whole warp, both CTAs); the activation copies
//         (lane 0)
//   17    MMA issuer (lane 0 of the pair's leader CTA, rank 0)
//   18    weight producer: the Q4 tile boxes (lane 0)
// Barriers: a 3-deep stage ring of A_hi | A_lo | X (xfull: activation copy bytes,
// per CTA; aready: one arrival per dequant warp of the k tile in both CTAs, at the
// leader, once its A tile is written and its CTA's activation share has landed;
// empty: tcgen05.commit multicast to both), a 5-deep ring of Q4 tile boxes (rfull:
// copy bytes; rempty: one arrival per dequant warp of the k tile once read), and
// dfull (commit multicast after the last k tile).  The weight boxes run ahead of
// the stages, so the dequant of a k tile overlaps the copy of its activation share.
// Arrivals at the leader's barriers are release.cluster and its waits on them
// acquire.cluster.  Every wait is bounded: a wait that gives up sets the device
// error word and the CTA's abort flag; the roles then leave their loops, the MMAs
// in flight are waited for (bounded), both CTAs meet at a cluster barrier and TMEM
// is released.
//
// Split-K (when the rows give too few tile pairs for the SMs): the k tiles are
// divided among SK pairs per output tile; each writes its partial to a workspace
// and the last to finish (an atomic counter per tile) adds the SK partials in split
// order -- the same order on every run -- and applies the epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace ch {
namespace {
constexpr int kTcBM = 128, kTcBN = 256, kTcBK = 64;      // per CTA: 128 rows; per pair: 256 tokens
constexpr int kTcHalfN = kTcBN / 2;                       // tokens of the activation operand per CTA
constexpr int kTcStages = 3;  // A_hi | A_lo | X stages (what the MMAs read)
constexpr int kTcRaw = 5;     // Q4 tile boxes (what the dequant reads), a deeper ring
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;        // 16 KB: 128 rows x 128 B (one of A_hi, A_lo)
constexpr uint32_t kTcPlane = kTcHalfN * kTcBK * 2;      // 16 KB: one f16 plane of 128 tokens
constexpr uint32_t kTcXBytes = 2 * kTcPlane;             // this CTA's share: hi plane, lo plane
constexpr uint32_t kTcRawBytes = 8 * kTileBytes;         // 8 whole Q4 tiles (nibbles + scales): one TMA box
constexpr uint32_t kTcStageBytes = 2 * kTcABytes + kTcXBytes;  // 64 KB: A_hi | A_lo | X_hi | X_lo
constexpr int kEpiWarps = 16;              // dequant during the k loop, epilogue after it
constexpr int kDqPerTile = kEpiWarps / 2;  // warps per k tile: one Q4 tile each; even/odd k tiles alternate
constexpr int kProdWarp = kEpiWarps, kMmaWarp = kProdWarp + 1, kRawWarp = kMmaWarp + 1;
constexpr int kTcThreads = (kRawWarp + 1) * 32;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr uint32_t kTmemCols = 512;  // D1: columns 0-255, D2: 256-511
constexpr uint32_t kCounterBytes = 16384;
constexpr uint32_t kMaxCounters = kCounterBytes / 4;

// shared-memory map, offsets from a 1024-byte aligned base (the swizzle atoms of
// the A and X tiles start on 1024-byte boundaries); identical in both CTAs
constexpr uint32_t kOffRaw = kTcStages * kTcStageBytes;
constexpr uint32_t kOffBars = kOffRaw + kTcRaw * kTcRawBytes;
constexpr uint32_t kNumBars = 3 * kTcStages + 1 + 2 * kTcRaw;
constexpr uint32_t kOffMisc = kOffBars + kNumBars * 8;
constexpr uint32_t kTcSmemUsed = kOffMisc + 16;
static_assert(kTcStageBytes % 1024 == 0, "stage alignment");
static_assert(kTcRawBytes % 128 == 0, "TMA destination alignment");
}  // namespace
constexpr size_t kTcSmemBytes = kTcSmemUsed + 1024;  // + alignment slack
static_assert(kTcSmemBytes <= 232448, "shared memory per CTA");

// Optional pipeline timeline (trace build, -DCH_PHASE_TRACE): one role thread of the
// leader CTA of pair 1 (token tile 0, split 0) records clock64 at each event:
// 0 activation copy issued, 1 dequant began the k tile (box landed, A slot free),
// 2 dequant published the A tiles, 3 MMA started the k tile, 4 MMA issued the k
// tile, 5 epilogue saw the accumulators complete, 6 epilogue done (warp 0),
// 7 dequant loaded its words and scales, 8 dequant stores issued, 9 box issued.
#ifdef CH_PHASE_TRACE
constexpr int kTcTraceKinds = 10, kTcTraceLen = 1024;
__device__ long long g_tc_trace[kTcTraceKinds * kTcTraceLen];
#define TC_MARK(kind, idx)                                                                     \
  do {                                                                                         \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 1 && (idx) < (uint32_t)kTcTraceLen) \
      g_tc_trace[(kind) * kTcTraceLen + (idx)] = clock64();                                    \
  } while (0)
#else
#define TC_MARK(kind, idx) \
  do {                     \
  } while (0)
#endif

// ---------------------------------------------------------------------------
// tcgen05 primitives of this kernel (the shared ones are in tcgen05.cuh)

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B f16 (0), both
// K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28; M = 256
// across the CTA pair.
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcBN >> 3) << 17) | ((uint32_t)((2 * kTcBM) >> 4) << 24);

// D[tmem] (+)= A[adesc] * B[bdesc]^T over the CTA pair (issued by the leader)
CH_DEV void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (same offset) in both CTAs of the pair once every tcgen05
// operation this thread issued so far is complete
CH_DEV void tc_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)3)
      : "memory");
}
// the epilogue warps' own barrier (named barrier 1, 512 threads)
CH_DEV void epi_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory"); }

// ---------------------------------------------------------------------------
// X [N][K] f32 -> per (256-token tile, k tile) block of 64 KB made of two 32 KB
// halves (tokens 0-127, 128-255: the share of CTA rank 0 and 1), each the f16 hi
// plane then the (lo 2^8) plane of 128 token rows x 64 k in the 128-byte swizzle (16-byte
// chunk c of row r stored at chunk c ^ (r % 8)).  Token rows >= N are zero.
__global__ void tc_split_x_kernel(const float *X, uint32_t N, uint32_t K, uint32_t ntok, uint8_t *xs) {
  const uint32_t KT = K / 64, c8n = K / 8;
  const uint64_t total = (uint64_t)ntok * c8n;
  for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t n = (uint32_t)(idx / c8n), c8 = (uint32_t)(idx % c8n);
    const uint32_t kt = c8 >> 3, c = c8 & 7, nt = n >> 8, h = (n >> 7) & 1, r = n & 127;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (n < N) {
      const float4 *src = reinterpret_cast<const float4 *>(X + (size_t)n * K + (size_t)c8 * 8);
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
    uint8_t *blk = xs + (((size_t)nt * KT + kt) * 2 + h) * kTcXBytes;
    const uint32_t off = (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
    *reinterpret_cast<uint4 *>(blk + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(blk + kTcPlane + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// ---------------------------------------------------------------------------
struct TcLaunch {
  uint32_t sk;         // split-K factor (k tiles per split = KT / sk)
  uint32_t nt_tiles;   // 256-token tiles
  uint32_t *counters;  // split-K: one per CTA tile, zero between launches
  float *ws;           // split-K partials [sk][nt_tiles*256][M]
};

// grid (2, token tiles, row pairs x splits), clusters of 2 along x: blockIdx.x = rank
template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    batch_gemm_tc_kernel(const TcGemmArgs a, const TcLaunch L, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ uint8_t smem_dyn[];
  const uint32_t dyn = smem_u32(smem_dyn);
  uint8_t *sm = smem_dyn + (((dyn + 1023u) & ~1023u) - dyn);
  const uint32_t sbase = smem_u32(sm);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kOffBars);
  uint64_t *xfull = bars, *aready = bars + kTcStages, *empty = bars + 2 * kTcStages, *dfull = bars + 3 * kTcStages;
  uint64_t *rfull = dfull + 1, *rempty = rfull + kTcRaw;
  uint32_t *misc = reinterpret_cast<uint32_t *>(sm + kOffMisc);
  uint32_t *tmem_slot = misc;
  volatile uint32_t *abort = misc + 1;
  volatile uint32_t *is_last = misc + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t KT = a.K / kTcBK, KTS = KT / L.sk;
  const uint32_t nt = blockIdx.y, mp = blockIdx.z / L.sk, sk = blockIdx.z % L.sk;
  const uint32_t kt0 = sk * KTS;
  const uint32_t rt0 = (mp * 2 + rank) * 8;
  const uint32_t row_tiles = a.M / 16;
  const uint32_t ntiles = rt0 < row_tiles ? min(8u, row_tiles - rt0) : 0u;  // Q4 row tiles of this CTA
  const uint32_t ready_l = map_shared(smem_u32(aready), 0);  // the leader's aready, as a cluster address

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; s++) {
      mbar_init(&xfull[s], 1);
      mbar_init(&aready[s], 2 * kDqPerTile);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < kTcRaw; r++) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], kDqPerTile);
    }
    mbar_init(dfull, 1);
    *abort = 0u;
    fence_mbar_init();
  }
  if (warp == kProdWarp) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    if (lane == 0) {
      const uint8_t *xs = a.xs + ((size_t)nt * KT * 2 + rank) * kTcXBytes;  // + kt * 2 * kTcXBytes
      uint32_t i = 0;
      for (; i < KTS; i++) {
        const int s = i % kTcStages;
        if (i >= (uint32_t)kTcStages && !tc_wait(&empty[s], ((i / kTcStages) - 1) & 1, abort, a.err)) break;
        mbar_arrive_expect_tx(&xfull[s], kTcXBytes);
        bulk_g2s(sm + s * kTcStageBytes + 2 * kTcABytes, xs + (size_t)(kt0 + i) * 2 * kTcXBytes, kTcXBytes, &xfull[s]);
        TC_MARK(0, i);
      }
      // the copies of the last issues land before the CTA may leave (normally long done)
      for (uint32_t j = i > (uint32_t)kTcStages ? i - kTcStages : 0; j < i; j++)
        tc_wait(&xfull[j % kTcStages], (j / kTcStages) & 1, nullptr, a.err);
    }
  } else if (warp == kRawWarp) {
    if (lane == 0) {
      uint32_t i = 0;
      for (; i < KTS; i++) {
        const int r = i % kTcRaw;
        if (i >= (uint32_t)kTcRaw && !tc_wait(&rempty[r], ((i / kTcRaw) - 1) & 1, abort, a.err)) break;
        // the TMA box always lands whole (rows past M read as zeros)
        mbar_arrive_expect_tx(&rfull[r], kTcRawBytes);
        tma_load_3d(sm + kOffRaw + r * kTcRawBytes, &wmap, 0, (int)(kt0 + i), (int)rt0, &rfull[r]);
        TC_MARK(9, i);
      }
      for (uint32_t j = i > (uint32_t)kTcRaw ? i - kTcRaw : 0; j < i; j++)
        tc_wait(&rfull[j % kTcRaw], (j / kTcRaw) & 1, nullptr, a.err);
    }
  } else if (warp == kMmaWarp) {
    if (leader && lane == 0) {
      bool issued = false;
      for (uint32_t i = 0; i < KTS; i++) {
        const int s = i % kTcStages;
        // both CTAs' A tiles written and activation shares landed
        if (!tc_wait(&aready[s], (i / kTcStages) & 1, abort, a.err, true)) break;
        tc_fence_after();
        TC_MARK(3, i);
        const uint32_t st = sbase + s * kTcStageBytes;
        const uint64_t ah = umma_desc_sw128(st), al = umma_desc_sw128(st + kTcABytes);
        const uint64_t xh = umma_desc_sw128(st + 2 * kTcABytes), xl = umma_desc_sw128(st + 2 * kTcABytes + kTcPlane);
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ko = (uint64_t)(ks * 2);  // 32 B per 16-wide k step, in 16-byte units
          const uint32_t acc = (i | ks) != 0;
          tc_mma(tmem, ah + ko, xh + ko, acc);          // D1 += A_hi X_hi
          tc_mma(tmem + kTcBN, ah + ko, xl + ko, acc);  // D2 += A_hi (X_lo 2^8)
          tc_mma(tmem + kTcBN, al + ko, xh + ko, 1u);   // D2 += A_lo X_hi
        }
        issued = true;
        tc_commit_pair(&empty[s]);
        TC_MARK(4, i);
      }
      // the accumulators are complete (or, after an abort, every MMA issued is)
      if (issued) tc_commit_pair(dfull);
    }
  } else if (warp < kEpiWarps) {
    // dequant.  A Q4 tile's 32 lanes hold an mma fragment -- lane (g, t4) has rows
    // g, g+8 at k = 2 t4, 2 t4 + 1 (+8) of each 16-wide k chunk -- so each
    // dequantised word is one stmatrix.x4 (four 8x8 f16 blocks) per operand, with
    // the row addresses in the 128-byte swizzle.
    const uint32_t j = warp % kDqPerTile, par = warp / kDqPerTile;
    const uint32_t g = lane >> 2, mi = lane >> 3, rr = lane & 7;
    const bool mark = j == 0 && lane == 0;
    for (uint32_t i = par; i < KTS; i += 2) {
      const int s = i % kTcStages, r = i % kTcRaw;
      // warp-uniform waits: the Q4 box landed, and the A slot's previous MMAs are done
      if (!__all_sync(0xFFFFFFFFu, tc_wait(&rfull[r], (i / kTcRaw) & 1, abort, a.err))) break;
      if (i >= (uint32_t)kTcStages &&
          !__all_sync(0xFFFFFFFFu, tc_wait(&empty[s], ((i / kTcStages) - 1) & 1, abort, a.err)))
        break;
      if (mark) TC_MARK(1, i);
      const uint32_t Ah = sbase + s * kTcStageBytes, Al = Ah + kTcABytes;
      if (j < ntiles) {
        const uint8_t *raw = sm + kOffRaw + r * kTcRawBytes + j * kTileBytes;
        const uint4 w = *reinterpret_cast<const uint4 *>(raw + lane * 16);
        const uint2 sc = *reinterpret_cast<const uint2 *>(raw + 512 + g * 8);  // rows g, g+8: (blk0 | blk1 << 16)
        if (mark && (w.x | sc.x) != 0xFFFFFFFFu) TC_MARK(7, i);
        uint32_t hs[2][2], ls[2][2];  // [row g / g+8][blk]
        bool ok = split_scale(sc.x & 0xFFFFu, hs[0][0], ls[0][0]);
        ok &= split_scale(sc.x >> 16, hs[0][1], ls[0][1]);
        ok &= split_scale(sc.y & 0xFFFFu, hs[1][0], ls[1][0]);
        ok &= split_scale(sc.y >> 16, hs[1][1], ls[1][1]);
        if (!ok) atomicOr(a.err, DEV_ERR_SCALE_RANGE);
        // this lane's stmatrix row address: block mi (rows +8 if mi & 1, k +8 if mi & 2), row rr
        const uint32_t rbase = (2 * j + (mi & 1)) * 1024 + rr * 128;
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};  // (blk, ch) = (0,0) (0,1) (1,0) (1,1)
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
          const int blk = wi >> 1;
          uint32_t f[4];
          dequant_q4_word(ws[wi], f);  // exact q-8 pairs: (g, k) (g+8, k) (g, k+8) (g+8, k+8), k = kb + 2 t4
          const uint32_t chunk = blk * 4 + (wi & 1) * 2 + (mi >> 1);  // 16-byte chunk of this lane's row
          const uint32_t off = rbase + ((chunk ^ rr) << 4);
          stmatrix_x4(Ah + off, hmul2_u32(f[0], hs[0][blk]), hmul2_u32(f[1], hs[1][blk]), hmul2_u32(f[2], hs[0][blk]),
                      hmul2_u32(f[3], hs[1][blk]));
          stmatrix_x4(Al + off, hmul2_u32(f[0], ls[0][blk]), hmul2_u32(f[1], ls[1][blk]), hmul2_u32(f[2], ls[0][blk]),
                      hmul2_u32(f[3], ls[1][blk]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[r]);  // the box is read
      if (mark) TC_MARK(8, i);
      fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
      if (!__all_sync(0xFFFFFFFFu, tc_wait(&xfull[s], (i / kTcStages) & 1, abort, a.err))) break;
      if (lane == 0) mbar_arrive_cluster(ready_l + s * 8);  // one arrival per warp, at the leader
      if (mark) TC_MARK(2, i);
    }

    // epilogue: waits for the accumulators, then 2 chunks of 32 token columns
    const uint32_t quad = warp & 3, cg = warp >> 2;
    const uint32_t m = quad * 32 + lane;  // row within the CTA's tile = TMEM lane
    const uint32_t jt = m >> 4, i16 = m & 15;
    bool ok = __all_sync(0xFFFFFFFFu, tc_wait(dfull, 0, abort, a.err));
    tc_fence_after();
    if (threadIdx.x == 0) TC_MARK(5, 0);
    ok = __all_sync(0xFFFFFFFFu, ok && !*abort);
    const uint32_t row = rt0 * 16 + m;
    const bool row_ok = jt < ntiles;
    const uint32_t tok0 = nt * kTcBN + cg * 64;
    const size_t Mr = a.M, ntok = (size_t)L.nt_tiles * kTcBN;
    // Y (or the act of the gate|up epilogue) for 32 tokens from tok; whole warp
    auto store_out = [&](const float (&y)[32], uint32_t tok) {
      if (EPI == EPI_STORE) {
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (tok + i < a.N) a.Y[(size_t)(tok + i) * Mr + row] = y[i];
        }
      } else {
        // interleaved gate|up tiles: tile row i16 < 8 is gate row (rt0+jt)*8 + i16, its
        // up partner sits 8 lanes higher in the same warp.  Each pair of lanes shares
        // the 32 tokens: the gate lane takes the first 16, the up lane the last 16.
        const bool is_gate = i16 < 8;
        const uint32_t Mo = a.M / 2, r = (rt0 + jt) * 8 + (i16 & 7);
        float gv[16] = {}, uv[16] = {};
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float other = __shfl_xor_sync(0xFFFFFFFFu, y[i], 8);
          if (i < 16) {
            gv[i] = is_gate ? y[i] : gv[i];
            uv[i] = is_gate ? other : uv[i];
          } else {
            gv[i - 16] = is_gate ? gv[i - 16] : other;
            uv[i - 16] = is_gate ? uv[i - 16] : y[i];
          }
        }
        const uint32_t t1 = tok + (is_gate ? 0u : 16u);
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 16; i++)
            if (t1 + i < a.N) a.Y[(size_t)(t1 + i) * Mo + r] = gelu_mul(gv[i], uv[i]);
        }
      }
    };
    if (ok) {
#pragma unroll 1
      for (int ch = 0; ch < 2; ch++) {
        const uint32_t taddr = tmem + ((quad * 32u) << 16) + cg * 64 + ch * 32;
        uint32_t v1[32], v2[32];
        tc_ld32(taddr, v1);
        tc_ld32(taddr + kTcBN, v2);
        tc_wait_ld();
        float y[32];
#pragma unroll
        for (int i = 0; i < 32; i++)
          y[i] = __fmaf_rn(__uint_as_float(v2[i]), 1.0f / 65536.f, __fmul_rn(__uint_as_float(v1[i]), 1.0f / 256.f));
        if (L.sk == 1) {
          store_out(y, tok0 + ch * 32);
        } else if (row_ok) {  // partial -> workspace [sk][token][row]
          float *wsk = L.ws + (size_t)sk * ntok * Mr;
#pragma unroll
          for (int i = 0; i < 32; i++) wsk[(size_t)(tok0 + ch * 32 + i) * Mr + row] = y[i];
        }
      }
    }
    if (L.sk > 1) {
      // the last split of this tile to finish adds all partials in split order
      __threadfence();
      epi_sync();
      if (threadIdx.x == 0) {
        const uint32_t tile = (mp * 2 + rank) * L.nt_tiles + nt;
        const uint32_t prev = atomicAdd(&L.counters[tile], 1u);
        *is_last = prev == L.sk - 1;
        if (prev == L.sk - 1) L.counters[tile] = 0u;  // ready for the next launch
      }
      epi_sync();
      if (ok && *is_last) {
        __threadfence();
        // the splits' partials of 32 tokens at a time: every load of a split is in flight
        // before any is added (one dependent L2 round trip per load cost tens of us);
        // the additions keep the split order
#pragma unroll 1
        for (int ch = 0; ch < 2; ch++) {
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; i++) y[i] = 0.f;
          if (row_ok) {
            const float *w0 = L.ws + (size_t)(tok0 + ch * 32) * Mr + row;
#pragma unroll
            for (int i = 0; i < 32; i++) y[i] = __ldcg(w0 + (size_t)i * Mr);
#pragma unroll 1
            for (uint32_t s2 = 1; s2 < L.sk; s2++) {
              const float *wsp = w0 + (size_t)s2 * ntok * Mr;
              float t[32];
#pragma unroll
              for (int i = 0; i < 32; i++) t[i] = __ldcg(wsp + (size_t)i * Mr);
#pragma unroll
              for (int i = 0; i < 32; i++) y[i] = __fadd_rn(y[i], t[i]);
            }
          }
          store_out(y, tok0 + ch * 32);
        }
      }
    }
    if (threadIdx.x == 0) TC_MARK(6, 0);
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // both CTAs done with TMEM and with each other's shared memory
  if (warp == kProdWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Persistent stream-K form of the same GEMM: one cluster per SM pair for the whole
// launch.  The k-tile iterations of all T tiles (tile t = row pair t / nt_tiles, token
// tile t % nt_tiles; KT k tiles each) are split evenly over the C clusters, and a
// cluster walks its range as segments -- the part of one tile's k range it owns --
// with its copy rings, dequant and MMA pipeline running on across segments (no
// per-tile launch, TMEM allocation or pipeline fill).  TMEM holds one tile's
// accumulators, so a segment's first MMA waits until both CTAs' epilogue warps have
// read the previous segment's (tmem_empty).  A segment that covers its whole tile
// stores Y; a tile cut between clusters is written as one partial per contributing
// cluster (part = its index among them, in k order) and the last contributor (counter
// per tile and CTA) adds the parts in k order -- the same order on every run -- and
// applies the epilogue.
struct SkLaunch {
  uint32_t C;          // clusters
  uint32_t T;          // tiles
  uint32_t nt_tiles;   // 256-token tiles
  uint32_t max_parts;  // workspace parts per tile
  uint32_t *counters;  // [T][2], zero between launches
  float *ws;           // [max_parts][nt_tiles * 256][M] partials of cut tiles
};
constexpr uint32_t kNumBarsSk = kNumBars + 1;  // + tmem_empty
constexpr uint32_t kOffMiscSk = kOffBars + kNumBarsSk * 8;
constexpr size_t kTcSmemBytesSk = kOffMiscSk + 16 + 1024;
static_assert(kTcSmemBytesSk <= 232448, "shared memory per CTA");

CH_DEV uint64_t sk_begin(uint64_t W, uint32_t c, uint32_t C) { return W * c / C; }
// the cluster whose range holds iteration it
CH_DEV uint32_t sk_owner(uint64_t W, uint64_t it, uint32_t C) {
  uint32_t c = (uint32_t)((it * C) / W);
  while (c + 1 < C && sk_begin(W, c + 1, C) <= it) c++;
  while (c > 0 && sk_begin(W, c, C) > it) c--;
  return c;
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    batch_gemm_tc_sk_kernel(const TcGemmArgs a, const SkLaunch L, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ uint8_t smem_dyn[];
  const uint32_t dyn = smem_u32(smem_dyn);
  uint8_t *sm = smem_dyn + (((dyn + 1023u) & ~1023u) - dyn);
  const uint32_t sbase = smem_u32(sm);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kOffBars);
  uint64_t *xfull = bars, *aready = bars + kTcStages, *empty = bars + 2 * kTcStages, *dfull = bars + 3 * kTcStages;
  uint64_t *rfull = dfull + 1, *rempty = rfull + kTcRaw, *tmem_empty = rempty + kTcRaw;
  uint32_t *misc = reinterpret_cast<uint32_t *>(sm + kOffMiscSk);
  uint32_t *tmem_slot = misc;
  volatile uint32_t *abort = misc + 1;
  volatile uint32_t *is_last = misc + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t cid = blockIdx.y;
  const uint32_t KT = a.K / kTcBK, row_tiles = a.M / 16;
  const uint64_t W = (uint64_t)L.T * KT;
  const uint64_t it0 = sk_begin(W, cid, L.C), it1 = sk_begin(W, cid + 1, L.C);
  const uint32_t ready_l = map_shared(smem_u32(aready), 0);  // the leader's aready, as a cluster address
  const uint32_t empty_l = map_shared(smem_u32(tmem_empty), 0);
  // segment at iteration it: tile t, k tiles [k0, k1)
  auto segment = [&](uint64_t it, uint32_t &t, uint32_t &k0, uint32_t &k1) {
    t = (uint32_t)(it / KT);
    k0 = (uint32_t)(it - (uint64_t)t * KT);
    const uint64_t tend = (uint64_t)(t + 1) * KT;
    k1 = (uint32_t)((it1 < tend ? it1 : tend) - (uint64_t)t * KT);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; s++) {
      mbar_init(&xfull[s], 1);
      mbar_init(&aready[s], 2 * kDqPerTile);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < kTcRaw; r++) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], kDqPerTile);
    }
    mbar_init(dfull, 1);
    mbar_init(tmem_empty, 2 * kEpiWarps);
    *abort = 0u;
    fence_mbar_init();
  }
  if (warp == kProdWarp) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    if (lane == 0) {  // this CTA's activation share of every k tile, in the cluster's order
      uint32_t g = 0;
      bool live = true;
      for (uint64_t it = it0; it < it1 && live;) {
        uint32_t t, k0, k1;
        segment(it, t, k0, k1);
        const uint8_t *xs = a.xs + ((size_t)(t % L.nt_tiles) * KT * 2 + rank) * kTcXBytes;
        for (uint32_t kt = k0; kt < k1; kt++) {
          const int s = g % kTcStages;
          if (g >= (uint32_t)kTcStages && !tc_wait(&empty[s], ((g / kTcStages) - 1) & 1, abort, a.err)) {
            live = false;
            break;
          }
          mbar_arrive_expect_tx(&xfull[s], kTcXBytes);
          bulk_g2s(sm + s * kTcStageBytes + 2 * kTcABytes, xs + (size_t)kt * 2 * kTcXBytes, kTcXBytes, &xfull[s]);
          g++;
        }
        it = (uint64_t)t * KT + k1;
      }
      for (uint32_t j = g > (uint32_t)kTcStages ? g - kTcStages : 0; j < g; j++)
        tc_wait(&xfull[j % kTcStages], (j / kTcStages) & 1, nullptr, a.err);
    }
  } else if (warp == kRawWarp) {
    if (lane == 0) {  // this CTA's 8 Q4 tiles of every k tile
      uint32_t g = 0;
      bool live = true;
      for (uint64_t it = it0; it < it1 && live;) {
        uint32_t t, k0, k1;
        segment(it, t, k0, k1);
        const uint32_t rt0 = ((t / L.nt_tiles) * 2 + rank) * 8;
        for (uint32_t kt = k0; kt < k1; kt++) {
          const int r = g % kTcRaw;
          if (g >= (uint32_t)kTcRaw && !tc_wait(&rempty[r], ((g / kTcRaw) - 1) & 1, abort, a.err)) {
            live = false;
            break;
          }
          mbar_arrive_expect_tx(&rfull[r], kTcRawBytes);  // the box always lands whole (rows past M read as zeros)
          tma_load_3d(sm + kOffRaw + r * kTcRawBytes, &wmap, 0, (int)kt, (int)rt0, &rfull[r]);
          g++;
        }
        it = (uint64_t)t * KT + k1;
      }
      for (uint32_t j = g > (uint32_t)kTcRaw ? g - kTcRaw : 0; j < g; j++)
        tc_wait(&rfull[j % kTcRaw], (j / kTcRaw) & 1, nullptr, a.err);
    }
  } else if (warp == kMmaWarp) {
    if (leader && lane == 0) {
      uint32_t g = 0, sidx = 0;
      bool live = true;
      for (uint64_t it = it0; it < it1 && live; sidx++) {
        uint32_t t, k0, k1;
        segment(it, t, k0, k1);
        // the previous segment's accumulators read out by both CTAs' epilogue warps
        if (sidx > 0 && !tc_wait(tmem_empty, (sidx - 1) & 1, abort, a.err, true)) break;
        tc_fence_after();
        bool issued = false;
        for (uint32_t kt = k0; kt < k1; kt++) {
          const int s = g % kTcStages;
          if (!tc_wait(&aready[s], (g / kTcStages) & 1, abort, a.err, true)) {
            live = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + s * kTcStageBytes;
          const uint64_t ah = umma_desc_sw128(st), al = umma_desc_sw128(st + kTcABytes);
          const uint64_t xh = umma_desc_sw128(st + 2 * kTcABytes), xl = umma_desc_sw128(st + 2 * kTcABytes + kTcPlane);
#pragma unroll
          for (int ks = 0; ks < 4; ks++) {
            const uint64_t ko = (uint64_t)(ks * 2);  // 32 B per 16-wide k step, in 16-byte units
            const uint32_t acc = (kt != k0 || ks != 0) ? 1u : 0u;
            tc_mma(tmem, ah + ko, xh + ko, acc);          // D1 += A_hi X_hi
            tc_mma(tmem + kTcBN, ah + ko, xl + ko, acc);  // D2 += A_hi (X_lo 2^8)
            tc_mma(tmem + kTcBN, al + ko, xh + ko, 1u);   // D2 += A_lo X_hi
          }
          issued = true;
          tc_commit_pair(&empty[s]);
          g++;
        }
        if (issued) tc_commit_pair(dfull);  // this segment's accumulators (or, after an abort, every MMA issued)
        it = (uint64_t)t * KT + k1;
      }
    }
  } else if (warp < kEpiWarps) {
    const uint32_t j = warp % kDqPerTile, par = warp / kDqPerTile;
    const uint32_t g4 = lane >> 2, mi = lane >> 3, rr = lane & 7;
    const uint32_t quad = warp & 3, cg = warp >> 2;
    const uint32_t m = quad * 32 + lane;  // row within the CTA's tile = TMEM lane
    const uint32_t jt = m >> 4, i16 = m & 15;
    const size_t Mr = a.M, ntok = (size_t)L.nt_tiles * kTcBN;
    uint32_t g = 0, sidx = 0;
    bool ok = true;
    // every epilogue warp walks every segment and reaches every named barrier, whatever
    // its own waits returned: `ok` only gates the work
    for (uint64_t it = it0; it < it1; sidx++) {
      uint32_t t, k0, k1;
      segment(it, t, k0, k1);
      const uint32_t rt0 = ((t / L.nt_tiles) * 2 + rank) * 8;
      const uint32_t ntiles = rt0 < row_tiles ? min(8u, row_tiles - rt0) : 0u;
      // dequant of this segment's k tiles of this warp's parity (see batch_gemm_tc_kernel)
      for (uint32_t kt = k0; kt < k1; kt++, g++) {
        if ((g & 1u) != par || !ok) continue;
        const int s = g % kTcStages, r = g % kTcRaw;
        if (!__all_sync(0xFFFFFFFFu, tc_wait(&rfull[r], (g / kTcRaw) & 1, abort, a.err))) {
          ok = false;
          continue;
        }
        if (g >= (uint32_t)kTcStages &&
            !__all_sync(0xFFFFFFFFu, tc_wait(&empty[s], ((g / kTcStages) - 1) & 1, abort, a.err))) {
          ok = false;
          continue;
        }
        const uint32_t Ah = sbase + s * kTcStageBytes, Al = Ah + kTcABytes;
        if (j < ntiles) {
          const uint8_t *raw = sm + kOffRaw + r * kTcRawBytes + j * kTileBytes;
          const uint4 w = *reinterpret_cast<const uint4 *>(raw + lane * 16);
          const uint2 sc = *reinterpret_cast<const uint2 *>(raw + 512 + g4 * 8);
          uint32_t hs[2][2], ls[2][2];
          bool sok = split_scale(sc.x & 0xFFFFu, hs[0][0], ls[0][0]);
          sok &= split_scale(sc.x >> 16, hs[0][1], ls[0][1]);
          sok &= split_scale(sc.y & 0xFFFFu, hs[1][0], ls[1][0]);
          sok &= split_scale(sc.y >> 16, hs[1][1], ls[1][1]);
          if (!sok) atomicOr(a.err, DEV_ERR_SCALE_RANGE);
          const uint32_t rbase = (2 * j + (mi & 1)) * 1024 + rr * 128;
          const uint32_t ws4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int wi = 0; wi < 4; wi++) {
            const int blk = wi >> 1;
            uint32_t f[4];
            dequant_q4_word(ws4[wi], f);
            const uint32_t chunk = blk * 4 + (wi & 1) * 2 + (mi >> 1);
            const uint32_t off = rbase + ((chunk ^ rr) << 4);
            stmatrix_x4(Ah + off, hmul2_u32(f[0], hs[0][blk]), hmul2_u32(f[1], hs[1][blk]), hmul2_u32(f[2], hs[0][blk]),
                        hmul2_u32(f[3], hs[1][blk]));
            stmatrix_x4(Al + off, hmul2_u32(f[0], ls[0][blk]), hmul2_u32(f[1], ls[1][blk]), hmul2_u32(f[2], ls[0][blk]),
                        hmul2_u32(f[3], ls[1][blk]));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[r]);
        fence_proxy_async();
        if (!__all_sync(0xFFFFFFFFu, tc_wait(&xfull[s], (g / kTcStages) & 1, abort, a.err))) {
          ok = false;
          continue;
        }
        if (lane == 0) mbar_arrive_cluster(ready_l + s * 8);
      }

      // epilogue of the segment
      const uint32_t nt = t % L.nt_tiles;
      const bool whole = k0 == 0 && k1 == KT;
      const uint32_t row = rt0 * 16 + m;
      const bool row_ok = jt < ntiles;
      const uint32_t tok0 = nt * kTcBN + cg * 64;
      const bool got = __all_sync(0xFFFFFFFFu, ok && tc_wait(dfull, sidx & 1, abort, a.err));
      tc_fence_after();
      const bool live = __all_sync(0xFFFFFFFFu, got && !*abort);
      // contributors of a cut tile (clusters in k order) and this cluster's part
      const uint32_t c_first = sk_owner(W, (uint64_t)t * KT, L.C), c_last = sk_owner(W, (uint64_t)(t + 1) * KT - 1, L.C);
      const uint32_t part = cid - c_first, nparts = c_last - c_first + 1;
      if (!whole && nparts > L.max_parts && threadIdx.x == 0) atomicOr(a.err, DEV_ERR_BAD_LIST);
      const bool part_ok = whole || nparts <= L.max_parts;
      auto store_out = [&](const float (&y)[32], uint32_t tok) {
        if (EPI == EPI_STORE) {
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (tok + i < a.N) a.Y[(size_t)(tok + i) * Mr + row] = y[i];
          }
        } else {  // gate|up pairs: as batch_gemm_tc_kernel's epilogue
          const bool is_gate = i16 < 8;
          const uint32_t Mo = a.M / 2, r = (rt0 + jt) * 8 + (i16 & 7);
          float gv[16] = {}, uv[16] = {};
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const float other = __shfl_xor_sync(0xFFFFFFFFu, y[i], 8);
            if (i < 16) {
              gv[i] = is_gate ? y[i] : gv[i];
              uv[i] = is_gate ? other : uv[i];
            } else {
              gv[i - 16] = is_gate ? gv[i - 16] : other;
              uv[i - 16] = is_gate ? uv[i - 16] : y[i];
            }
          }
          const uint32_t t1 = tok + (is_gate ? 0u : 16u);
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 16; i++)
              if (t1 + i < a.N) a.Y[(size_t)(t1 + i) * Mo + r] = gelu_mul(gv[i], uv[i]);
          }
        }
      };
      if (live) {
#pragma unroll 1
        for (int ch = 0; ch < 2; ch++) {
          const uint32_t taddr = tmem + ((quad * 32u) << 16) + cg * 64 + ch * 32;
          uint32_t v1[32], v2[32];
          tc_ld32(taddr, v1);
          tc_ld32(taddr + kTcBN, v2);
          tc_wait_ld();
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; i++)
            y[i] = __fmaf_rn(__uint_as_float(v2[i]), 1.0f / 65536.f, __fmul_rn(__uint_as_float(v1[i]), 1.0f / 256.f));
          if (whole) {
            store_out(y, tok0 + ch * 32);
          } else if (row_ok && part_ok) {  // partial -> workspace [part][token][row]
            float *wsp = L.ws + (size_t)part * ntok * Mr;
#pragma unroll
            for (int i = 0; i < 32; i++) wsp[(size_t)(tok0 + ch * 32 + i) * Mr + row] = y[i];
          }
        }
      }
      // the accumulators are read: the next segment's MMAs may start
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty_l);
      if (!whole) {  // cut tile: the last contributor adds the parts in k order
        __threadfence();
        epi_sync();
        if (threadIdx.x == 0) {
          const uint32_t slot = t * 2 + rank;
          const uint32_t prev = atomicAdd(&L.counters[slot], 1u);
          *is_last = prev == nparts - 1;
          if (prev == nparts - 1) L.counters[slot] = 0u;  // ready for the next launch
        }
        epi_sync();
        if (live && part_ok && *is_last) {
          __threadfence();
#pragma unroll 1
          for (int ch = 0; ch < 2; ch++) {
            float y[32];
#pragma unroll
            for (int i = 0; i < 32; i++) y[i] = 0.f;
            if (row_ok) {
              const float *w0 = L.ws + (size_t)(tok0 + ch * 32) * Mr + row;
#pragma unroll
              for (int i = 0; i < 32; i++) y[i] = __ldcg(w0 + (size_t)i * Mr);
#pragma unroll 1
              for (uint32_t p2 = 1; p2 < nparts; p2++) {
                const float *wsp = w0 + (size_t)p2 * ntok * Mr;
                float tt[32];
#pragma unroll
                for (int i = 0; i < 32; i++) tt[i] = __ldcg(wsp + (size_t)i * Mr);
#pragma unroll
                for (int i = 0; i < 32; i++) y[i] = __fadd_rn(y[i], tt[i]);
              }
            }
            store_out(y, tok0 + ch * 32);
          }
        }
        epi_sync();  // every warp has read is_last before the next cut tile rewrites it
      }
      ok = ok && live;
      it = (uint64_t)t * KT + k1;
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // both CTAs done with TMEM and with each other's shared memory
  if (warp == kProdWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// The Q4 tile array [M/16][K/64][576 B] as a 3-D tensor of u64: x = 72 words of a
// tile, y = k tile (stride 576 B), z = row tile (stride K/64 * 576 B); box 72 x 1 x box_rows.
cudaError_t encode_tile_map(CUtensorMap *map, const uint8_t *tiles, uint32_t M, uint32_t K, uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorNotSupported;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[3] = {kTileBytes / 8, K / kTcBK, M / 16};
  const cuuint64_t strides[2] = {kTileBytes, (cuuint64_t)(K / kTcBK) * kTileBytes};
  const cuuint32_t box[3] = {kTileBytes / 8, 1, box_rows}, estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t *>(tiles), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// split-K factor: more CTA pairs when the rows alone leave SM pairs idle, choosing
// the factor with the fewest waves x k tiles per split; each split keeps >= 8 k tiles
static uint32_t choose_split(uint32_t pairs, uint32_t KT) {
  const uint32_t sm_pairs = (uint32_t)num_sms() / 2;
  if (pairs * 4 >= sm_pairs * 3) return 1;
  uint32_t best = 1;
  uint64_t best_cost = (uint64_t)((pairs + sm_pairs - 1) / sm_pairs) * KT;
  for (uint32_t sk = 2; sk <= 8; sk++) {
    if (KT % sk || KT / sk < 8) continue;
    const uint64_t cost = (uint64_t)((pairs * sk + sm_pairs - 1) / sm_pairs) * (KT / sk);
    if (cost < best_cost) best = sk, best_cost = cost;
  }
  return best;
}
static uint32_t gemm_split(uint32_t N, uint32_t M, uint32_t K) {
  const uint32_t nt = (N + kTcBN - 1) / kTcBN, mp = (M / 16 + 15) / 16;
  const uint32_t sk = choose_split(nt * mp, K / kTcBK);
  return (sk > 1 && mp * 2 * nt > kMaxCounters) ? 1 : sk;
}
static size_t xs_region(uint32_t N, uint32_t K) { return (tc_split_x_bytes(N, K) + 255) & ~(size_t)255; }

size_t tc_split_x_bytes(uint32_t N, uint32_t K) {
  return (size_t)((N + kTcBN - 1) / kTcBN) * (K / kTcBK) * 2 * kTcXBytes;
}
// Clusters of the persistent stream-K kernel that are resident at once on this device
// (0: the occupancy query failed -- use the per-tile kernel)
static uint32_t sk_max_clusters() {
  constexpr int kMaxDev = 64;
  static std::atomic<int> cache[kMaxDev];  // 0: not asked yet, -1: unavailable
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  int c = cache[dev].load(std::memory_order_relaxed);
  if (c == 0) {
    c = -1;
    if (ensure_smem_attr((const void *)batch_gemm_tc_sk_kernel<EPI_STORE>, kTcSmemBytesSk) == cudaSuccess &&
        ensure_smem_attr((const void *)batch_gemm_tc_sk_kernel<EPI_GELU_MUL>, kTcSmemBytesSk) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, (unsigned)(num_sms() / 2));
      cfg.blockDim = dim3(kTcThreads);
      cfg.dynamicSmemBytes = kTcSmemBytesSk;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, (const void *)batch_gemm_tc_sk_kernel<EPI_STORE>, &cfg) == cudaSuccess &&
          n > 0)
        c = n;
      else
        (void)cudaGetLastError();
    }
    cache[dev].store(c, std::memory_order_relaxed);
  }
  return c > 0 ? (uint32_t)c : 0u;
}
struct SkShape {
  uint32_t C, T, nt, max_parts;
};
// the stream-K split of an N x M x K GEMM; C == 0: the per-tile kernel runs instead
static SkShape sk_shape(uint32_t N, uint32_t M, uint32_t K) {
  SkShape sh{};
  const uint32_t cmax = sk_max_clusters();
  sh.nt = (N + kTcBN - 1) / kTcBN;
  sh.T = sh.nt * ((M / 16 + 15) / 16);
  const uint64_t KT = K / kTcBK, W = (uint64_t)sh.T * KT;
  // TMEM holds one tile's accumulators, so a segment boundary drains the pipeline
  // (epilogue, then dequant restart): the persistent form pays only where it replaces
  // more than two waves of per-tile launches (each wave's CTA start-up and fill)
  if (cmax == 0 || W == 0 || sh.T <= 2 * cmax || (uint64_t)sh.T * 2 > kMaxCounters) return sh;
  sh.C = (uint32_t)std::min<uint64_t>(cmax, std::max<uint64_t>(1, W / 8));  // >= 8 k tiles per cluster
  const uint64_t span = W / sh.C;                                           // every range holds >= span
  sh.max_parts = (uint32_t)((KT + span - 1) / span + 1);
  return sh;
}
static size_t sk_ws_bytes(uint32_t N, uint32_t M, uint32_t K) {
  const SkShape sh = sk_shape(N, M, K);
  return sh.C ? (size_t)sh.max_parts * sh.nt * kTcBN * M * sizeof(float) : 0;
}

// enough for any token count up to N (fewer tokens can choose a larger split)
size_t tc_gemm_scratch_bytes(uint32_t N, uint32_t M, uint32_t K) {
  size_t ws = 0;
  for (uint32_t nt = 1; nt <= (N + kTcBN - 1) / kTcBN; nt++) {
    const uint32_t sk = gemm_split(nt * kTcBN, M, K);
    if (sk > 1) ws = std::max(ws, (size_t)sk * nt * kTcBN * M * sizeof(float));
    ws = std::max(ws, sk_ws_bytes(nt * kTcBN, M, K));
  }
  return kCounterBytes + xs_region(N, K) + ws;
}

cudaError_t launch_tc_split_x(const float *X, uint32_t N, uint32_t K, uint8_t *xs, cudaStream_t s) {
  if (K % 64 || N == 0) return N == 0 ? cudaSuccess : cudaErrorInvalidValue;
  const uint32_t ntok = (N + kTcBN - 1) / kTcBN * kTcBN;
  const uint64_t total = (uint64_t)ntok * (K / 8);
  const uint64_t cap = (uint64_t)num_sms() * 8;
  const uint64_t blocks = (total + 255) / 256;
  tc_split_x_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(X, N, K, ntok, xs);
  return cudaGetLastError();
}

// bytes of scratch one launch of this shape uses (tc_gemm_scratch_bytes covers every
// token count up to N)
static size_t tc_launch_scratch_bytes(uint32_t N, uint32_t M, uint32_t K) {
  if (sk_shape(N, M, K).C) return kCounterBytes + xs_region(N, K) + sk_ws_bytes(N, M, K);
  const uint32_t sk = gemm_split(N, M, K);
  const size_t nt = (N + kTcBN - 1) / kTcBN;
  return kCounterBytes + xs_region(N, K) + (sk > 1 ? (size_t)sk * nt * kTcBN * M * sizeof(float) : 0);
}

cudaError_t launch_batch_gemm_tc(const TcGemmArgs &a, uint8_t *scratch, size_t scratch_bytes, cudaStream_t s) {
  if (a.M % 16 || a.K % kTcBK || a.N == 0) return a.N == 0 ? cudaSuccess : cudaErrorInvalidValue;
  if (((uintptr_t)a.xs & 15) || ((uintptr_t)a.tiles & 15) || ((uintptr_t)scratch & 255))
    return cudaErrorInvalidValue;  // copy alignment
  if (!scratch || scratch_bytes < tc_launch_scratch_bytes(a.N, a.M, a.K)) return cudaErrorInvalidValue;
  alignas(64) CUtensorMap wmap;
  cudaError_t me = encode_tile_map(&wmap, a.tiles, a.M, a.K, 8);
  if (me != cudaSuccess) return me;
  const SkShape sh = sk_shape(a.N, a.M, a.K);
  if (sh.C) {  // persistent stream-K: one cluster per SM pair (all resident)
    SkLaunch S{};
    S.C = sh.C;
    S.T = sh.T;
    S.nt_tiles = sh.nt;
    S.max_parts = sh.max_parts;
    S.counters = reinterpret_cast<uint32_t *>(scratch);
    S.ws = reinterpret_cast<float *>(scratch + kCounterBytes + xs_region(a.N, a.K));
    const dim3 grid(2, sh.C);
    if (a.epi == EPI_STORE)
      batch_gemm_tc_sk_kernel<EPI_STORE><<<grid, kTcThreads, kTcSmemBytesSk, s>>>(a, S, wmap);
    else
      batch_gemm_tc_sk_kernel<EPI_GELU_MUL><<<grid, kTcThreads, kTcSmemBytesSk, s>>>(a, S, wmap);
    return cudaGetLastError();
  }
  const uint32_t nt = (a.N + kTcBN - 1) / kTcBN, mp = (a.M / 16 + 15) / 16;
  TcLaunch L{};
  L.sk = gemm_split(a.N, a.M, a.K);
  L.nt_tiles = nt;
  L.counters = reinterpret_cast<uint32_t *>(scratch);
  L.ws = reinterpret_cast<float *>(scratch + kCounterBytes + xs_region(a.N, a.K));
  const dim3 grid(2, nt, mp * L.sk);  // clusters of 2: 256 rows x 256 tokens, per split
  if (a.epi == EPI_STORE) {
    cudaError_t e = ensure_smem_attr((const void *)batch_gemm_tc_kernel<EPI_STORE>, kTcSmemBytes);
    if (e != cudaSuccess) return e;
    batch_gemm_tc_kernel<EPI_STORE><<<grid, kTcThreads, kTcSmemBytes, s>>>(a, L, wmap);
  } else {
    cudaError_t e = ensure_smem_attr((const void *)batch_gemm_tc_kernel<EPI_GELU_MUL>, kTcSmemBytes);
    if (e != cudaSuccess) return e;
    batch_gemm_tc_kernel<EPI_GELU_MUL><<<grid, kTcThreads, kTcSmemBytes, s>>>(a, L, wmap);
  }
  return cudaGetLastError();
}

cudaError_t launch_batch_gemm_q4_tc(const BatchGemmArgs &g, uint8_t *scratch, size_t scratch_bytes, uint32_t *err,
                                    cudaStream_t s) {
  if (g.N == 0) return cudaSuccess;
  if (g.M % 16 || g.K % kTcBK) return cudaErrorInvalidValue;
  if (!scratch || scratch_bytes < tc_launch_scratch_bytes(g.N, g.M, g.K)) return cudaErrorInvalidValue;
  uint8_t *xs = scratch + kCounterBytes;
  cudaError_t e = launch_tc_split_x(g.X, g.N, g.K, xs, s);
  if (e != cudaSuccess) return e;
  return launch_batch_gemm_tc(TcGemmArgs{g.tiles, xs, g.Y, g.M, g.K, g.N, g.epi, err}, scratch, scratch_bytes, s);
}

}  // namespace ch

#ifdef CH_PHASE_TRACE
extern "C" int ch_tc_trace_copy(long long *host, size_t count) {
  if (count > sizeof(ch::g_tc_trace) / 8) count = sizeof(ch::g_tc_trace) / 8;
  return cudaMemcpyFromSymbol(host, ch::g_tc_trace, count * 8) == cudaSuccess ? 0 : -3;
}
#endif
