// lmhead.cu -- skinny GEMMs of the multi-stream decode step: the Q8 LM head and the
// Q4 layer projections for a batch of up to 64 hidden states.
//
// logits[b][r] = sum_blk s_{r,blk} * sum_i q_{r,i} * x_{b,i}   (gemv_q8.wgsl, for B vectors)
//
// B200 design: a skinny GEMM on mma.sync.m16n8k16.  Each warp owns one 16-row tile
// and streams its Q8 k-tiles once, through its own 2-stage bulk-copy ring, so the
// 1.13 GB head is read once per step for the whole batch.  The tokens enter as f16
// hi / lo B fragments -- built once per step by lmhead_frag_kernel, four tokens per
// MMA (columns token-major, hi then lo) -- and staged by the CTA in chunks of
// kKc k-tiles through a 2-stage ring that all warps of the CTA share.  Per 32-block
// the two k16 MMAs of a token group are summed (hi + lo) and scaled by the row's f32
// block scale into the lane's accumulators, like the single-vector tiles (core.cuh:
// tile_mma<FMT_Q8>), so every logit is fp32-faithful.
#include <algorithm>

#include "common.cuh"
#include "core.cuh"
#include "kernels.cuh"

namespace ch {

namespace {
constexpr int kLw = 16;  // warps (row tiles) per CTA
constexpr int kKc = 4;   // k-tiles per staged chunk
}  // namespace

// xf[(kt * ng + j) * 32 + lane] = {b0, b1} of k16 chunk 0 then chunk 1 of k-tile kt, token
// group j: lane (g, t) supplies column g = token 4j + g/2, hi (g even) or lo (g odd), at
// k = 2t, 2t+1 (b0) and 2t+8, 2t+9 (b1).  Tokens >= B are zero.
__global__ void lmhead_frag_kernel(const float *x, uint32_t ldx, uint32_t B, uint32_t K, uint32_t ng, uint4 *xf) {
  const uint32_t n = K / 32 * ng * 32;
  for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += gridDim.x * blockDim.x) {
    const uint32_t lane = idx & 31, j = (idx >> 5) % ng, kt = (idx >> 5) / ng;
    const uint32_t g = lane >> 2, t = lane & 3, tok = 4 * j + (g >> 1);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (tok < B) {
      const float *row = x + (size_t)tok * ldx + kt * 32;
#pragma unroll
      for (int c = 0; c < 2; c++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const float v0 = row[c * 16 + 2 * t + 8 * h], v1 = row[c * 16 + 2 * t + 8 * h + 1];
          const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
          if (g & 1)
            w[c * 2 + h] = pack_half2(__float2half_rn(__fsub_rn(v0, __half2float(h0))),
                                      __float2half_rn(__fsub_rn(v1, __half2float(h1))));
          else
            w[c * 2 + h] = pack_half2(h0, h1);
        }
    }
    xf[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int NG>
__global__ void __launch_bounds__(kLw * 32, 1) lmhead_q8_kernel(const LmHeadArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr uint32_t kXChunk = kKc * NG * 32 * 16;  // bytes of x fragments per chunk
  constexpr uint32_t kWChunk = kKc * kTileBytes;    // bytes of one warp's weights per chunk
  uint4 *xs = reinterpret_cast<uint4 *>(smem);      // [2][kKc][NG][32]
  uint8_t *ws = smem + 2 * kXChunk;                 // [kLw][2][kWChunk]
  uint64_t *xbar = reinterpret_cast<uint64_t *>(ws + (size_t)kLw * 2 * kWChunk);  // [2]
  uint64_t *wbar = xbar + 2;                                                       // [kLw][2]
  __shared__ uint32_t bad, fail_ch;  // a copy wait gave up (at chunk fail_ch): stop computing and issuing

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t rt = blockIdx.x * kLw + warp;
  const bool active = rt < a.row_tiles;
  const uint32_t KT = a.K / 32, nch = (KT + kKc - 1) / kKc;
  auto chunk_tiles = [&](uint32_t ch) { return min((uint32_t)kKc, KT - ch * kKc); };
  uint8_t *my_w = ws + (size_t)warp * 2 * kWChunk;
  auto issue_x = [&](uint32_t ch) {
    const uint32_t bytes = chunk_tiles(ch) * NG * 32 * 16;
    mbar_arrive_expect_tx(&xbar[ch & 1], bytes);
    bulk_g2s(xs + (size_t)(ch & 1) * kKc * NG * 32, a.xf + (size_t)ch * kKc * NG * 32, bytes, &xbar[ch & 1]);
  };
  auto issue_w = [&](uint32_t ch) {
    const uint32_t bytes = chunk_tiles(ch) * kTileBytes;
    mbar_arrive_expect_tx(&wbar[warp * 2 + (ch & 1)], bytes);
    bulk_g2s(my_w + (size_t)(ch & 1) * kWChunk, a.tiles + ((size_t)rt * KT + (size_t)ch * kKc) * kTileBytes, bytes,
             &wbar[warp * 2 + (ch & 1)]);
  };
  if (threadIdx.x == 0) {
    bad = 0u;
    fail_ch = nch;
    mbar_init(&xbar[0], 1);
    mbar_init(&xbar[1], 1);
  }
  if (lane == 0) {
    mbar_init(&wbar[warp * 2], 1);
    mbar_init(&wbar[warp * 2 + 1], 1);
  }
  fence_mbar_init();
  __syncthreads();
  if (threadIdx.x == 0)
    for (uint32_t ch = 0; ch < 2 && ch < nch; ch++) issue_x(ch);
  if (active && lane == 0)
    for (uint32_t ch = 0; ch < 2 && ch < nch; ch++) issue_w(ch);

  float acc[NG][2];
#pragma unroll
  for (int j = 0; j < NG; j++) acc[j][0] = acc[j][1] = 0.f;
  for (uint32_t ch = 0; ch < nch; ch++) {
    const uint32_t s = ch & 1, par = (ch >> 1) & 1;
    if (!*(volatile uint32_t *)&bad && !mbar_wait_bounded(&xbar[s], par, a.err)) {
      bad = 1u;
      atomicMin(&fail_ch, ch);
    }
    if (active && !*(volatile uint32_t *)&bad && !mbar_wait_bounded(&wbar[warp * 2 + s], par, a.err)) {
      bad = 1u;
      atomicMin(&fail_ch, ch);
    }
    if (active && !*(volatile uint32_t *)&bad) {
      const uint4 *xc = xs + (size_t)s * kKc * NG * 32;
      const uint8_t *wc = my_w + (size_t)s * kWChunk;
      const uint32_t nk = chunk_tiles(ch);
      for (uint32_t kk = 0; kk < nk; kk++) {
        const uint8_t *tile = wc + (size_t)kk * kTileBytes;
        const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
        const float2 sc = *reinterpret_cast<const float2 *>(tile + 512 + g * 8);
        uint32_t a0[4], a1[4];
        dequant_q8_words(w.x, w.y, a0);
        dequant_q8_words(w.z, w.w, a1);
#pragma unroll
        for (int j = 0; j < NG; j++) {
          const uint4 bf = xc[((size_t)kk * NG + j) * 32 + lane];
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816(d, a0, bf.x, bf.y);
          mma_16816(d, a1, bf.z, bf.w);
          acc[j][0] = __fmaf_rn(sc.x, __fadd_rn(d[0], d[1]), acc[j][0]);
          acc[j][1] = __fmaf_rn(sc.y, __fadd_rn(d[2], d[3]), acc[j][1]);
        }
      }
    }
    __syncthreads();  // every warp is done with stage s (and sees `bad`)
    if (ch + 2 < nch && !bad) {
      fence_proxy_async();
      if (threadIdx.x == 0) issue_x(ch + 2);
      if (active && lane == 0) issue_w(ch + 2);
    }
  }
  if (bad) {  // a copy wait gave up: let the copies still in flight (chunks fail_ch, fail_ch + 1) land, bounded
    for (uint32_t ch = fail_ch; ch < fail_ch + 2 && ch < nch; ch++) {
      if (threadIdx.x == 0) mbar_wait_bounded(&xbar[ch & 1], (ch >> 1) & 1, nullptr, 100000000ull);
      if (active && lane == 0) mbar_wait_bounded(&wbar[warp * 2 + (ch & 1)], (ch >> 1) & 1, nullptr, 100000000ull);
    }
    return;
  }
  if (!active) return;
  const uint32_t r0 = rt * 16 + g;
#pragma unroll
  for (int j = 0; j < NG; j++) {
    const uint32_t tok = 4 * j + t;
    if (tok < a.B) {
      a.logits[(size_t)tok * a.V + r0] = acc[j][0];
      a.logits[(size_t)tok * a.V + r0 + 8] = acc[j][1];
    }
  }
}

// ---------------------------------------------------------------------------
// Q4 projections (q|k|v, o, gate|up, down) for the batch: the same scheme on Q4 tiles
// (16 rows x 64 k, two 32-blocks with f16 scales; tile_mma<FMT_Q4>'s arithmetic per
// token), with the K dimension split over gridDim.y so that the 240-row-tile o and down
// matrices still cover the GPU.  Each split writes its partial sums to
// partial[split][token][row]; skinny_reduce_kernel adds the splits in order (so the
// result does not depend on scheduling) and applies the epilogue.
template <int NG>
__global__ void __launch_bounds__(kLw * 32, 1) skinny_q4_kernel(const SkinnyArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr uint32_t kXChunk = 2 * kKc * NG * 32 * 16;  // x fragments of kKc Q4 k-tiles (2 per k-tile)
  constexpr uint32_t kWChunk = kKc * kTileBytes;
  uint4 *xs = reinterpret_cast<uint4 *>(smem);  // [2][2 kKc][NG][32]
  uint8_t *ws = smem + 2 * kXChunk;             // [kLw][2][kWChunk]
  uint64_t *xbar = reinterpret_cast<uint64_t *>(ws + (size_t)kLw * 2 * kWChunk);
  uint64_t *wbar = xbar + 2;
  __shared__ uint32_t bad, fail_ch;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t rt = blockIdx.x * kLw + warp;
  const bool active = rt < a.row_tiles;
  const uint32_t KT = a.K / 64, k0 = blockIdx.y * a.kt_per_split, k1 = min(KT, k0 + a.kt_per_split);
  const uint32_t nkt = k1 > k0 ? k1 - k0 : 0, nch = (nkt + kKc - 1) / kKc;
  auto chunk_tiles = [&](uint32_t ch) { return min((uint32_t)kKc, nkt - ch * kKc); };
  uint8_t *my_w = ws + (size_t)warp * 2 * kWChunk;
  auto issue_x = [&](uint32_t ch) {  // x fragments are per 32-block: two per Q4 k-tile
    const uint32_t bytes = 2 * chunk_tiles(ch) * NG * 32 * 16;
    mbar_arrive_expect_tx(&xbar[ch & 1], bytes);
    bulk_g2s(xs + (size_t)(ch & 1) * 2 * kKc * NG * 32, a.xf + (size_t)(2 * (k0 + ch * kKc)) * NG * 32, bytes,
             &xbar[ch & 1]);
  };
  auto issue_w = [&](uint32_t ch) {
    const uint32_t bytes = chunk_tiles(ch) * kTileBytes;
    mbar_arrive_expect_tx(&wbar[warp * 2 + (ch & 1)], bytes);
    bulk_g2s(my_w + (size_t)(ch & 1) * kWChunk, a.tiles + ((size_t)rt * KT + k0 + (size_t)ch * kKc) * kTileBytes,
             bytes, &wbar[warp * 2 + (ch & 1)]);
  };
  if (threadIdx.x == 0) {
    bad = 0u;
    fail_ch = nch;
    mbar_init(&xbar[0], 1);
    mbar_init(&xbar[1], 1);
  }
  if (lane == 0) {
    mbar_init(&wbar[warp * 2], 1);
    mbar_init(&wbar[warp * 2 + 1], 1);
  }
  fence_mbar_init();
  __syncthreads();
  if (threadIdx.x == 0)
    for (uint32_t ch = 0; ch < 2 && ch < nch; ch++) issue_x(ch);
  if (active && lane == 0)
    for (uint32_t ch = 0; ch < 2 && ch < nch; ch++) issue_w(ch);

  float acc[NG][2];
#pragma unroll
  for (int j = 0; j < NG; j++) acc[j][0] = acc[j][1] = 0.f;
  for (uint32_t ch = 0; ch < nch; ch++) {
    const uint32_t s = ch & 1, par = (ch >> 1) & 1;
    if (!*(volatile uint32_t *)&bad && !mbar_wait_bounded(&xbar[s], par, a.err)) {
      bad = 1u;
      atomicMin(&fail_ch, ch);
    }
    if (active && !*(volatile uint32_t *)&bad && !mbar_wait_bounded(&wbar[warp * 2 + s], par, a.err)) {
      bad = 1u;
      atomicMin(&fail_ch, ch);
    }
    if (active && !*(volatile uint32_t *)&bad) {
      const uint4 *xc = xs + (size_t)s * 2 * kKc * NG * 32;
      const uint8_t *wc = my_w + (size_t)s * kWChunk;
      const uint32_t nk = chunk_tiles(ch);
      for (uint32_t kk = 0; kk < nk; kk++) {
        const uint8_t *tile = wc + (size_t)kk * kTileBytes;
        const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
        const uint2 sc = *reinterpret_cast<const uint2 *>(tile + 512 + g * 8);
        const float2 fg = __half22float2(*reinterpret_cast<const __half2 *>(&sc.x));   // row g: blk0, blk1
        const float2 fg8 = __half22float2(*reinterpret_cast<const __half2 *>(&sc.y));  // row g+8
        uint32_t a0[4], a1[4], a2[4], a3[4];
        dequant_q4_word(w.x, a0);
        dequant_q4_word(w.y, a1);
        dequant_q4_word(w.z, a2);
        dequant_q4_word(w.w, a3);
#pragma unroll
        for (int j = 0; j < NG; j++) {
          const uint4 b0 = xc[((size_t)(2 * kk) * NG + j) * 32 + lane];
          const uint4 b1 = xc[((size_t)(2 * kk + 1) * NG + j) * 32 + lane];
          float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816(d0, a0, b0.x, b0.y);
          mma_16816(d1, a2, b1.x, b1.y);
          mma_16816(d0, a1, b0.z, b0.w);
          mma_16816(d1, a3, b1.z, b1.w);
          acc[j][0] = __fmaf_rn(fg.x, __fadd_rn(d0[0], d0[1]), acc[j][0]);
          acc[j][1] = __fmaf_rn(fg8.x, __fadd_rn(d0[2], d0[3]), acc[j][1]);
          acc[j][0] = __fmaf_rn(fg.y, __fadd_rn(d1[0], d1[1]), acc[j][0]);
          acc[j][1] = __fmaf_rn(fg8.y, __fadd_rn(d1[2], d1[3]), acc[j][1]);
        }
      }
    }
    __syncthreads();
    if (ch + 2 < nch && !bad) {
      fence_proxy_async();
      if (threadIdx.x == 0) issue_x(ch + 2);
      if (active && lane == 0) issue_w(ch + 2);
    }
  }
  if (bad) {
    for (uint32_t ch = fail_ch; ch < fail_ch + 2 && ch < nch; ch++) {
      if (threadIdx.x == 0) mbar_wait_bounded(&xbar[ch & 1], (ch >> 1) & 1, nullptr, 100000000ull);
      if (active && lane == 0) mbar_wait_bounded(&wbar[warp * 2 + (ch & 1)], (ch >> 1) & 1, nullptr, 100000000ull);
    }
    return;
  }
  if (!active) return;
  const size_t R16 = (size_t)a.row_tiles * 16;
  const uint32_t r0 = rt * 16 + g;
#pragma unroll
  for (int j = 0; j < NG; j++) {
    const uint32_t tok = 4 * j + t;
    if (tok < a.B) {
      float *pr = a.partial + ((size_t)blockIdx.y * a.B + tok) * R16;
      pr[r0] = acc[j][0];
      pr[r0 + 8] = acc[j][1];
    }
  }
}

// sum of the splits in order, then the epilogue: y[tok * ldy + row] (EPI_STORE) or, for
// gate|up tiles (rows 0-7 gate, 8-15 up of each row tile), y[tok * ldy + rt*8 + i] =
// gelu(gate row i) * up row i
__global__ void skinny_reduce_kernel(const float *partial, uint32_t splits, uint32_t B, uint32_t row_tiles, int epi,
                                     float *y, uint32_t ldy) {
  const size_t R16 = (size_t)row_tiles * 16;
  const uint32_t per_tok = epi == EPI_GELU_MUL ? row_tiles * 8 : row_tiles * 16;
  const size_t n = (size_t)B * per_tok;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
    const uint32_t tok = (uint32_t)(idx / per_tok), o = (uint32_t)(idx % per_tok);
    const uint32_t row = epi == EPI_GELU_MUL ? (o / 8) * 16 + o % 8 : o;
    float v = 0.f, u = 0.f;
    for (uint32_t s = 0; s < splits; s++) {
      const float *pr = partial + ((size_t)s * B + tok) * R16;
      v = s ? __fadd_rn(v, pr[row]) : pr[row];
      if (epi == EPI_GELU_MUL) u = s ? __fadd_rn(u, pr[row + 8]) : pr[row + 8];
    }
    y[(size_t)tok * ldy + o] = epi == EPI_GELU_MUL ? __fmul_rn(gelu_tanh(v), u) : v;
  }
}

// token groups of 4 the kernel runs for B tokens (instantiated: 1, 2, 4, 8, 16)
static uint32_t lmhead_groups(uint32_t B) {
  const uint32_t ng = (B + 3) / 4;
  return ng <= 1 ? 1 : ng <= 2 ? 2 : ng <= 4 ? 4 : ng <= 8 ? 8 : 16;
}
size_t lmhead_frag_words(uint32_t B, uint32_t K) { return (size_t)K / 32 * lmhead_groups(B) * 32 * 4; }

template <int NG>
static cudaError_t launch_lmhead_t(const LmHeadArgs &a, cudaStream_t s) {
  const size_t smem = (size_t)2 * kKc * NG * 32 * 16 + (size_t)kLw * 2 * kKc * kTileBytes + (2 + 2 * kLw) * 8;
  {
    const cudaError_t e = ensure_smem_attr((const void *)lmhead_q8_kernel<NG>, smem);
    if (e != cudaSuccess) return e;
  }
  const uint32_t grid = (a.row_tiles + kLw - 1) / kLw;
  lmhead_q8_kernel<NG><<<grid, kLw * 32, smem, s>>>(a);
  return cudaGetLastError();
}

// K splits for a Q4 skinny GEMM of row_tiles x (K/64) tiles: enough CTAs for two waves of
// the GPU, each split at least kKc k-tiles
uint32_t skinny_splits(uint32_t row_tiles, uint32_t K) {
  const uint32_t KT = K / 64, ctas = (row_tiles + kLw - 1) / kLw, want = (2 * (uint32_t)num_sms() + ctas - 1) / ctas;
  const uint32_t cap = std::max(1u, KT / kKc);
  return std::max(1u, std::min(want, cap));
}

template <int NG>
static cudaError_t launch_skinny_t(const SkinnyArgs &a, cudaStream_t s) {
  const size_t smem = (size_t)2 * 2 * kKc * NG * 32 * 16 + (size_t)kLw * 2 * kKc * kTileBytes + (2 + 2 * kLw) * 8;
  {
    const cudaError_t e = ensure_smem_attr((const void *)skinny_q4_kernel<NG>, smem);
    if (e != cudaSuccess) return e;
  }
  skinny_q4_kernel<NG><<<dim3((a.row_tiles + kLw - 1) / kLw, a.splits), kLw * 32, smem, s>>>(a);
  return cudaGetLastError();
}

// y = W x for B tokens (x row stride ldx, y row stride ldy); xf and partial are scratch of
// skinny_x_words(B, K) words and skinny_partial_floats(B, row_tiles, K) floats
cudaError_t launch_skinny_q4(const uint8_t *tiles, uint32_t row_tiles, uint32_t K, const float *x, uint32_t ldx,
                             uint32_t B, int epi, float *y, uint32_t ldy, uint32_t *xf, float *partial, uint32_t *err,
                             cudaStream_t s, bool x_ready) {
  if (B == 0 || B > 64 || K % 64 || row_tiles == 0) return cudaErrorInvalidValue;
  if (x_ready && B < kSkinnyTcMinTokens) return cudaErrorInvalidValue;  // only the tcgen05 blocks are prepared
  const size_t outs = (size_t)B * row_tiles * 16;
  const unsigned rblocks = (unsigned)std::min<size_t>((outs + 255) / 256, 4096);
  if (B >= kSkinnyTcMinTokens) {
    uint32_t splits = 0;
    cudaError_t e = launch_skinny_q4_tc(tiles, row_tiles, K, x, ldx, B, reinterpret_cast<uint8_t *>(xf), partial, err,
                                        &splits, s, x_ready);
    if (e != cudaSuccess) return e;
    skinny_reduce_kernel<<<rblocks, 256, 0, s>>>(partial, splits, B, row_tiles, epi, y, ldy);
    return cudaGetLastError();
  }
  const uint32_t ngp = lmhead_groups(B), n = K / 32 * ngp * 32;
  lmhead_frag_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, ldx, B, K, ngp, reinterpret_cast<uint4 *>(xf));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  SkinnyArgs a{};
  a.tiles = tiles;
  a.row_tiles = row_tiles;
  a.K = K;
  a.B = B;
  a.splits = skinny_splits(row_tiles, K);
  a.kt_per_split = (K / 64 + a.splits - 1) / a.splits;
  a.splits = (K / 64 + a.kt_per_split - 1) / a.kt_per_split;  // no empty split
  a.xf = reinterpret_cast<const uint4 *>(xf);
  a.partial = partial;
  a.err = err;
  switch (ngp) {
    case 1: e = launch_skinny_t<1>(a, s); break;
    case 2: e = launch_skinny_t<2>(a, s); break;
    case 4: e = launch_skinny_t<4>(a, s); break;
    case 8: e = launch_skinny_t<8>(a, s); break;
    default: e = launch_skinny_t<16>(a, s); break;
  }
  if (e != cudaSuccess) return e;
  skinny_reduce_kernel<<<rblocks, 256, 0, s>>>(partial, a.splits, B, row_tiles, epi, y, ldy);
  return cudaGetLastError();
}
// enough for any batch up to B (the two variants split K differently)
size_t skinny_partial_floats(uint32_t B, uint32_t row_tiles, uint32_t K) {
  size_t p = (size_t)skinny_splits(row_tiles, K) * B * row_tiles * 16;
  if (B >= kSkinnyTcMinTokens) p = std::max(p, skinny_tc_partial_floats(B, row_tiles, K));
  return p;
}
size_t skinny_x_words(uint32_t B, uint32_t K) {
  size_t w = lmhead_frag_words(B, K);
  if (B >= kSkinnyTcMinTokens) w = std::max(w, skinny_tc_x_bytes(K) / 4);
  return w;
}

// x: B hidden states (row stride ldx floats); xf scratch: lmhead_frag_words(B, K) words
cudaError_t launch_lmhead_q8(const float *x, uint32_t ldx, LmHeadArgs a, uint32_t *xf, cudaStream_t s) {
  if (a.B == 0 || a.B > 64 || a.K % 32 || a.row_tiles == 0) return cudaErrorInvalidValue;
  const uint32_t ngp = lmhead_groups(a.B);
  const uint32_t n = a.K / 32 * ngp * 32;
  lmhead_frag_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, ldx, a.B, a.K, ngp, reinterpret_cast<uint4 *>(xf));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  a.xf = reinterpret_cast<const uint4 *>(xf);
  switch (ngp) {
    case 1: return launch_lmhead_t<1>(a, s);
    case 2: return launch_lmhead_t<2>(a, s);
    case 4: return launch_lmhead_t<4>(a, s);
    case 8: return launch_lmhead_t<8>(a, s);
    default: return launch_lmhead_t<16>(a, s);
  }
}

}  // namespace ch
