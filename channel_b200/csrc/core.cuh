// core.cuh -- device building blocks shared by the per-op kernels and the
// persistent decode-step kernel: tile dequant + mma, input fragments, head
// norm/RoPE, GELU, and the radix top-64 select.
#pragma once
#include "common.cuh"
#include "kernels.cuh"

namespace ch {

CH_DEV float gelu_tanh(float x) {
  // src/kernels.zig:7-10 / fused_mlp_q4.wgsl:15-18 (explicit rounding, no contraction)
  float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, x3));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// ---------------------------------------------------------------------------
// prologue: build the f16 hi/lo B fragments of the (optionally normed) input.
// xf layout: [32-k block][t 0..3][g 0 = hi | 1 = lo] uint4 {c0.b0, c0.b1, c1.b0, c1.b1}
// (c0 / c1 = the block's two k16 chunks).  One thread per block; every load of a
// phase is issued before any is used, so a phase costs one L2 round trip.
CH_DEV void block_to_fragments(const float (&v)[32], uint4 *xf_blk) {
  float lo[32];
#pragma unroll
  for (int e = 0; e < 32; e++) lo[e] = __fsub_rn(v[e], __half2float(__float2half_rn(v[e])));
#pragma unroll
  for (int t = 0; t < 4; t++) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int c = 0; c < 2; c++) {
      const int k0 = c * 16 + 2 * t;
      hw[c * 2 + 0] = pack_half2(__float2half_rn(v[k0]), __float2half_rn(v[k0 + 1]));
      hw[c * 2 + 1] = pack_half2(__float2half_rn(v[k0 + 8]), __float2half_rn(v[k0 + 9]));
      lw[c * 2 + 0] = pack_half2(__float2half_rn(lo[k0]), __float2half_rn(lo[k0 + 1]));
      lw[c * 2 + 1] = pack_half2(__float2half_rn(lo[k0 + 8]), __float2half_rn(lo[k0 + 9]));
    }
    xf_blk[t * 2 + 0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    xf_blk[t * 2 + 1] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}
// The same fragments built by all threads of the block: one (32-block b, lane
// quad t) item per thread -- the 8 values of v[b*32 ..] a lane with t needs, hi and
// lo -- instead of one whole 32-block per thread.  v may be global or shared.
CH_DEV void build_fragments(const float *v, uint4 *xf, uint32_t K) {
  for (uint32_t idx = threadIdx.x; idx < K / 32 * 4; idx += blockDim.x) {
    const uint32_t b = idx >> 2, t = idx & 3;
    const float *p = v + b * 32 + 2 * t;
    const float2 e0 = *reinterpret_cast<const float2 *>(p), e1 = *reinterpret_cast<const float2 *>(p + 8);
    const float2 e2 = *reinterpret_cast<const float2 *>(p + 16), e3 = *reinterpret_cast<const float2 *>(p + 24);
    const float e[8] = {e0.x, e0.y, e1.x, e1.y, e2.x, e2.y, e3.x, e3.y};
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const __half h0 = __float2half_rn(e[2 * q]), h1 = __float2half_rn(e[2 * q + 1]);
      hw[q] = pack_half2(h0, h1);
      lw[q] = pack_half2(__float2half_rn(__fsub_rn(e[2 * q], __half2float(h0))),
                         __float2half_rn(__fsub_rn(e[2 * q + 1], __half2float(h1))));
    }
    xf[b * 8 + t * 2 + 0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    xf[b * 8 + t * 2 + 1] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}
CH_DEV void load32(const float *p, float (&v)[32]) {
  const float4 *q = reinterpret_cast<const float4 *>(p);
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float4 f = q[i];
    v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
  }
}
CH_DEV void store32(float *p, const float (&v)[32]) {
  float4 *q = reinterpret_cast<float4 *>(p);
#pragma unroll
  for (int i = 0; i < 8; i++) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// one 576-byte tile: 16 rows; lanes with t == 0 accumulate rows g and g+8.
// xb: this lane's x-fragment base (hi for g == 0, lo for g == 1, a zero page for
// g >= 2) and xs its block stride (8 or 0 uint4).
template <int FMT>
CH_DEV void tile_mma(const uint8_t *tile, uint32_t kt, const uint4 *xb, uint32_t xs, int lane, float &acc0,
                     float &acc1) {
  const int g = lane >> 2;
  const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
  if (FMT == FMT_Q4) {
    const uint2 sc = *reinterpret_cast<const uint2 *>(tile + 512 + g * 8);
    const uint4 b0 = xb[(kt * 2 + 0) * xs], b1 = xb[(kt * 2 + 1) * xs];
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t af[4];
    dequant_q4_word(w.x, af);
    mma_16816(d0, af, b0.x, b0.y);
    dequant_q4_word(w.z, af);
    mma_16816(d1, af, b1.x, b1.y);
    dequant_q4_word(w.y, af);
    mma_16816(d0, af, b0.z, b0.w);
    dequant_q4_word(w.w, af);
    mma_16816(d1, af, b1.z, b1.w);
    const __half2 s_lo = *reinterpret_cast<const __half2 *>(&sc.x);  // (row g: blk0, blk1)
    const __half2 s_hi = *reinterpret_cast<const __half2 *>(&sc.y);  // (row g+8: blk0, blk1)
    const float2 fg = __half22float2(s_lo), fg8 = __half22float2(s_hi);
    acc0 = __fmaf_rn(fg.x, __fadd_rn(d0[0], d0[1]), acc0);
    acc1 = __fmaf_rn(fg8.x, __fadd_rn(d0[2], d0[3]), acc1);
    acc0 = __fmaf_rn(fg.y, __fadd_rn(d1[0], d1[1]), acc0);
    acc1 = __fmaf_rn(fg8.y, __fadd_rn(d1[2], d1[3]), acc1);
  } else {
    const float2 sc = *reinterpret_cast<const float2 *>(tile + 512 + g * 8);
    const uint4 b = xb[kt * xs];
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t af[4];
    dequant_q8_words(w.x, w.y, af);
    mma_16816(d, af, b.x, b.y);
    dequant_q8_words(w.z, w.w, af);
    mma_16816(d, af, b.z, b.w);
    acc0 = __fmaf_rn(sc.x, __fadd_rn(d[0], d[1]), acc0);
    acc1 = __fmaf_rn(sc.y, __fadd_rn(d[2], d[3]), acc1);
  }
}

// ---------------------------------------------------------------------------
// Integer tensor-core tiles (standalone GEMV).  The weights enter mma.sync
// m16n8k32 as s8 without a float dequant: a Q4 nibble q becomes the byte
// 16 * (q - 8) by one mask-and-xor, a Q8 byte (stored q ^ 0x80) becomes q by one
// xor.  The input enters as four s8 limbs per value against a power-of-two scale
// per 32-block, x = sx * (l0 + l1 / 2^7 + l2 / 2^14 + l3 / 2^21): X = rint(x /
// sx * 2^21) is a 27-bit integer, l0 = X >> 21 in [-64, 63] and l1..l3 its 7-bit
// fields in [0, 127], so each block dot product is an exact int32 and x is kept
// to 2^-27 of the block's largest magnitude.  Limb c is B column c (lanes g >= 4
// repeat columns 0..3; those results are not used).  The accumulators start at
// 1.5 * 2^23 in integer form, so a result's float view minus 1.5 * 2^23 is the
// exact dot product (|dot| < 2^22) with no integer-to-float conversion.
//
// k order inside a register: splitting the nibbles of a repacked Q4 word (low
// nibble: row g, high nibble: row g+8) gives bytes for k0 + {2t, 2t+8, 2t+1,
// 2t+9} (k0 = the 16-chunk base); Q8 words are regrouped by byte_perm into the
// same order and the limb bytes are built in it.  A and B agree on the order,
// which is all the MMA needs.
constexpr float kLimbMagicF = 12582912.0f;  // 1.5 * 2^23
constexpr int kLimbMagicI = 0x4B400000;     // its bit pattern

// One (32-block b, lane quad t) item: e = the 8 values of block b that quad t
// multiplies, in register byte order (k = 2t, 2t+8, 2t+1, 2t+9, then +16) ->
// xq[b*16 + t*4 + c] = their limb c, sxs[b] = 2^(e-6) where max|x_b| < 2^e.  The 4
// items of a block run on the 4 lanes of an aligned quad at the same time; their
// shuffles for the block maximum come after every read of the inputs and before any
// write, so the limbs may overwrite the block's own inputs in place.
CH_DEV void limb_item(const float (&e)[8], uint32_t b, uint32_t t, uint2 *xq, float *sxs) {
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(e[j]));
  const uint32_t quad = 0xFu << (threadIdx.x & 28u);
  m = fmaxf(m, __shfl_xor_sync(quad, m, 1));
  m = fmaxf(m, __shfl_xor_sync(quad, m, 2));
  // biased exponent E: m < 2^(E-126); X = rint(x * 2^(153-E)) has |X| < 2^27
  const uint32_t E = max((__float_as_uint(m) >> 23) & 0xFFu, 26u);
  const float scale = __uint_as_float((280u - E) << 23);
  int X[8];
#pragma unroll
  for (int j = 0; j < 8; j++) X[j] = __float2int_rn(__fmul_rn(e[j], scale));
  uint32_t wd[4][2];  // limb c of values 4h .. 4h+3, one byte each
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int *x = X + 4 * h;
    wd[0][h] = __byte_perm(__byte_perm(x[0] >> 21, x[1] >> 21, 0x0040u), __byte_perm(x[2] >> 21, x[3] >> 21, 0x0040u),
                           0x5410u);
#pragma unroll
    for (int c = 1; c < 4; c++) {
      const int sh = 21 - 7 * c;
      wd[c][h] = __byte_perm(__byte_perm(x[0] >> sh, x[1] >> sh, 0x0040u), __byte_perm(x[2] >> sh, x[3] >> sh, 0x0040u),
                             0x5410u) &
                 0x7F7F7F7Fu;
    }
  }
  uint4 *o = reinterpret_cast<uint4 *>(xq + b * 16 + t * 4);
  o[0] = make_uint4(wd[0][0], wd[0][1], wd[1][0], wd[1][1]);
  o[1] = make_uint4(wd[2][0], wd[2][1], wd[3][0], wd[3][1]);
  if (t == 0) sxs[b] = __uint_as_float((E - 5u) << 23);
}
// x (K floats, global or shared) -> the limbs of every block; one item per thread
// (blockDim.x % 32 == 0).  In place (v == xq) is allowed.
CH_DEV void build_limbs(const float *v, uint2 *xq, float *sxs, uint32_t K) {
  for (uint32_t idx = threadIdx.x; idx < K / 32 * 4; idx += blockDim.x) {
    const uint32_t b = idx >> 2, t = idx & 3;
    const float *p = v + b * 32 + 2 * t;
    const float2 e0 = *reinterpret_cast<const float2 *>(p), e1 = *reinterpret_cast<const float2 *>(p + 8);
    const float2 e2 = *reinterpret_cast<const float2 *>(p + 16), e3 = *reinterpret_cast<const float2 *>(p + 24);
    const float e[8] = {e0.x, e1.x, e0.y, e1.y, e2.x, e3.x, e2.y, e3.y};
    limb_item(e, b, t, xq, sxs);
  }
}

CH_DEV float limb_dot(int d) { return __fsub_rn(__int_as_float(d), kLimbMagicF); }

// one 576-byte tile on the integer path; acc[0..1] = row g, columns 2t / 2t+1,
// acc[2..3] = row g+8.  xql = xq + t*4 + (g & 3).
template <int FMT>
CH_DEV void tile_i8(const uint8_t *tile, uint32_t kt, const uint2 *xql, const float *sxs, int lane, float (&acc)[4]) {
  const int g = lane >> 2;
  const uint4 w = *reinterpret_cast<const uint4 *>(tile + lane * 16);
  uint32_t a[4];
  int d[4];
  if (FMT == FMT_Q4) {
    const uint2 sc = *reinterpret_cast<const uint2 *>(tile + 512 + g * 8);  // f16 (row g | g+8: blk0, blk1)
    const uint2 bA = xql[kt * 32], bB = xql[kt * 32 + 16];
    const float2 sxv = *reinterpret_cast<const float2 *>(sxs + kt * 2);
    const uint32_t M = 0xF0F0F0F0u, X = 0x80808080u;
    a[0] = lop3_and_xor(w.x << 4, M, X);
    a[1] = lop3_and_xor(w.x, M, X);
    a[2] = lop3_and_xor(w.y << 4, M, X);
    a[3] = lop3_and_xor(w.y, M, X);
    imma_16832(d, a, bA.x, bA.y, kLimbMagicI);
    const float2 fg = __half22float2(*reinterpret_cast<const __half2 *>(&sc.x));
    const float2 fg8 = __half22float2(*reinterpret_cast<const __half2 *>(&sc.y));
    float s0 = __fmul_rn(fg.x, sxv.x), s8 = __fmul_rn(fg8.x, sxv.x);
    acc[0] = __fmaf_rn(s0, limb_dot(d[0]), acc[0]);
    acc[1] = __fmaf_rn(s0, limb_dot(d[1]), acc[1]);
    acc[2] = __fmaf_rn(s8, limb_dot(d[2]), acc[2]);
    acc[3] = __fmaf_rn(s8, limb_dot(d[3]), acc[3]);
    a[0] = lop3_and_xor(w.z << 4, M, X);
    a[1] = lop3_and_xor(w.z, M, X);
    a[2] = lop3_and_xor(w.w << 4, M, X);
    a[3] = lop3_and_xor(w.w, M, X);
    imma_16832(d, a, bB.x, bB.y, kLimbMagicI);
    s0 = __fmul_rn(fg.y, sxv.y);
    s8 = __fmul_rn(fg8.y, sxv.y);
    acc[0] = __fmaf_rn(s0, limb_dot(d[0]), acc[0]);
    acc[1] = __fmaf_rn(s0, limb_dot(d[1]), acc[1]);
    acc[2] = __fmaf_rn(s8, limb_dot(d[2]), acc[2]);
    acc[3] = __fmaf_rn(s8, limb_dot(d[3]), acc[3]);
  } else {
    const float2 sc = *reinterpret_cast<const float2 *>(tile + 512 + g * 8);  // f32 (row g, row g+8)
    const uint2 b = xql[kt * 16];
    const float sx = sxs[kt];
    a[0] = __byte_perm(w.x, w.y, 0x5140u) ^ 0x80808080u;
    a[1] = __byte_perm(w.x, w.y, 0x7362u) ^ 0x80808080u;
    a[2] = __byte_perm(w.z, w.w, 0x5140u) ^ 0x80808080u;
    a[3] = __byte_perm(w.z, w.w, 0x7362u) ^ 0x80808080u;
    imma_16832(d, a, b.x, b.y, kLimbMagicI);
    const float s0 = __fmul_rn(sc.x, sx), s8 = __fmul_rn(sc.y, sx);
    acc[0] = __fmaf_rn(s0, limb_dot(d[0]), acc[0]);
    acc[1] = __fmaf_rn(s0, limb_dot(d[1]), acc[1]);
    acc[2] = __fmaf_rn(s8, limb_dot(d[2]), acc[2]);
    acc[3] = __fmaf_rn(s8, limb_dot(d[3]), acc[3]);
  }
}

// rows g / g+8 of two accumulator sets (valid on lanes t == 0): limb c weighs
// 2^-7c, and Q4 bytes carry a factor 16.  Whole warp.
template <int FMT>
CH_DEV void limb_rows(const float (&acc)[4], const float (&accb)[4], int t, float &v0, float &v1) {
  constexpr float f = FMT == FMT_Q4 ? 0.0625f : 1.0f;
  const float w0 = t == 0 ? f : (t == 1 ? f * 0x1p-14f : 0.f);
  const float w1 = t == 0 ? f * 0x1p-7f : (t == 1 ? f * 0x1p-21f : 0.f);
  v0 = __fadd_rn(__fmul_rn(__fadd_rn(acc[0], accb[0]), w0), __fmul_rn(__fadd_rn(acc[1], accb[1]), w1));
  v1 = __fadd_rn(__fmul_rn(__fadd_rn(acc[2], accb[2]), w0), __fmul_rn(__fadd_rn(acc[3], accb[3]), w1));
  v0 = __fadd_rn(v0, __shfl_down_sync(0xffffffffu, v0, 1));
  v1 = __fadd_rn(v1, __shfl_down_sync(0xffffffffu, v1, 1));
}

// One warp normalizes one head held in shared memory (in -> out, may alias):
// rope: out = rope(rmsnorm(in) * w) with the (cos, sin) table; else unit rmsnorm.
CH_DEV void head_norm_rope_s(const float *in, const float *w, float *out, uint32_t D, uint32_t rot, const float2 *cs,
                             float eps, bool rope, int lane) {
  float ss = 0.f;
  for (uint32_t d = lane; d < D; d += 32) ss = __fmaf_rn(in[d], in[d], ss);
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
  if (!rope) {
    for (uint32_t d = lane; d < D; d += 32) out[d] = __fmul_rn(in[d], inv);
    return;
  }
  const uint32_t half = rot / 2;
  for (uint32_t d = lane; d < half; d += 32) {
    const float v0 = __fmul_rn(__fmul_rn(in[d], inv), w[d]);
    const float v1 = __fmul_rn(__fmul_rn(in[d + half], inv), w[d + half]);
    const float2 c = cs[d];
    out[d] = __fsub_rn(__fmul_rn(v0, c.x), __fmul_rn(v1, c.y));
    out[d + half] = __fadd_rn(__fmul_rn(v0, c.y), __fmul_rn(v1, c.x));
  }
  for (uint32_t d = rot + lane; d < D; d += 32) out[d] = __fmul_rn(__fmul_rn(in[d], inv), w[d]);
}

CH_DEV uint32_t sortable(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
CH_DEV float unsortable(uint32_t s) {
  uint32_t u = (s & 0x80000000u) ? (s ^ 0x80000000u) : ~s;
  return __uint_as_float(u);
}
CH_DEV float softcap(float v) {
  // shaders/topk_pass1.wgsl:17-19
  return __fmul_rn(30.0f, tanhf(__fmul_rn(v, 1.0f / 30.0f)));
}

// Threshold of the K largest 64-bit keys held E-per-thread across the block (keys unique
// except 0 padding): the K-th largest key, or a smaller value that no key outside the K
// largest reaches -- keys >= the result are exactly the K largest (radix select, 8 bits
// per pass from the top, stopping once the selected bin holds exactly the keys still needed)
template <int E>
CH_DEV uint64_t block_kth_largest(const uint64_t (&k)[E], int K, uint32_t *hist, uint32_t *sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t prefix = 0, mask = 0;
  int need = K;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < E; e++)
      if ((k[e] & mask) == prefix) atomicAdd(&hist[(uint32_t)(k[e] >> shift) & 0xFFu], 1u);
    __syncthreads();
    if (warp == 0) {
      uint32_t cnt = 0;
#pragma unroll
      for (int b = 0; b < 8; b++) cnt += hist[lane * 8 + b];
      uint32_t suf = cnt;  // inclusive suffix sum over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += v;
      }
      uint32_t above = __shfl_down_sync(0xffffffffu, suf, 1);
      if (lane == 31) above = 0;
      if (suf >= (uint32_t)need && above < (uint32_t)need) {
        uint32_t run = above;
        for (int b = 7; b >= 0; b--) {
          uint32_t h = hist[lane * 8 + b];
          if (run + h >= (uint32_t)need) {
            sh[0] = (uint32_t)(lane * 8 + b);
            sh[1] = (uint32_t)need - run;
            break;
          }
          run += h;
        }
      }
    }
    __syncthreads();
    const uint32_t sel = sh[0];
    need = (int)sh[1];
    prefix |= (uint64_t)sel << shift;
    mask |= 0xFFull << shift;
    // every key of the selected bin is among the K largest: the prefix (lower bits 0)
    // already separates them from the rest, so later digits change nothing
    const bool done = hist[sel] == (uint32_t)need;
    __syncthreads();
    if (done) break;
  }
  return prefix;
}

// keys >= thr collected into out[64] sorted descending (rank by comparison; pads are 0)
template <int E>
CH_DEV void collect_sorted64(const uint64_t (&k)[E], uint64_t thr, uint64_t *buf, uint32_t *cnt, uint64_t *out) {
  const int tid = threadIdx.x;
  if (tid == 0) *cnt = 0;
  if (tid < 64) buf[tid] = 0;
  __syncthreads();
#pragma unroll
  for (int e = 0; e < E; e++)
    if (k[e] >= thr && k[e] != 0) {
      uint32_t p = atomicAdd(cnt, 1u);
      if (p < 64) buf[p] = k[e];
    }
  __syncthreads();
  if (tid < 64) {
    const uint64_t me = buf[tid];
    int rank = 0;
    for (int j = 0; j < 64; j++) {
      const uint64_t o = buf[j];
      rank += (o > me) || (o == me && j < tid);
    }
    out[rank] = me;
  }
  __syncthreads();
}

}  // namespace ch
