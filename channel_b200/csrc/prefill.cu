// prefill.cu -- batched prefill kernels (one chunk of N <= 1024 prompt tokens).
//
// Restated reference shaders:
//   batch_gemm_q4.wgsl:26-160       Y[t*M + r] = sum_b d_rb sum_i (q-8) X[t][32b+i]
//   batch_fused_mlp_q4.wgsl:33-196  Y[t*M + r] = gelu_tanh(g) * u
//   batch_qkv_rope.wgsl:29-176      token t: clock = start + t, slot = Slots[offset + t]
//   batch_causal_attn.wgsl:25-223   token t attends Slots[start .. num_prev+t+1), sliding: last 1024
//   batch_rmsnorm.wgsl / batch_add_rmsnorm.wgsl
// The GEMM here runs on the decode tile layout with mma.sync: weights are
// exact (q-8) f16 A fragments, activations are split into f16 hi + lo B
// fragments and the per-block f16 scale is applied in f32 -- fp32-faithful.
#include "common.cuh"
#include "kernels.cuh"

namespace ch {

// ---------------------------------------------------------------------------
// norms: one CTA per row.  Rows of H <= 4 * 4 * 256 floats with H % 4 == 0 take the
// register path: each thread loads its (up to four) float4 of the row at once and keeps
// them for the second pass; other rows the strided scalar loop.
constexpr int kNormThreads = 256, kNormVec = 4;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_rows_vec_kernel(const float *x, const float *w, float *y,
                                                                       uint32_t H, float eps) {
  __shared__ float red[32];
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)blockIdx.x * H);
  float4 *yr = reinterpret_cast<float4 *>(y + (size_t)blockIdx.x * H);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  const uint32_t n4 = H / 4;
  float4 v[kNormVec];
#pragma unroll
  for (int k = 0; k < kNormVec; k++) {
    const uint32_t j = threadIdx.x + k * kNormThreads;
    v[k] = j < n4 ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormVec; k++) {
    ss = __fmaf_rn(v[k].x, v[k].x, ss);
    ss = __fmaf_rn(v[k].y, v[k].y, ss);
    ss = __fmaf_rn(v[k].z, v[k].z, ss);
    ss = __fmaf_rn(v[k].w, v[k].w, ss);
  }
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
#pragma unroll
  for (int k = 0; k < kNormVec; k++) {
    const uint32_t j = threadIdx.x + k * kNormThreads;
    if (j < n4) {
      const float4 g = w4[j];
      yr[j] = make_float4(__fmul_rn(__fmul_rn(v[k].x, inv), g.x), __fmul_rn(__fmul_rn(v[k].y, inv), g.y),
                          __fmul_rn(__fmul_rn(v[k].z, inv), g.z), __fmul_rn(__fmul_rn(v[k].w, inv), g.w));
    }
  }
}
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_rows_vec_kernel(float *x, const float *r, const float *w,
                                                                           float *y, uint32_t H, float eps,
                                                                           float scalar) {
  __shared__ float red[32];
  float4 *xr = reinterpret_cast<float4 *>(x + (size_t)blockIdx.x * H);
  const float4 *rr = reinterpret_cast<const float4 *>(r + (size_t)blockIdx.x * H);
  float4 *yr = reinterpret_cast<float4 *>(y + (size_t)blockIdx.x * H);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  const uint32_t n4 = H / 4;
  float4 v[kNormVec];
#pragma unroll
  for (int k = 0; k < kNormVec; k++) {
    const uint32_t j = threadIdx.x + k * kNormThreads;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (j < n4) a = xr[j], b = rr[j];
    v[k] = make_float4(__fmul_rn(__fadd_rn(a.x, b.x), scalar), __fmul_rn(__fadd_rn(a.y, b.y), scalar),
                       __fmul_rn(__fadd_rn(a.z, b.z), scalar), __fmul_rn(__fadd_rn(a.w, b.w), scalar));
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormVec; k++) {
    const uint32_t j = threadIdx.x + k * kNormThreads;
    if (j < n4) xr[j] = v[k];
    ss = __fmaf_rn(v[k].x, v[k].x, ss);
    ss = __fmaf_rn(v[k].y, v[k].y, ss);
    ss = __fmaf_rn(v[k].z, v[k].z, ss);
    ss = __fmaf_rn(v[k].w, v[k].w, ss);
  }
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
#pragma unroll
  for (int k = 0; k < kNormVec; k++) {
    const uint32_t j = threadIdx.x + k * kNormThreads;
    if (j < n4) {
      const float4 g = w4[j];
      yr[j] = make_float4(__fmul_rn(__fmul_rn(v[k].x, inv), g.x), __fmul_rn(__fmul_rn(v[k].y, inv), g.y),
                          __fmul_rn(__fmul_rn(v[k].z, inv), g.z), __fmul_rn(__fmul_rn(v[k].w, inv), g.w));
    }
  }
}
__global__ void rmsnorm_rows_kernel(const float *x, const float *w, float *y, uint32_t H, float eps) {
  __shared__ float red[32];
  const float *xr = x + (size_t)blockIdx.x * H;
  float *yr = y + (size_t)blockIdx.x * H;
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) ss = __fmaf_rn(xr[i], xr[i], ss);
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}
__global__ void add_rmsnorm_rows_kernel(float *x, const float *r, const float *w, float *y, uint32_t H, float eps,
                                        float scalar) {
  __shared__ float red[32];
  float *xr = x + (size_t)blockIdx.x * H;
  const float *rr = r + (size_t)blockIdx.x * H;
  float *yr = y + (size_t)blockIdx.x * H;
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = __fmul_rn(__fadd_rn(xr[i], rr[i]), scalar);
    xr[i] = v;
    ss = __fmaf_rn(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}
cudaError_t launch_rmsnorm_rows(const float *x, const float *w, float *y, uint32_t N, uint32_t H, float eps,
                                cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  const bool vec = H % 4 == 0 && H <= 4u * kNormVec * kNormThreads && !(((uintptr_t)x | (uintptr_t)w | (uintptr_t)y) & 15);
  if (vec)
    rmsnorm_rows_vec_kernel<<<N, kNormThreads, 0, s>>>(x, w, y, H, eps);
  else
    rmsnorm_rows_kernel<<<N, 256, 0, s>>>(x, w, y, H, eps);
  return cudaGetLastError();
}
cudaError_t launch_add_rmsnorm_rows(float *x, const float *r, const float *w, float *y, uint32_t N, uint32_t H,
                                    float eps, float scalar, cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  const bool vec = H % 4 == 0 && H <= 4u * kNormVec * kNormThreads &&
                   !(((uintptr_t)x | (uintptr_t)r | (uintptr_t)w | (uintptr_t)y) & 15);
  if (vec)
    add_rmsnorm_rows_vec_kernel<<<N, kNormThreads, 0, s>>>(x, r, w, y, H, eps, scalar);
  else
    add_rmsnorm_rows_kernel<<<N, 256, 0, s>>>(x, r, w, y, H, eps, scalar);
  return cudaGetLastError();
}
__global__ void embed_rows_kernel(const uint16_t *embed, const uint32_t *tokens, uint32_t H, float scale, float *x) {
  const uint16_t *row = embed + (size_t)tokens[blockIdx.x] * H;
  float *xr = x + (size_t)blockIdx.x * H;
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) xr[i] = __fmul_rn(bf16_to_f32(row[i]), scale);
}
cudaError_t launch_embed_rows(const uint16_t *embed, const uint32_t *tokens, uint32_t N, uint32_t H, float scale,
                              float *x, cudaStream_t s) {
  if (N == 0) return cudaSuccess;
  embed_rows_kernel<<<N, 256, 0, s>>>(embed, tokens, H, scale, x);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// batch qkv_rope: one warp per (head, token)
CH_DEV void warp_norm_rope(const float *in, const float *w, float *out, uint32_t D, uint32_t rot, const float *inv_freq,
                           uint32_t clock, float eps, bool rope, int lane) {
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
    const float ang = __fmul_rn((float)clock, inv_freq[d]);
    double sd, cd;
    sincos((double)ang, &sd, &cd);
    const float c = (float)cd, s = (float)sd;
    out[d] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    out[d + half] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
  }
  for (uint32_t d = rot + lane; d < D; d += 32) out[d] = __fmul_rn(__fmul_rn(in[d], inv), w[d]);
}
__global__ void batch_qkv_rope_kernel(const BatchQkvRopeArgs a) {
  __shared__ float tmp[8][512];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t heads = a.nq + a.nkv;
  const uint64_t item = (uint64_t)blockIdx.x * 8 + warp;
  if (item >= (uint64_t)heads * a.N) return;
  const uint32_t t = (uint32_t)(item / heads), h = (uint32_t)(item % heads);
  const uint32_t D = a.D, clock = a.start_clock + t;
  const size_t qd = (size_t)a.nq * D, kvd = (size_t)a.nkv * D;
  if (h < a.nq) {
    warp_norm_rope(a.q + (size_t)t * a.q_stride + (size_t)h * D, a.q_norm_w, a.q_out + t * qd + (size_t)h * D, D, a.rot, a.inv_freq,
                   clock, a.eps, true, lane);
    return;
  }
  const uint32_t kh = h - a.nq;
  const uint32_t slot = a.slots[a.slot_offset + t];
  float *o = tmp[warp];
  warp_norm_rope(a.k + (size_t)t * a.kv_stride + (size_t)kh * D, a.k_norm_w, o, D, a.rot, a.inv_freq, clock, a.eps, true, lane);
  __syncwarp();
  for (uint32_t d = lane; d < D; d += 32) a.k_cache[(size_t)slot * kvd + (size_t)kh * D + d] = __float2half_rn(o[d]);
  __syncwarp();
  warp_norm_rope((a.k_eq_v ? a.k : a.v) + (size_t)t * a.kv_stride + (size_t)kh * D, nullptr, o, D, a.rot, nullptr, 0, a.eps, false, lane);
  __syncwarp();
  for (uint32_t d = lane; d < D; d += 32) a.v_cache[(size_t)slot * kvd + (size_t)kh * D + d] = __float2half_rn(o[d]);
}
cudaError_t launch_batch_qkv_rope(const BatchQkvRopeArgs &a, cudaStream_t s) {
  if (a.D > 512 || a.N == 0) return a.N == 0 ? cudaSuccess : cudaErrorInvalidValue;
  const uint64_t items = (uint64_t)(a.nq + a.nkv) * a.N;
  batch_qkv_rope_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// batch causal attention: one warp per (token, pair of q heads of one kv head) -- one warp
// per (q head, token) when the group size is odd -- online softmax over the gathered
// slots (K/V rows shared through L1/L2 by the 8 tokens of a CTA, and by the two heads
// within the warp).
constexpr int kCaBlk = 32;  // slots per staged block
constexpr size_t kCaSmem = 2 * 2 * kCaBlk * 32 * sizeof(uint4);  // [2 buffers][K, V][32 slots][512 B]

template <int HW>  // q heads per warp: HW heads of one kv head share every K/V row
__global__ void __launch_bounds__(256, 3) batch_causal_attn_kernel(const BatchAttnArgs a) {
  constexpr int D = 256, EPL = 8;
  extern __shared__ uint4 kv_s[];  // [buf][0 K, 1 V][slot][lane]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t h0 = blockIdx.y * HW;
  // the last tokens attend to the most slots: their CTAs are issued first
  const uint32_t tb = (gridDim.x - 1 - blockIdx.x) * 8;  // this CTA's first token (< N)
  const uint32_t t = tb + warp;
  const bool live = t < a.N;
  const uint32_t ratio = a.nq / a.nkv, kvh = h0 / ratio;  // HW divides ratio: one kv head for all HW
  const size_t qd = (size_t)a.nq * D, kvd = (size_t)a.nkv * D;
  float q[HW][EPL];
#pragma unroll
  for (int hh = 0; hh < HW; hh++) {
    const float *qp = a.q + (size_t)min(t, a.N - 1) * qd + (size_t)(h0 + hh) * D + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; e++) q[hh][e] = qp[e];
  }
  auto first_slot = [&](uint32_t S) { return (a.is_sliding && S > 1024) ? S - 1024 : 0u; };
  const uint32_t S = a.num_prev + t + 1, start = first_slot(S);
  // the CTA's slots: from its first token's window start to its last token
  const uint32_t u0 = first_slot(a.num_prev + tb + 1), u1 = a.num_prev + min(tb + 7, a.N - 1) + 1;
  const uint32_t nblk = (u1 - u0 + kCaBlk - 1) / kCaBlk;
  float m[HW], l[HW], acc[HW][EPL];
#pragma unroll
  for (int hh = 0; hh < HW; hh++) {
    m[hh] = -1e9f;
    l[hh] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; e++) acc[hh][e] = 0.f;
  }
  // online softmax in slot order, per head the same operations as one head per warp
  auto step = [&](const uint4 &kr, const uint4 &vr) {
    const __half2 *kh = reinterpret_cast<const __half2 *>(&kr);
    const __half2 *vh = reinterpret_cast<const __half2 *>(&vr);
    float kf[EPL], vf[EPL];
#pragma unroll
    for (int e = 0; e < EPL / 2; e++) {
      const float2 fk = __half22float2(kh[e]), fv = __half22float2(vh[e]);
      kf[2 * e] = fk.x, kf[2 * e + 1] = fk.y, vf[2 * e] = fv.x, vf[2 * e + 1] = fv.y;
    }
    float dot[HW];
#pragma unroll
    for (int hh = 0; hh < HW; hh++) {
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; e++) d = __fmaf_rn(q[hh][e], kf[e], d);
      dot[hh] = d;
    }
#pragma unroll
    for (int hh = 0; hh < HW; hh++) dot[hh] = __fmul_rn(warp_sum(dot[hh]), a.scale);
#pragma unroll
    for (int hh = 0; hh < HW; hh++) {
      // dot is the same in every lane (warp_sum), so the branch is uniform.  A slot that
      // does not raise the max has corr = expf(+0) = 1 exactly, and fma(x, 1, y) is x + y
      // rounded once: the short path gives the same bits without the second expf.
      if (dot[hh] <= m[hh]) {
        const float p = expf(__fsub_rn(dot[hh], m[hh]));
        l[hh] = __fadd_rn(l[hh], p);
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[hh][e] = __fadd_rn(acc[hh][e], __fmul_rn(p, vf[e]));
      } else {
        const float mn = dot[hh];
        const float corr = expf(__fsub_rn(m[hh], mn));
        const float p = expf(__fsub_rn(dot[hh], mn));
        l[hh] = __fmaf_rn(l[hh], corr, p);
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[hh][e] = __fmaf_rn(acc[hh][e], corr, __fmul_rn(p, vf[e]));
        m[hh] = mn;
      }
    }
  };
  // blocks of 32 slots' K and V rows (32 KB) staged by the whole CTA with cp.async, two
  // buffers: the copy of block b + 1 runs while the warps consume block b.  Thread
  // tid copies 64 bytes of the K and of the V row of slot tid / 8.
  auto stage = [&](uint32_t blk, int buf) {
    const uint32_t j = threadIdx.x >> 3, part = (threadIdx.x & 7) * 4;
    const uint32_t i = u0 + blk * kCaBlk + j;
    if (i < u1) {
      const size_t off = (size_t)a.slots[i] * kvd + (size_t)kvh * D;
      const uint4 *kg = reinterpret_cast<const uint4 *>(a.k_cache + off) + part;
      const uint4 *vg = reinterpret_cast<const uint4 *>(a.v_cache + off) + part;
      uint4 *kd = kv_s + ((size_t)(buf * 2) * kCaBlk + j) * 32 + part;
      uint4 *vd = kv_s + ((size_t)(buf * 2 + 1) * kCaBlk + j) * 32 + part;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        cp_async16(kd + c, kg + c);
        cp_async16(vd + c, vg + c);
      }
    }
    cp_async_commit();  // one group per block in every thread (empty past the last slot)
  };
  stage(0, 0);
  for (uint32_t blk = 0; blk < nblk; blk++) {
    if (blk + 1 < nblk)
      stage(blk + 1, (blk + 1) & 1);
    else
      cp_async_commit();
    cp_async_wait_group<1>();  // this thread's copies of block blk have landed
    __syncthreads();           // ... and everyone's
    const int buf = blk & 1;
    const uint32_t i0 = u0 + blk * kCaBlk;
    if (live) {
      const uint32_t lo = max(i0, start), hi = min(i0 + kCaBlk, S);
      for (uint32_t i = lo; i < hi; i++) {
        const uint32_t j = i - i0;
        step(kv_s[((size_t)(buf * 2) * kCaBlk + j) * 32 + lane], kv_s[((size_t)(buf * 2 + 1) * kCaBlk + j) * 32 + lane]);
      }
    }
    __syncthreads();  // block blk consumed before its buffer takes block blk + 2
  }
  if (!live) return;
#pragma unroll
  for (int hh = 0; hh < HW; hh++) {
    const float inv = __fdiv_rn(1.0f, __fadd_rn(l[hh], 1e-9f));
    float *op = a.out + t * qd + (size_t)(h0 + hh) * D + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; e++) op[e] = __fmul_rn(acc[hh][e], inv);
  }
}
// ---------------------------------------------------------------------------
// batch causal attention on the tensor cores (mma.sync.m16n8k16, f32 accumulate) for
// grouped heads: a CTA is 32 tokens x the two q heads of one kv head (4 warps, 16 rows
// each), the K / V rows of 32 slots at a time staged in shared memory for all of them.
//   S = (Q_hi + Q_lo) K^T: q 2^8 as an f16 pair (two MMAs per step; the scale keeps
//   q_lo = q - q_hi, ~2^-12 q, a normal f16 for |q| >= 2^-10), K exact f16, S 2^-8;
//   online softmax per block of 32 slots (row max over the block, one correction of the
//   running sums per block; masked slots -inf: past the token, or before its window);
//   O += (P_hi + P_lo) V with p 2^14 as an f16 pair too (two MMAs per step into the same
//   accumulators; p_lo stays a normal f16 for p >= 2^-16), V exact; the sum l from the
//   f32 p; out = (O 2^-14) / (l + 1e-9) as batch_causal_attn.wgsl.  The power-of-two
//   scales are exact.
constexpr int kFaTok = 32, kFaSlots = 32, kFaPitch = 264;  // 256 halves + 8: conflict-free rows
constexpr size_t kFaSmem = (size_t)(2 * 2 * kFaTok + 2 * kFaSlots) * kFaPitch * sizeof(__half);

CH_DEV void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__global__ void __launch_bounds__(128, 2) batch_causal_attn_mma_kernel(const BatchAttnArgs a) {
  constexpr int D = 256;
  extern __shared__ __align__(16) __half fa_s[];
  __half *qh = fa_s, *ql = qh + 2 * kFaTok * kFaPitch;  // [head pair row: hh*32 + token][d]
  __half *ks = ql + 2 * kFaTok * kFaPitch, *vs = ks + kFaSlots * kFaPitch;  // [slot][d]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tq = lane & 3;
  const uint32_t h0 = blockIdx.y * 2, ratio = a.nq / a.nkv, kvh = h0 / ratio;
  // the last tokens attend to the most slots: their CTAs are issued first
  const uint32_t t0 = (gridDim.x - 1 - blockIdx.x) * kFaTok;  // < N
  const size_t qd = (size_t)a.nq * D, kvd = (size_t)a.nkv * D;

  // q rows of both heads -> f16 hi / lo planes (tokens past N: zeros)
  for (int idx = tid; idx < 2 * kFaTok * (D / 8); idx += 128) {
    const int row = idx / (D / 8), c8 = idx % (D / 8), hh = row / kFaTok, tk = row % kFaTok;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (t0 + tk < a.N) {
      const float4 *src = reinterpret_cast<const float4 *>(a.q + (size_t)(t0 + tk) * qd + (size_t)(h0 + hh) * D + c8 * 8);
      const float4 x0 = src[0], x1 = src[1];
      v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w, v[4] = x1.x, v[5] = x1.y, v[6] = x1.z, v[7] = x1.w;
    }
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = __fmul_rn(v[e], 256.f);  // q 2^8 (exact)
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const __half a0 = __float2half_rn(v[2 * e]), a1 = __float2half_rn(v[2 * e + 1]);
      hi[e] = pack_half2(a0, a1);
      lo[e] = pack_half2(__float2half_rn(__fsub_rn(v[2 * e], __half2float(a0))),
                         __float2half_rn(__fsub_rn(v[2 * e + 1], __half2float(a1))));
    }
    *reinterpret_cast<uint4 *>(qh + row * kFaPitch + c8 * 8) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(ql + row * kFaPitch + c8 * 8) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }

  // this warp: head h0 + (warp >> 1), tokens t0 + 16 (warp & 1) .. + 15; lane rows g, g + 8
  const int qrow = (warp >> 1) * kFaTok + (warp & 1) * 16;
  const uint32_t tr[2] = {t0 + (warp & 1) * 16 + g, t0 + (warp & 1) * 16 + g + 8};
  auto first_slot = [&](uint32_t S) { return (a.is_sliding && S > 1024) ? S - 1024 : 0u; };
  uint32_t rs[2], re[2];  // each row's slot range [rs, re)
#pragma unroll
  for (int r = 0; r < 2; r++) {
    re[r] = tr[r] < a.N ? a.num_prev + tr[r] + 1 : 0u;
    rs[r] = tr[r] < a.N ? first_slot(re[r]) : 0u;
  }
  const uint32_t tl = min(t0 + kFaTok - 1, a.N - 1);
  const uint32_t u0 = first_slot(a.num_prev + t0 + 1), u1 = a.num_prev + tl + 1;  // the CTA's slots
  const uint32_t nblk = (u1 - u0 + kFaSlots - 1) / kFaSlots;

  float o[32][4];  // 16 rows x 256 d: n-tile j = d 8j..8j+7
#pragma unroll
  for (int j = 0; j < 32; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m[2] = {-1e9f, -1e9f}, l[2] = {0.f, 0.f};  // running max (as the shader starts it) and this lane's part of the sum

  const uint32_t vs_base = smem_u32(vs);
  for (uint32_t blk = 0; blk < nblk; blk++) {
    const uint32_t i0 = u0 + blk * kFaSlots;
    __syncthreads();  // the previous block's rows are no longer read (and q is staged)
    {  // K and V rows of slots i0..i0+31: thread -> slot tid / 4, 128 bytes of each row
      const uint32_t j = tid >> 2, part = (tid & 3) * 64;  // halves
      const uint32_t i = i0 + j;
      __half *kd = ks + j * kFaPitch + part, *vd = vs + j * kFaPitch + part;
      if (i < u1) {
        const size_t off = (size_t)a.slots[i] * kvd + (size_t)kvh * D + part;
#pragma unroll
        for (int c = 0; c < 8; c++) {
          cp_async16(kd + c * 8, a.k_cache + off + c * 8);
          cp_async16(vd + c * 8, a.v_cache + off + c * 8);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 8; c++) {
          *reinterpret_cast<uint4 *>(kd + c * 8) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4 *>(vd + c * 8) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      cp_async_wait_all();
    }
    __syncthreads();

    // S (16 x 32) = Q K^T, both q halves into the same accumulators
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < D / 16; kk++) {
      const int c0 = kk * 16 + 2 * tq;
      uint32_t ah[4], al[4];
      ah[0] = *reinterpret_cast<const uint32_t *>(qh + (qrow + g) * kFaPitch + c0);
      ah[1] = *reinterpret_cast<const uint32_t *>(qh + (qrow + g + 8) * kFaPitch + c0);
      ah[2] = *reinterpret_cast<const uint32_t *>(qh + (qrow + g) * kFaPitch + c0 + 8);
      ah[3] = *reinterpret_cast<const uint32_t *>(qh + (qrow + g + 8) * kFaPitch + c0 + 8);
      al[0] = *reinterpret_cast<const uint32_t *>(ql + (qrow + g) * kFaPitch + c0);
      al[1] = *reinterpret_cast<const uint32_t *>(ql + (qrow + g + 8) * kFaPitch + c0);
      al[2] = *reinterpret_cast<const uint32_t *>(ql + (qrow + g) * kFaPitch + c0 + 8);
      al[3] = *reinterpret_cast<const uint32_t *>(ql + (qrow + g + 8) * kFaPitch + c0 + 8);
#pragma unroll
      for (int nt = 0; nt < 4; nt++) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(ks + (nt * 8 + g) * kFaPitch + c0);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(ks + (nt * 8 + g) * kFaPitch + c0 + 8);
        mma_16816(sc[nt], ah, b0, b1);
        mma_16816(sc[nt], al, b0, b1);
      }
    }

    // mask, block max per row (the quad of lanes sharing a row), probabilities
    float bm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 4; nt++)
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const int r = c >> 1;
        const uint32_t i = i0 + nt * 8 + 2 * tq + (c & 1);
        const float v = (i >= rs[r] && i < re[r]) ? __fmul_rn(__fmul_rn(sc[nt][c], 1.0f / 256.f), a.scale) : -INFINITY;
        sc[nt][c] = v;
        bm[r] = fmaxf(bm[r], v);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      bm[r] = fmaxf(bm[r], __shfl_xor_sync(0xFFFFFFFFu, bm[r], 1));
      bm[r] = fmaxf(bm[r], __shfl_xor_sync(0xFFFFFFFFu, bm[r], 2));
      const float mn = fmaxf(m[r], bm[r]);
      corr[r] = expf(__fsub_rn(m[r], mn));
      m[r] = mn;
      l[r] = __fmul_rn(l[r], corr[r]);
    }
    uint32_t pa[2][4], pl[2][4];  // P (hi, lo) as the A operand of two k16 steps (slots 0-15, 16-31)
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      float p[4];
      __half ph[4], plo[4];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        p[c] = expf(__fsub_rn(sc[nt][c], m[c >> 1]));
        l[c >> 1] = __fadd_rn(l[c >> 1], p[c]);
        const float ps = __fmul_rn(p[c], 16384.f);  // p 2^14 (exact)
        ph[c] = __float2half_rn(ps);
        plo[c] = __float2half_rn(__fsub_rn(ps, __half2float(ph[c])));
      }
      const int ksx = nt >> 1, hi8 = nt & 1;
      pa[ksx][hi8 * 2 + 0] = pack_half2(ph[0], ph[1]);
      pa[ksx][hi8 * 2 + 1] = pack_half2(ph[2], ph[3]);
      pl[ksx][hi8 * 2 + 0] = pack_half2(plo[0], plo[1]);
      pl[ksx][hi8 * 2 + 1] = pack_half2(plo[2], plo[3]);
    }
#pragma unroll
    for (int j = 0; j < 32; j++) {
      o[j][0] = __fmul_rn(o[j][0], corr[0]);
      o[j][1] = __fmul_rn(o[j][1], corr[0]);
      o[j][2] = __fmul_rn(o[j][2], corr[1]);
      o[j][3] = __fmul_rn(o[j][3], corr[1]);
    }
    // O += P V: V as B operand by ldmatrix.trans, two n-tiles (16 d) per load
#pragma unroll
    for (int ksx = 0; ksx < 2; ksx++) {
      const uint32_t vrow = ksx * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int nd = 0; nd < 16; nd++) {
        const uint32_t col = nd * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(vs_base + (vrow * kFaPitch + col) * 2, b0, b1, b2, b3);
        mma_16816(o[2 * nd], pa[ksx], b0, b1);
        mma_16816(o[2 * nd], pl[ksx], b0, b1);
        mma_16816(o[2 * nd + 1], pa[ksx], b2, b3);
        mma_16816(o[2 * nd + 1], pl[ksx], b2, b3);
      }
    }
  }

  // rows' sums over the quad, then out = O / (l + 1e-9)
#pragma unroll
  for (int r = 0; r < 2; r++) {
    l[r] = __fadd_rn(l[r], __shfl_xor_sync(0xFFFFFFFFu, l[r], 1));
    l[r] = __fadd_rn(l[r], __shfl_xor_sync(0xFFFFFFFFu, l[r], 2));
  }
  const uint32_t h = h0 + (warp >> 1);
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if (tr[r] >= a.N) continue;
    const float inv = __fdiv_rn(1.0f, __fadd_rn(l[r], 1e-9f));
    float *op = a.out + (size_t)tr[r] * qd + (size_t)h * D + 2 * tq;
    constexpr float kUnscale = 1.0f / 16384.f;
#pragma unroll
    for (int j = 0; j < 32; j++)
      *reinterpret_cast<float2 *>(op + j * 8) = make_float2(__fmul_rn(__fmul_rn(o[j][2 * r], kUnscale), inv),
                                                            __fmul_rn(__fmul_rn(o[j][2 * r + 1], kUnscale), inv));
  }
}

cudaError_t launch_batch_causal_attn(const BatchAttnArgs &a, cudaStream_t s) {
  if (a.D != 256 || a.N == 0) return a.N == 0 ? cudaSuccess : cudaErrorInvalidValue;
  if (a.nkv == 0 || a.nq % a.nkv) return cudaErrorInvalidValue;
  if ((a.nq / a.nkv) % 2 == 0) {  // pairs of q heads of one kv head: the tensor-core kernel
    cudaError_t e = cudaFuncSetAttribute(batch_causal_attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kFaSmem);
    if (e != cudaSuccess) return e;
    batch_causal_attn_mma_kernel<<<dim3((a.N + kFaTok - 1) / kFaTok, a.nq / 2), 128, kFaSmem, s>>>(a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(batch_causal_attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kCaSmem);
    if (e != cudaSuccess) return e;
    batch_causal_attn_kernel<1><<<dim3((a.N + 7) / 8, a.nq), 256, kCaSmem, s>>>(a);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// batch GEMM on Q4 tiles: CTA = 8 warps = 128 weight rows x 64 tokens.
// X tile [64 tokens][64 k] staged in shared memory as f16 hi and lo planes.
namespace {
constexpr int kBgTok = 64;
constexpr int kBgStride = 72;  // halves per token row (64 + 8 pad -> conflict-free fragment loads)
}  // namespace

template <int EPI>
__global__ void __launch_bounds__(256) batch_gemm_q4_kernel(const BatchGemmArgs a) {
  __shared__ __align__(16) __half xh[2][kBgTok * kBgStride];
  __shared__ __align__(16) __half xl[2][kBgTok * kBgStride];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t KT = a.K / 64, row_tiles = a.M / 16;
  const uint32_t rt = blockIdx.x * 8 + warp;
  const uint32_t tok0 = blockIdx.y * kBgTok;
  const bool active = rt < row_tiles;

  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[j][e] = 0.f;

  auto load_x = [&](uint32_t kt, int buf) {
    // 256 threads: token = tid / 4, 16 consecutive k each
    const uint32_t tk = tid >> 2, kseg = (tid & 3) * 16;
    const uint32_t tok = tok0 + tk;
    __half *hr = xh[buf] + tk * kBgStride + kseg;
    __half *lr = xl[buf] + tk * kBgStride + kseg;
    if (tok < a.N) {
      const float4 *src = reinterpret_cast<const float4 *>(a.X + (size_t)tok * a.K + kt * 64 + kseg);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float4 v = src[q];
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const __half hh = __float2half_rn(vv[e]);
          hr[q * 4 + e] = hh;
          lr[q * 4 + e] = __float2half_rn(__fsub_rn(vv[e], __half2float(hh)));
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; e++) {
        hr[e] = __float2half_rn(0.f);
        lr[e] = __float2half_rn(0.f);
      }
    }
  };

  load_x(0, 0);
  __syncthreads();
  for (uint32_t kt = 0; kt < KT; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < KT) load_x(kt + 1, buf ^ 1);
    if (active) {
      const uint8_t *tile = a.tiles + ((size_t)rt * KT + kt) * kTileBytes;
      const uint4 w = __ldg(reinterpret_cast<const uint4 *>(tile + lane * 16));
      const uint2 sc = __ldg(reinterpret_cast<const uint2 *>(tile + 512 + g * 8));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int blk = 0; blk < 2; blk++) {
        uint32_t af[2][4];
        dequant_q4_word(ws[blk * 2 + 0], af[0]);
        dequant_q4_word(ws[blk * 2 + 1], af[1]);
        const float s0 = __half2float(__ushort_as_half((unsigned short)((blk ? sc.x >> 16 : sc.x) & 0xFFFFu)));
        const float s1 = __half2float(__ushort_as_half((unsigned short)((blk ? sc.y >> 16 : sc.y) & 0xFFFFu)));
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          const int row = j * 8 + g;
#pragma unroll
          for (int ch = 0; ch < 2; ch++) {
            const int kk = blk * 32 + ch * 16 + 2 * t;
            const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(&xh[buf][row * kBgStride + kk]);
            const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(&xh[buf][row * kBgStride + kk + 8]);
            const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(&xl[buf][row * kBgStride + kk]);
            const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(&xl[buf][row * kBgStride + kk + 8]);
            mma_16816(d, af[ch], bh0, bh1);
            mma_16816(d, af[ch], bl0, bl1);
          }
          acc[j][0] = __fmaf_rn(s0, d[0], acc[j][0]);
          acc[j][1] = __fmaf_rn(s0, d[1], acc[j][1]);
          acc[j][2] = __fmaf_rn(s1, d[2], acc[j][2]);
          acc[j][3] = __fmaf_rn(s1, d[3], acc[j][3]);
        }
      }
    }
    __syncthreads();
  }
  if (!active) return;
  // D layout: d0 = (row g, token 2t), d1 = (row g, token 2t+1), d2/d3 = row g+8
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint32_t ta = tok0 + j * 8 + 2 * t, tb = ta + 1;
    if (EPI == EPI_STORE) {
      const uint32_t r0 = rt * 16 + g, r1 = r0 + 8;
      if (ta < a.N) {
        a.Y[(size_t)ta * a.M + r0] = acc[j][0];
        a.Y[(size_t)ta * a.M + r1] = acc[j][2];
      }
      if (tb < a.N) {
        a.Y[(size_t)tb * a.M + r0] = acc[j][1];
        a.Y[(size_t)tb * a.M + r1] = acc[j][3];
      }
    } else {
      const uint32_t Mo = a.M / 2, r = rt * 8 + g;
      float x3, inner;
      if (ta < a.N) {
        const float x = acc[j][0];
        x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
        inner = __fmul_rn(0.7978845608f, __fadd_rn(x, x3));
        a.Y[(size_t)ta * Mo + r] = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner))), acc[j][2]);
      }
      if (tb < a.N) {
        const float x = acc[j][1];
        x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
        inner = __fmul_rn(0.7978845608f, __fadd_rn(x, x3));
        a.Y[(size_t)tb * Mo + r] = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner))), acc[j][3]);
      }
    }
  }
}

cudaError_t launch_batch_gemm_q4(const BatchGemmArgs &a, cudaStream_t s) {
  if (a.M % 16 || a.K % 64 || a.N == 0) return a.N == 0 ? cudaSuccess : cudaErrorInvalidValue;
  dim3 grid((a.M / 16 + 7) / 8, (a.N + kBgTok - 1) / kBgTok);
  if (a.epi == EPI_STORE)
    batch_gemm_q4_kernel<EPI_STORE><<<grid, 256, 0, s>>>(a);
  else
    batch_gemm_q4_kernel<EPI_GELU_MUL><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace ch
