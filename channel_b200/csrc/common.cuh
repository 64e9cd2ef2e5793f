// common.cuh -- shared device helpers for the sm_100a kernels: PTX wrappers for
// mbarrier / cp.async.bulk (TMA bulk copies, each to this CTA only), programmatic
// dependent launch, f16 packing, the seeded synthetic generator and the
// device-side error word.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define CH_DEV __device__ __forceinline__

namespace ch {

// ---------------------------------------------------------------------------
// error word written by kernels whose bounded waits give up (never a trap)
enum DevError : uint32_t {
  DEV_ERR_NONE = 0,
  DEV_ERR_TMA_TIMEOUT = 1u << 0,
  DEV_ERR_BAD_SLOT = 1u << 1,
  DEV_ERR_BAD_LIST = 1u << 2,
  DEV_ERR_PEER_TIMEOUT = 1u << 3,
  DEV_ERR_SCALE_RANGE = 1u << 4,  // a Q4 block scale outside the tensor-core GEMM's exact range
};


CH_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

CH_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
CH_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CH_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
CH_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// add expected transaction bytes to the current phase without arriving
CH_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
CH_DEV void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// order this thread's earlier generic-proxy view of global memory (data other CTAs
// wrote and published through a barrier) before its later bulk-copy reads
CH_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
CH_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
CH_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
CH_DEV bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait that polls without suspending (for waits the whole CTA takes at once,
// where a suspended warp's wake-up would delay the CTA's next barrier)
CH_DEV bool mbar_spin_bounded(uint64_t *bar, uint32_t parity, uint32_t *err, uint64_t limit_ns = 2000000000ull) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 64; i++)
      if (mbar_test_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) break;
  }
  if (err) atomicOr(err, DEV_ERR_TMA_TIMEOUT);
  return false;
}
// bounded wait (wall-clock limit); returns false and records the error when it gives up
CH_DEV bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t *err,
                              uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 64; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) break;
  }
  if (err) atomicOr(err, DEV_ERR_TMA_TIMEOUT);
  return false;
}
// 1-D bulk copy global -> this CTA's shared memory, completion on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.  Single destination: this CTA.
CH_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data read exactly once (the weight stream): evict it first, so
// the small activations, norm weights and KV rows that phases re-read stay in L2.
CH_DEV uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// bulk_g2s with an L2 cache policy
CH_DEV void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 16-byte asynchronous global -> shared copy through L2 (no registers held)
CH_DEV void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CH_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
CH_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CH_DEV void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// programmatic dependent launch
CH_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CH_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// f16 helpers
CH_DEV uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
CH_DEV uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm volatile("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}
CH_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm volatile("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
CH_DEV uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm volatile("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
CH_DEV uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm volatile("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
CH_DEV void mma_16816(float *d, const uint32_t *a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D(16x8 s32) = A(16x32 s8, row) * B(32x8 s8, col) + c (c in every accumulator)
CH_DEV void imma_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}
CH_DEV uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {  // (a & b) ^ c
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4 word (8 nibbles in the repacked order) -> A fragment {a0,a1,a2,a3}, values q-8 exact in f16.
//   bits 0-3 / 16-19  -> a0 ; bits 4-7 / 20-23 -> a1 ; bits 8-11 / 24-27 -> a2 ; bits 12-15 / 28-31 -> a3
CH_DEV void dequant_q4_word(uint32_t w, uint32_t *a) {
  const uint32_t MAGIC = 0x64006400u;  // f16 1024
  const uint32_t SUB = 0x64086408u;    // f16 1032 = 1024 + 8
  const uint32_t MUL = 0x2C002C00u;    // f16 1/16
  const uint32_t ADD = 0xD480D480u;    // f16 -72  = -(1024 + 128) / 16
  a[0] = hsub2_u32(lop3_and_or(w, 0x000F000Fu, MAGIC), SUB);
  a[1] = hfma2_u32(lop3_and_or(w, 0x00F000F0u, MAGIC), MUL, ADD);
  uint32_t w8 = w >> 8;
  a[2] = hsub2_u32(lop3_and_or(w8, 0x000F000Fu, MAGIC), SUB);
  a[3] = hfma2_u32(lop3_and_or(w8, 0x00F000F0u, MAGIC), MUL, ADD);
}
// Q8 pair of words (bytes stored as q+128) -> A fragment; values q exact in f16.
CH_DEV void dequant_q8_words(uint32_t w0, uint32_t w1, uint32_t *a) {
  const uint32_t MAGIC = 0x64646464u;
  const uint32_t SUB = 0x64806480u;  // f16 1152 = 1024 + 128
  a[0] = hsub2_u32(prmt(w0, MAGIC, 0x4140u), SUB);
  a[1] = hsub2_u32(prmt(w0, MAGIC, 0x4342u), SUB);
  a[2] = hsub2_u32(prmt(w1, MAGIC, 0x4140u), SUB);
  a[3] = hsub2_u32(prmt(w1, MAGIC, 0x4342u), SUB);
}

// ---------------------------------------------------------------------------
// warp / block reductions (fixed shapes -> identical results in every CTA)
CH_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
CH_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// block sum; `red` needs blockDim.x/32 floats; all threads get the result
CH_DEV float block_sum(float v, float *red) {
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

// ---------------------------------------------------------------------------
// seeded synthetic generator -- same spec as oracle/channel_oracle.cpp
CH_DEV uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
CH_DEV uint64_t hash3(uint64_t tseed, uint64_t stream, uint64_t i) {
  return mix64(mix64(tseed ^ (stream * 0xD6E8FEB86659FD93ull)) ^ (i * 0xD1B54A32D192ED03ull));
}
CH_DEV float gen_normal(uint64_t tseed, uint64_t stream, uint64_t i) {
  int64_t s = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint64_t r = hash3(tseed, stream, i * 4 + j);
    s += (int64_t)(r & 0x1FFFFF) + (int64_t)((r >> 21) & 0x1FFFFF) + (int64_t)((r >> 42) & 0x1FFFFF);
  }
  int32_t c = (int32_t)(2 * s - 12 * (int64_t)0x1FFFFF);
  return __fmul_rn(__int2float_rn(c), 2.384185791015625e-07f);
}
// bf16 round-to-nearest-even exactly as src/tensor.zig:7-13
CH_DEV uint16_t bf16_rne(float v) {
  uint32_t u = __float_as_uint(v);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
CH_DEV float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

}  // namespace ch
