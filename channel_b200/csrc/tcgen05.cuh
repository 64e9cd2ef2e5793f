// tcgen05.cuh -- tensor-memory, tcgen05, TMA and cluster primitives shared by the
// tcgen05 GEMM kernels (PTX ISA 8.7, sm_100a): prefill_tc.cu (M = 256 weight rows x
// N = 256 tokens per CTA pair) and skinny_tc.cu (M = 128 token rows x N = 256 weight
// rows per CTA, the multi-stream decode step).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ch {

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle: rows of
// 128 B, 8-row atoms of 1024 B (stride byte offset), leading byte offset unused (1),
// descriptor version 1, layout type 2 = SWIZZLE_128B.
CH_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

CH_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CH_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
CH_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 consecutive f32 columns of this thread's TMEM lane
CH_DEV void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
// 3-D tiled TMA load (no multicast) of the box at (x, y, z) into this CTA's shared memory
CH_DEV void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// four 8x8 b16 blocks from mma fragments; lane l gives the address of row l % 8 of block l / 8
CH_DEV void stmatrix_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
CH_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// address of this CTA's shared variable `local` in CTA `rank` of the cluster
CH_DEV uint32_t map_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
CH_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
CH_DEV bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
CH_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bounded mbarrier wait (cluster: acquire at cluster scope, for barriers the other
// CTA arrives at).  With `abort` it also gives up as soon as another role has
// aborted; a wait that runs out of time raises the abort flag and the error.
CH_DEV bool tc_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort, uint32_t *err, bool cluster = false) {
  auto poll = [&]() { return cluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
  if (poll()) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 32; i++)
      if (poll()) return true;
    if (abort && *abort) return false;
    if (globaltimer_ns() - t0 > 2000000000ull) break;
  }
  if (abort) *abort = 1u;
  if (err) atomicOr(err, DEV_ERR_TMA_TIMEOUT);
  return false;
}

// gelu_tanh(g) * u with the operation order of batch_fused_mlp_q4.wgsl's epilogue
CH_DEV float gelu_mul(float g, float u) {
  const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g);
  const float inner = __fmul_rn(0.7978845608f, __fadd_rn(g, x3));
  return __fmul_rn(__fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, tanhf(inner))), u);
}

// f16 block scale d -> the f16x2 multipliers (d_hi 2^8, d_hi 2^8) and (d_lo 2^16,
// d_lo 2^16); both exact.  Returns false for |d| >= 16 (outside the exact range).
CH_DEV bool split_scale(uint32_t dbits, uint32_t &hs, uint32_t &ls) {
  const uint32_t hb = dbits & 0xFFF8u;  // top 8 significant bits (sign kept)
  const float d = __half2float(__ushort_as_half((unsigned short)dbits));
  const float dh = __half2float(__ushort_as_half((unsigned short)hb));
  const float dl = __fsub_rn(d, dh);  // exact: at most 3 significant bits
  const unsigned short h16 = __half_as_ushort(__float2half_rn(__fmul_rn(dh, 256.f)));
  const unsigned short l16 = __half_as_ushort(__float2half_rn(__fmul_rn(dl, 65536.f)));
  hs = (uint32_t)h16 | ((uint32_t)h16 << 16);
  ls = (uint32_t)l16 | ((uint32_t)l16 << 16);
  return fabsf(d) < 16.f;
}
CH_DEV uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Host: tensor map of a Q4 tile array [M/16][K/64][576 B] (prefill_tc.cu) as a 3-D tensor of
// u64 -- x = 72 words of a tile, y = k tile, z = row tile -- with boxes of one k tile of
// box_rows row tiles.
cudaError_t encode_tile_map(CUtensorMap *map, const uint8_t *tiles, uint32_t M, uint32_t K, uint32_t box_rows);

}  // namespace ch
