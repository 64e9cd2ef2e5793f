// topk.cu -- logit softcap + top-64 (+ greedy token) over the vocabulary.
//
// Restates topk_pass1.wgsl:17-19 (softcap 30*tanh(v/30)), topk_pass1/2 (top-64
// sorted descending) and sampler greedy = candidates[0] (src/sampler.zig:213).
// The reference's bitonic merges leave tie order unspecified; here every value
// carries a unique 64-bit key (sortable softcap bits << 32 | ~index), so the
// order is value descending then lowest index first -- deterministic, and the
// same rule the oracle uses.
// B200 design: one pass of radix-select per CTA over 2,048 logits (8 rounds of
// 8-bit histograms in shared memory), 64 candidates per CTA, and the last CTA
// to finish repeats the select over all candidates.  Two launches collapse
// into one; no global sort.
#include "common.cuh"
#include "core.cuh"
#include "kernels.cuh"

namespace ch {

namespace {
constexpr int kTkThreads = 256;
constexpr int kTkPer = 8;  // logits per thread in pass 1
constexpr int kTkChunk = kTkThreads * kTkPer;
constexpr int kFinalPer = 32;  // candidates per thread in the final pass (up to 8192 candidates)
}  // namespace

int topk_blocks(uint32_t V) { return (int)((V + kTkChunk - 1) / kTkChunk); }

__global__ void __launch_bounds__(kTkThreads) topk64_kernel(const TopkArgs a) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh[4];
  __shared__ uint64_t buf[64];
  __shared__ uint64_t sorted[64];
  __shared__ uint32_t cnt;
  __shared__ uint32_t last_flag;
  const int tid = threadIdx.x;
  grid_dep_wait();
  grid_dep_launch();

  {
    uint64_t k[kTkPer];
    const uint32_t base = blockIdx.x * kTkChunk;
#pragma unroll
    for (int e = 0; e < kTkPer; e++) {
      const uint32_t idx = base + e * kTkThreads + tid;
      if (idx < a.V) {
        const float v = softcap(a.logits[idx]);
        k[e] = ((uint64_t)sortable(v) << 32) | (uint64_t)(0xFFFFFFFFu - idx);
      } else {
        k[e] = 0;
      }
    }
    const uint64_t thr = block_kth_largest<kTkPer>(k, 64, hist, sh);
    collect_sorted64<kTkPer>(k, thr, buf, &cnt, sorted);
    if (tid < 64) a.cand[(size_t)blockIdx.x * 64 + tid] = sorted[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = (atomicAdd(a.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();

  uint64_t k[kFinalPer];
  const uint32_t ncand = gridDim.x * 64;
#pragma unroll
  for (int e = 0; e < kFinalPer; e++) {
    const uint32_t i = e * kTkThreads + tid;
    k[e] = i < ncand ? __ldcg(&a.cand[i]) : 0ull;
  }
  const uint64_t thr = block_kth_largest<kFinalPer>(k, 64, hist, sh);
  collect_sorted64<kFinalPer>(k, thr, buf, &cnt, sorted);
  if (tid < 64) {
    const uint64_t key = sorted[tid];
    uint32_t id = 0;
    float val = -1e30f;
    if (key != 0) {
      id = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
      val = unsortable((uint32_t)(key >> 32));
    }
    a.ids[tid] = id;
    a.vals[tid] = val;
    if (tid == 0) {
      if (a.token_out) *a.token_out = id;
      if (a.sp) {
        const uint32_t step = a.sp->step;
        if (a.token_hist && step < a.hist_cap) a.token_hist[step] = id;
      }
    }
  }
  if (tid == 0) *a.counter = 0u;
}

cudaError_t launch_topk64(const TopkArgs &a, cudaStream_t s, bool pdl) {
  const int blocks = topk_blocks(a.V);
  if (blocks * 64 > kTkThreads * kFinalPer) return cudaErrorInvalidValue;  // V <= 262,144 with these sizes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kTkThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, topk64_kernel, a);
}

// ---------------------------------------------------------------------------
// step_begin: advance the device-resident decode loop -- copy plan[step] into
// the live StepParams and expand the embedding of the current token
// (src/model/forward.zig:33-37: x = bf16(embed[token]) * sqrt(H)).
__global__ void step_begin_kernel(const StepBeginArgs a) {
  grid_dep_wait();
  __shared__ StepParams cur;
  if (threadIdx.x == 0) {
    if (a.plan) {
      uint32_t step = a.sp->next;
      if (step >= a.n_plan) {  // replayed past the uploaded plan: keep the last entry, flag it
        atomicOr(a.err, DEV_ERR_BAD_LIST);
        step = a.n_plan - 1;
      }
      cur = a.plan[step];
      cur.step = step;
      cur.next = step + 1;
    } else {
      cur = *a.sp;  // no plan: the device ring wrote this step's parameters (ring_dev.cu)
    }
  }
  __syncthreads();
  if (a.plan && blockIdx.x == 0 && threadIdx.x == 0) *a.sp = cur;
  // RoPE (cos, sin) of this step's clock for both thetas, evaluated once per step
  // in double and rounded once (same values as the host path and the oracle)
  for (uint32_t i = threadIdx.x; i < 2 * a.rot_half; i += blockDim.x) {
    const float f = i < a.rot_half ? a.inv_freq_s[i] : a.inv_freq_f[i - a.rot_half];
    const float ang = __fmul_rn((float)cur.clock, f);
    double sd, cd;
    sincos((double)ang, &sd, &cd);
    a.rope_cs[i] = make_float2((float)cd, (float)sd);
  }
  const uint32_t tok = cur.force ? cur.force - 1 : *a.token;  // a forced (prompt) token, or the fed-back one
  const uint16_t *row = a.embed + (size_t)tok * a.H;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.H; i += gridDim.x * blockDim.x)
    a.x[i] = __fmul_rn(bf16_to_f32(row[i]), a.embed_scale);
  grid_dep_launch();
}
// Greedy token of each of n logit rows: the largest key (sortable softcap bits << 32 |
// ~index) -- the top-1 of topk64_kernel, value first, then the lowest index.  One CTA
// per row.
__global__ void __launch_bounds__(kTkThreads) argmax_rows_kernel(const float *logits, uint32_t V, uint32_t *ids) {
  __shared__ uint64_t wbest[kTkThreads / 32];
  const float *row = logits + (size_t)blockIdx.x * V;
  uint64_t best = 0;
  for (uint32_t idx = threadIdx.x; idx < V; idx += kTkThreads) {
    const uint64_t k = ((uint64_t)sortable(softcap(row[idx])) << 32) | (uint64_t)(0xFFFFFFFFu - idx);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) wbest[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kTkThreads / 32; w++) best = wbest[w] > best ? wbest[w] : best;
    ids[blockIdx.x] = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu);
  }
}
cudaError_t launch_argmax_rows(const float *logits, uint32_t n, uint32_t V, uint32_t *ids, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  argmax_rows_kernel<<<n, kTkThreads, 0, s>>>(logits, V, ids);
  return cudaGetLastError();
}

cudaError_t launch_step_begin(const StepBeginArgs &a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(512);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, step_begin_kernel, a);
}

}  // namespace ch
