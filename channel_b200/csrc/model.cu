// model.cu -- the C-ABI (include/channel_cuda.h): context, model upload and
// repack, the decode step (captured once into a CUDA graph with programmatic
// dependent launches), batched prefill, state access, the device-resident
// greedy loop and the op-level entry points.
//
// Reference interfaces replaced (Sullux/channel):
//   GpuContext.init/deinit            src/gpu/context.zig:17-109
//   GpuModelContext.init/deinit       src/gpu/model_gpu.zig:68-216
//   recordForwardGraph / gpuDispatchForwardToken  src/gpu/model_dispatch.zig:103-153
//   gpuDispatchPrefillBatch           src/gpu/batch_dispatch.zig:27-172
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/channel_cuda.h"
#include "common.cuh"
#include "decode_step.cuh"
#include "kernels.cuh"

using namespace ch;

// ---------------------------------------------------------------------------
// error plumbing
static thread_local std::string g_err;
static int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}
#define CH_CUDA(call)                                                                          \
  do {                                                                                         \
    cudaError_t _e = (call);                                                                   \
    if (_e != cudaSuccess)                                                                     \
      return fail(CH_ECUDA, std::string(#call) + ": " + cudaGetErrorString(_e) + " @" + \
                                std::to_string(__LINE__));                                     \
  } while (0)

namespace ch {
// lets other translation units of the C-ABI set the calling thread's message
int set_last_error(int code, const std::string &msg) { return fail(code, msg); }
}  // namespace ch

extern "C" const char *ch_last_error(void) { return g_err.c_str(); }
extern "C" int ch_api_version(void) { return CH_API_VERSION; }

// ---------------------------------------------------------------------------
// context
struct ch_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t *err = nullptr;  // device status word
  // op-level scratch (lazily sized)
  float *gemv_partial = nullptr;
  uint32_t *gemv_counters = nullptr;
  size_t gemv_counters_n = 0;
  float *attn_partial = nullptr;
  size_t attn_partial_n = 0;
  uint32_t *attn_counters = nullptr;
  size_t attn_counters_n = 0;
  uint64_t *topk_cand = nullptr;
  uint32_t *topk_counter = nullptr;
  float2 *attn_rope = nullptr;
  size_t attn_rope_n = 0;
  StepParams *op_sp = nullptr;
  uint8_t *xs = nullptr;  // scratch of the tcgen05 GEMM (counters | split activation | partials)
  size_t xs_n = 0;
};

static int ctx_ensure_gemv(ch_ctx *c, uint32_t row_tiles) {
  if (!c->gemv_partial) CH_CUDA(cudaMalloc(&c->gemv_partial, gemv_partial_floats(gemv_default_grid()) * sizeof(float)));
  if (c->gemv_counters_n < row_tiles) {
    if (c->gemv_counters) CH_CUDA(cudaFree(c->gemv_counters));
    c->gemv_counters_n = row_tiles;
    CH_CUDA(cudaMalloc(&c->gemv_counters, row_tiles * sizeof(uint32_t)));
    CH_CUDA(cudaMemsetAsync(c->gemv_counters, 0, row_tiles * sizeof(uint32_t), c->stream));
  }
  return CH_OK;
}

static int ctx_ensure_xs(ch_ctx *c, size_t bytes) {
  if (c->xs_n >= bytes) return CH_OK;
  CH_CUDA(cudaStreamSynchronize(c->stream));
  if (c->xs) CH_CUDA(cudaFree(c->xs));
  c->xs = nullptr;
  c->xs_n = 0;
  CH_CUDA(cudaMalloc(&c->xs, bytes));
  CH_CUDA(cudaMemsetAsync(c->xs, 0, 16384, c->stream));  // split-K tile counters start at zero
  c->xs_n = bytes;
  return CH_OK;
}

extern "C" int ch_ctx_create(int device, ch_ctx **out) {
  if (!out) return fail(CH_EINVAL, "out is NULL");
  int n = 0;
  CH_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(CH_EINVAL, "device index out of range");
  CH_CUDA(cudaSetDevice(device));
  ch_ctx *c = new ch_ctx();
  c->device = device;
  CH_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  CH_CUDA(cudaMalloc(&c->err, sizeof(uint32_t)));
  CH_CUDA(cudaMemsetAsync(c->err, 0, sizeof(uint32_t), c->stream));
  CH_CUDA(cudaMalloc(&c->topk_cand, (size_t)8192 * sizeof(uint64_t)));
  CH_CUDA(cudaMalloc(&c->topk_counter, sizeof(uint32_t)));
  CH_CUDA(cudaMemsetAsync(c->topk_counter, 0, sizeof(uint32_t), c->stream));
  CH_CUDA(cudaMalloc(&c->op_sp, sizeof(StepParams)));
  CH_CUDA(cudaStreamSynchronize(c->stream));
  *out = c;
  return CH_OK;
}
extern "C" void ch_ctx_destroy(ch_ctx *c) {
  if (!c) return;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  cudaFree(c->err);
  cudaFree(c->gemv_partial);
  cudaFree(c->gemv_counters);
  cudaFree(c->attn_partial);
  cudaFree(c->attn_counters);
  cudaFree(c->topk_cand);
  cudaFree(c->topk_counter);
  cudaFree(c->attn_rope);
  cudaFree(c->op_sp);
  cudaFree(c->xs);
  cudaStreamDestroy(c->stream);
  delete c;
}
extern "C" int ch_ctx_synchronize(ch_ctx *c) {
  if (!c) return fail(CH_EINVAL, "ctx is NULL");
  CH_CUDA(cudaStreamSynchronize(c->stream));
  return CH_OK;
}
extern "C" void *ch_ctx_stream(ch_ctx *c) { return c ? (void *)c->stream : nullptr; }
extern "C" int ch_ctx_device_status(ch_ctx *c, uint32_t *flags) {
  if (!c || !flags) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaMemcpyAsync(flags, c->err, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
  CH_CUDA(cudaMemsetAsync(c->err, 0, sizeof(uint32_t), c->stream));
  CH_CUDA(cudaStreamSynchronize(c->stream));
  return CH_OK;
}
static int status_from_flags(uint32_t f) {
  if (f & (DEV_ERR_TMA_TIMEOUT | DEV_ERR_PEER_TIMEOUT)) return fail(CH_ETIMEOUT, "a bounded device wait gave up");
  if (f & (DEV_ERR_BAD_SLOT | DEV_ERR_BAD_LIST)) return fail(CH_EDEVICE, "kernel saw a slot index >= 4096");
  return CH_OK;
}

// ---------------------------------------------------------------------------
// model
namespace {
struct DevLayer {
  uint8_t *qkv = nullptr, *o = nullptr, *gateup = nullptr, *down = nullptr;
  float *input_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn = nullptr, *pre_ffn = nullptr,
        *post_ffn = nullptr;
  float scalar = 1.0f;
  __half *kc = nullptr, *vc = nullptr;
  bool full = false;
};
constexpr uint32_t kSlots = 4096;
}  // namespace

struct ch_model {
  ch_ctx *ctx = nullptr;
  ch_model_config cfg{};
  uint32_t H = 0, I = 0, V = 0, D = 0, nq = 0, nkv = 0, qd = 0, kvd = 0, L = 0;
  // tensor parallel: this process holds shard `rank` of `world` (1 = the whole model).
  // Local sizes: q / kv heads, o and down output rows, gate and up rows, vocab rows.
  uint32_t rank = 0, world = 1;
  uint32_t nq_l = 0, nkv_l = 0, qd_l = 0, kvd_l = 0, Il = 0, Vl = 0;
  uint8_t *arena = nullptr;                // exchange arena (CUDA IPC shared): gathered vectors + arrivals
  uint8_t *peer_arena[kMaxWorld] = {};     // every rank's arena mapped here (peer_arena[rank] = arena)
  bool peers_ready = false;
  size_t off_arrive = 0, off_o = 0, off_down = 0, off_cand = 0, arena_bytes = 0;
  StepParams *pplan = nullptr;             // tensor-parallel prefill: forced-token plan
  uint32_t *pplan_lists = nullptr;
  std::vector<DevLayer> layers;
  uint8_t *lm = nullptr;
  float *final_norm = nullptr;
  uint16_t *embed = nullptr;
  float *inv_freq_s = nullptr, *inv_freq_f = nullptr;
  std::vector<float> h_inv_s, h_inv_f;  // same tables on the host (per-step RoPE on the host path)
  float2 *rope_cs = nullptr;            // [2][rot/2] (cos, sin) of the current clock
  float2 *h_rope = nullptr;             // pinned staging
  // decode buffers
  float *X[2] = {nullptr, nullptr};
  float *normed = nullptr, *qkv = nullptr, *attn = nullptr, *o_out = nullptr, *act = nullptr, *down_out = nullptr,
        *logits = nullptr, *vals = nullptr;
  uint32_t *ids = nullptr, *token = nullptr, *token_hist = nullptr;
  StepParams *sp = nullptr;
  uint32_t *active = nullptr, *sliding = nullptr;
  // scratch
  float *gemv_partial = nullptr;
  uint32_t *gemv_counters = nullptr;
  float *attn_partial = nullptr;
  uint32_t *attn_counters = nullptr;
  uint64_t *topk_cand = nullptr;
  uint32_t *topk_counter = nullptr;
  int attn_splits = 0;
  // host staging (pinned)
  float *h_x = nullptr;
  StepParams *h_sp = nullptr;
  uint32_t *h_lists = nullptr;  // [2][4096]
  uint32_t *h_ids = nullptr;
  float *h_vals = nullptr;
  uint32_t *h_run = nullptr;  // [2] staging for ch_decode_run
  uint32_t *h_status = nullptr;  // the device status word read back with each forward token
  // graphs
  cudaGraphExec_t g_host_logits = nullptr, g_host_nologits = nullptr, g_loop = nullptr;
  bool pdl = true;
  // device loop plan
  ch_sampler *sampler = nullptr;  // device loops sample with it (NULL: greedy)
  StepParams *plan = nullptr;
  uint32_t *plan_lists = nullptr;
  uint32_t plan_steps = 0, hist_cap = 0, loop_pos = 0;
  bool loop_ready = false;
  // persistent decode-step kernel: phase tables, per-GEMV outputs, barrier counters
  Phase *d_phases = nullptr, *d_phases_nl = nullptr;
  Partition kpart[2][kKinds] = {};  // GEMV partitions of each phase table (with / without logits)
  uint32_t n_phases = 0, n_phases_nl = 0;
  StreamDesc *d_streams = nullptr, *d_streams_nl = nullptr;  // weight streams of the GEMV phases
  uint32_t n_streams = 0, n_streams_nl = 0;
  float *gdir[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  float *gpart[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  unsigned long long *mk_arrive = nullptr;
  unsigned long long *mk_base = nullptr;  // [3] barrier arrivals (local, cross-rank), exchange epochs
  uint32_t n_cross = 0, n_cross_nl = 0;    // cross-rank barriers per launch (logits / no-logits tables)
  uint32_t n_local = 0, n_local_nl = 0;    // grid barriers per launch
  uint32_t n_x = 0, n_x_nl = 0;            // low-latency exchanges per launch
  size_t mk_smem = 0;
  int mk_grid = 0;
  bool use_ops = false;  // kernel-per-op decode (CH_DECODE_OPS=1), kept for A/B measurement
  // prefill buffers
  uint32_t pf_cap = 0;
  float *pX = nullptr, *pNX = nullptr, *pQKV = nullptr, *pQO = nullptr, *pA = nullptr, *pMO = nullptr, *pACT = nullptr;
  uint32_t *pSlots = nullptr, *pTok = nullptr;
  uint8_t *pXS = nullptr;  // scratch of the tcgen05 GEMM (counters | split activation | partials)
  size_t pXS_n = 0;
  // multi-stream decode: per-stream KV caches and the buffers of one batched step
  uint32_t ms_n = 0, ms_cap = 0;   // decode streams and the largest step
  std::vector<__half *> skc, svc;  // per layer: [ms_n][4096][kv_dim]
  float *ms_logits = nullptr;      // [ms_cap][V]
  uint32_t *ms_tok = nullptr, *ms_stream = nullptr, *ms_ids = nullptr, *ms_lists = nullptr;
  StepParams *ms_sp = nullptr;     // [ms_cap]
  float2 *ms_rope = nullptr;       // [2][ms_cap][rot/2]: sliding theta, then full theta
  float *ms_partial = nullptr;     // attention split partials, [ms_cap] slices
  uint32_t *ms_counters = nullptr; // [ms_cap][n_kv]
  uint32_t *ms_xf = nullptr;       // token fragments of the skinny GEMMs (largest K)
  float *ms_skp = nullptr;         // split-K partials of the skinny Q4 GEMMs
  std::vector<cudaGraphExec_t> ms_exec;  // the batched step per batch size (index n)
  uint32_t *h_ms_u32 = nullptr;    // pinned: tokens | streams | lists | ids
  StepParams *h_ms_sp = nullptr;
  float2 *h_ms_rope = nullptr;
};

static void free_streams(ch_model *m);
static void free_model(ch_model *m) {
  if (!m) return;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (auto &l : m->layers) {
    cudaFree(l.qkv);
    cudaFree(l.o);
    cudaFree(l.gateup);
    cudaFree(l.down);
    cudaFree(l.input_norm);
    cudaFree(l.q_norm);
    cudaFree(l.k_norm);
    cudaFree(l.post_attn);
    cudaFree(l.pre_ffn);
    cudaFree(l.post_ffn);
    cudaFree(l.kc);
    cudaFree(l.vc);
  }
  free_streams(m);
  void *dev[] = {m->lm, m->final_norm, m->embed, m->inv_freq_s, m->inv_freq_f, m->rope_cs, m->X[0], m->X[1], m->normed, m->qkv,
                 m->attn, m->o_out, m->act, m->down_out, m->logits, m->vals, m->ids, m->token, m->token_hist, m->sp,
                 m->active, m->sliding, m->gemv_partial, m->gemv_counters, m->attn_partial, m->attn_counters,
                 m->topk_cand, m->topk_counter, m->plan, m->plan_lists, m->pX, m->pNX, m->pQKV, m->pQO, m->pA, m->pMO,
                 m->pACT, m->pSlots, m->pTok, m->pXS};
  for (void *p : dev) cudaFree(p);
  for (int k = 0; k < 5; k++) {
    cudaFree(m->gdir[k]);
    cudaFree(m->gpart[k]);
  }
  cudaFree(m->d_phases);
  cudaFree(m->d_phases_nl);
  cudaFree(m->d_streams);
  cudaFree(m->d_streams_nl);
  cudaFree(m->mk_arrive);
  cudaFree(m->mk_base);
  cudaFree(m->pplan);
  cudaFree(m->pplan_lists);
  for (uint32_t r = 0; r < m->world && r < kMaxWorld; r++)
    if (r != m->rank && m->peer_arena[r]) cudaIpcCloseMemHandle(m->peer_arena[r]);
  cudaFree(m->arena);
  void *host[] = {m->h_x, m->h_sp, m->h_lists, m->h_ids, m->h_vals, m->h_run, m->h_rope, m->h_status};
  for (void *p : host) cudaFreeHost(p);
  if (m->g_host_logits) cudaGraphExecDestroy(m->g_host_logits);
  if (m->g_host_nologits) cudaGraphExecDestroy(m->g_host_nologits);
  if (m->g_loop) cudaGraphExecDestroy(m->g_loop);
  delete m;
}

static int check_cfg(const ch_model_config *c) {
  if (!c) return fail(CH_EINVAL, "cfg is NULL");
  if (c->num_hidden_layers == 0 || c->num_hidden_layers > 64) return fail(CH_EINVAL, "num_hidden_layers must be 1..64");
  if (c->head_dim != 256) return fail(CH_EINVAL, "head_dim must be 256");
  if (c->rotary_dim == 0 || c->rotary_dim > c->head_dim || (c->rotary_dim & 1))
    return fail(CH_EINVAL, "rotary_dim must be even and <= head_dim");
  if (c->num_key_value_heads == 0 || c->num_attention_heads % c->num_key_value_heads)
    return fail(CH_EINVAL, "num_attention_heads must be a multiple of num_key_value_heads");
  uint32_t r = c->num_attention_heads / c->num_key_value_heads;
  if (r != 1 && r != 2 && r != 4 && r != 8) return fail(CH_EINVAL, "GQA ratio must be 1, 2, 4 or 8");
  if (c->hidden_size % 64 || c->intermediate_size % 64) return fail(CH_EINVAL, "hidden/intermediate must be % 64");
  if (c->vocab_size % 16 || c->vocab_size > 262144) return fail(CH_EINVAL, "vocab must be % 16 and <= 262144");
  if (c->hidden_size % 32) return fail(CH_EINVAL, "hidden % 32");
  return CH_OK;
}

template <typename T>
static int dmalloc(T **p, size_t n) {
  cudaError_t e = cudaMalloc((void **)p, n * sizeof(T) > 0 ? n * sizeof(T) : 16);
  if (e != cudaSuccess) return fail(CH_ENOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  return CH_OK;
}
#define CH_TRY(x)          \
  do {                     \
    int _r = (x);          \
    if (_r != CH_OK) return _r; \
  } while (0)

static int alloc_model_buffers(ch_model *m) {
  const ch_model_config &c = m->cfg;
  m->H = c.hidden_size;
  m->I = c.intermediate_size;
  m->V = c.vocab_size;
  m->D = c.head_dim;
  m->nq = c.num_attention_heads;
  m->nkv = c.num_key_value_heads;
  m->qd = m->nq * m->D;
  m->kvd = m->nkv * m->D;
  m->L = c.num_hidden_layers;
  const uint32_t P = m->world;
  m->nq_l = m->nq / P;
  m->nkv_l = m->nkv / P;
  m->qd_l = m->nq_l * m->D;
  m->kvd_l = m->nkv_l * m->D;
  m->Il = m->I / P;
  m->Vl = m->V / P;
  m->layers.resize(m->L);
  for (uint32_t l = 0; l < m->L; l++) {
    DevLayer &dl = m->layers[l];
    dl.full = c.layer_types[l] != 0;
    CH_TRY(dmalloc(&dl.qkv, q4_tile_bytes(m->qd_l + 2 * m->kvd_l, m->H)));
    CH_TRY(dmalloc(&dl.o, q4_tile_bytes(m->H, m->qd_l)));  // row-parallel shards: all rows, this rank's columns
    CH_TRY(dmalloc(&dl.gateup, q4_tile_bytes(2 * m->Il, m->H)));
    CH_TRY(dmalloc(&dl.down, q4_tile_bytes(m->H, m->Il)));
    CH_TRY(dmalloc(&dl.input_norm, m->H));
    CH_TRY(dmalloc(&dl.q_norm, m->D));
    CH_TRY(dmalloc(&dl.k_norm, m->D));
    CH_TRY(dmalloc(&dl.pre_ffn, m->H));
    CH_TRY(dmalloc(&dl.kc, (size_t)kSlots * m->kvd_l));
    CH_TRY(dmalloc(&dl.vc, (size_t)kSlots * m->kvd_l));
    CH_CUDA(cudaMemsetAsync(dl.kc, 0, (size_t)kSlots * m->kvd_l * 2, m->ctx->stream));
    CH_CUDA(cudaMemsetAsync(dl.vc, 0, (size_t)kSlots * m->kvd_l * 2, m->ctx->stream));
  }
  CH_TRY(dmalloc(&m->lm, q8_tile_bytes(m->Vl, m->H)));
  CH_TRY(dmalloc(&m->final_norm, m->H));
  CH_TRY(dmalloc(&m->inv_freq_s, c.rotary_dim / 2));
  CH_TRY(dmalloc(&m->inv_freq_f, c.rotary_dim / 2));
  CH_TRY(dmalloc(&m->X[0], m->H));
  CH_TRY(dmalloc(&m->X[1], m->H));
  CH_TRY(dmalloc(&m->normed, m->H));
  CH_TRY(dmalloc(&m->qkv, m->qd + 2 * m->kvd));
  CH_TRY(dmalloc(&m->attn, m->qd));
  CH_TRY(dmalloc(&m->o_out, m->H));
  CH_TRY(dmalloc(&m->act, m->I));
  CH_TRY(dmalloc(&m->down_out, m->H));
  CH_TRY(dmalloc(&m->logits, m->V));
  CH_TRY(dmalloc(&m->vals, 64));
  CH_TRY(dmalloc(&m->ids, 64));
  CH_TRY(dmalloc(&m->token, 1));
  CH_TRY(dmalloc(&m->sp, 1));
  CH_TRY(dmalloc(&m->active, kSlots));
  CH_TRY(dmalloc(&m->sliding, kSlots));
  CH_CUDA(cudaMemsetAsync(m->X[0], 0, m->H * 4, m->ctx->stream));
  CH_CUDA(cudaMemsetAsync(m->X[1], 0, m->H * 4, m->ctx->stream));
  CH_CUDA(cudaMemsetAsync(m->sp, 0, sizeof(StepParams), m->ctx->stream));
  CH_CUDA(cudaMemsetAsync(m->token, 0, 4, m->ctx->stream));
  // scratch
  const int grid = gemv_default_grid();
  CH_TRY(dmalloc(&m->gemv_partial, gemv_partial_floats(grid)));
  const uint32_t max_rt = std::max({(m->qd + 2 * m->kvd) / 16, m->H / 16, 2 * m->I / 16, m->V / 16});
  CH_TRY(dmalloc(&m->gemv_counters, max_rt));
  CH_CUDA(cudaMemsetAsync(m->gemv_counters, 0, max_rt * 4, m->ctx->stream));
  m->attn_splits = attn_default_splits(m->nkv);
  CH_TRY(dmalloc(&m->attn_partial, attn_partial_floats(m->nkv, m->nq / m->nkv, m->D, m->attn_splits)));
  CH_TRY(dmalloc(&m->attn_counters, m->nkv));
  CH_CUDA(cudaMemsetAsync(m->attn_counters, 0, m->nkv * 4, m->ctx->stream));
  CH_TRY(dmalloc(&m->topk_cand, (size_t)std::max(topk_blocks(m->V), num_sms()) * 64));
  CH_TRY(dmalloc(&m->topk_counter, 1));
  CH_CUDA(cudaMemsetAsync(m->topk_counter, 0, 4, m->ctx->stream));
  // pinned staging
  CH_CUDA(cudaMallocHost(&m->h_x, m->H * sizeof(float)));
  CH_CUDA(cudaMallocHost(&m->h_sp, sizeof(StepParams)));
  CH_CUDA(cudaMallocHost(&m->h_lists, 2 * kSlots * sizeof(uint32_t)));
  CH_CUDA(cudaMallocHost(&m->h_ids, 64 * sizeof(uint32_t)));
  CH_CUDA(cudaMallocHost(&m->h_status, sizeof(uint32_t)));
  CH_CUDA(cudaMallocHost(&m->h_vals, 64 * sizeof(float)));
  CH_CUDA(cudaMallocHost(&m->h_run, 2 * sizeof(uint32_t)));
  // RoPE inverse frequencies: same formula as the oracle (double pow, one rounding)
  std::vector<float> fs(c.rotary_dim / 2), ff(c.rotary_dim / 2);
  for (uint32_t i = 0; i < c.rotary_dim / 2; i++) {
    float e = (2.0f * (float)i) / (float)c.rotary_dim;
    fs[i] = (float)(1.0 / pow((double)c.rope_theta, (double)e));
    ff[i] = (float)(1.0 / pow((double)c.rope_theta_full, (double)e));
  }
  CH_CUDA(cudaMemcpy(m->inv_freq_s, fs.data(), fs.size() * 4, cudaMemcpyHostToDevice));
  CH_CUDA(cudaMemcpy(m->inv_freq_f, ff.data(), ff.size() * 4, cudaMemcpyHostToDevice));
  m->h_inv_s = fs;
  m->h_inv_f = ff;
  CH_TRY(dmalloc(&m->rope_cs, c.rotary_dim));
  CH_CUDA(cudaMallocHost(&m->h_rope, c.rotary_dim * sizeof(float2)));
  return CH_OK;
}

// ---------------------------------------------------------------------------
// phase table of the persistent decode-step kernel (decode_step.cu)
enum GemvKind { GK_QKV = 0, GK_O = 1, GK_GU = 2, GK_DOWN = 3, GK_LM = 4 };

static int build_phases(ch_model *m, bool with_logits, Phase **d_out, uint32_t *n_out, StreamDesc **d_str,
                        uint32_t *n_str, uint32_t *n_cross, uint32_t *n_local, uint32_t *n_x, Partition *kpart) {
  static_assert(GK_LM + 1 == kKinds, "one partition per GEMV kind");
  const uint32_t G = (uint32_t)m->mk_grid, GW = G * mk_warps();
  const bool tp = m->world > 1;
  // Local output rows of each GEMV and its k tiles.  Tensor parallel (Megatron
  // layout): q|k|v and gate|up are column-parallel (this rank's heads / act rows, full
  // K), o and down row-parallel (all H rows over this rank's K columns); each rank
  // sends its o / down partial vector to slot `rank` of every rank's arena and the
  // next add+norm prologue adds the world partials -- two exchanges per layer.
  const uint32_t rows[5] = {m->qd_l + 2 * m->kvd_l, m->H, 2 * m->Il, m->H, m->Vl};
  const uint32_t KT[5] = {m->H / 64, m->qd_l / 64, m->H / 64, m->Il / 64, m->H / 32};
  const bool gathered[5] = {false, tp, false, tp, false};
  float *dst[5] = {m->gdir[GK_QKV], m->gdir[GK_O], m->gdir[GK_GU], m->gdir[GK_DOWN], m->gdir[GK_LM]};
  uint32_t row0[5] = {0, 0, 0, 0, 0};
  const uint32_t nsum = tp ? m->world : 1u;
  if (tp) {  // low-latency exchange arrays [2 parities][world][H] of {value, epoch} words
    dst[GK_O] = reinterpret_cast<float *>(m->arena + m->off_o);
    dst[GK_DOWN] = reinterpret_cast<float *>(m->arena + m->off_down);
    row0[GK_O] = row0[GK_DOWN] = m->H;
  }
  GemvOut outs[5];
  for (int k = 0; k < 5; k++) {
    const uint64_t T = (uint64_t)(rows[k] / 16) * KT[k];
    Partition pt{KT[k], (uint32_t)(T / GW), (uint32_t)(T % GW), 0u, 0u, 0u};
    if (gathered[k]) {  // whole row tiles per CTA: every row finished inside one CTA, then sent to all ranks
      pt.aligned = 1;
      pt.rq = (rows[k] / 16) / G;
      pt.rrem = (rows[k] / 16) % G;
    }
    outs[k] = GemvOut{dst[k], m->gpart[k], pt, k == GK_GU ? 1u : 0u, row0[k], gathered[k] ? 2u : 0u, 0u, (uint32_t)k};
  }
  auto gemv = [&](int kind, const uint8_t *tiles, int fmt, uint32_t K) {
    Phase p{};
    p.kind = PH_GEMV;
    p.fmt = fmt;
    p.tiles = tiles;
    p.row_tiles = rows[kind] / 16;
    p.k_tiles = KT[kind];
    p.K = K;
    p.out = outs[kind];
    p.scalar = 1.0f;
    return p;
  };
  float *attn_in = m->attn;  // this rank's heads only (row-parallel o)
  std::vector<Phase> ph;
  const uint32_t rh = m->cfg.rotary_dim / 2;
  uint32_t nx = 0;          // exchanges numbered in phase order: o of layer l = 2l, down = 2l + 1
  GemvOut prev_down{};      // the previous layer's down output (its exchange index)
  for (uint32_t l = 0; l < m->L; l++) {
    const DevLayer &dl = m->layers[l];
    Phase q = gemv(GK_QKV, dl.qkv, FMT_Q4, m->H);
    q.norm_w = dl.input_norm;
    q.normed_out = m->normed;
    if (l == 0) {
      q.pm = PM_NORM;
      q.x_in = m->X[0];
    } else {
      const DevLayer &pl = m->layers[l - 1];
      q.pm = PM_ADD_NORM;
      q.x_in = m->X[1];
      q.r_in = prev_down;
      q.nsum = nsum;
      q.post_w = pl.post_ffn;
      q.scalar = pl.scalar;
      q.x_out = m->X[0];
    }
    ph.push_back(q);
    Phase at{};
    at.kind = PH_ATTN;
    at.r_in = outs[GK_QKV];
    at.q_norm_w = dl.q_norm;
    at.k_norm_w = dl.k_norm;
    at.rope_cs = m->rope_cs + (dl.full ? rh : 0);
    at.k_cache = dl.kc;
    at.v_cache = dl.vc;
    at.is_sliding = dl.full ? 0 : 1;
    at.attn_scale = 1.0f;  // Gemma-style: q/k norms replace 1/sqrt(d) (forward.zig:85)
    at.attn_out = attn_in;
    ph.push_back(at);
    Phase o = gemv(GK_O, dl.o, FMT_Q4, m->qd_l);
    if (o.out.push == 2) o.out.xidx = nx++;
    o.pm = PM_DIRECT;
    o.x_in = attn_in;
    ph.push_back(o);
    Phase gu = gemv(GK_GU, dl.gateup, FMT_Q4, m->H);
    gu.pm = PM_ADD_NORM;
    gu.x_in = m->X[0];
    gu.r_in = o.out;
    gu.nsum = nsum;
    gu.post_w = dl.post_attn;
    gu.norm_w = dl.pre_ffn;
    gu.x_out = m->X[1];
    gu.normed_out = m->normed;
    ph.push_back(gu);
    Phase dn = gemv(GK_DOWN, dl.down, FMT_Q4, m->Il);
    if (dn.out.push == 2) dn.out.xidx = nx++;
    prev_down = dn.out;
    dn.pm = PM_GELU;
    dn.r_in = outs[GK_GU];
    ph.push_back(dn);
  }
  const DevLayer &last = m->layers[m->L - 1];
  Phase lm = gemv(GK_LM, m->lm, FMT_Q8, m->H);
  lm.pm = PM_ADD_NORM;
  lm.x_in = m->X[1];
  lm.r_in = prev_down;
  lm.nsum = nsum;
  lm.post_w = last.post_ffn;
  lm.scalar = last.scalar;
  lm.norm_w = m->final_norm;
  lm.x_out = m->X[0];
  lm.normed_out = m->normed;
  if (!with_logits) {  // prologue only: fold the last residual add + final norm
    lm.row_tiles = 0;
    lm.out.pt.q = lm.out.pt.rem = 0;
  }
  for (int k = 0; k < 5; k++) kpart[k] = k == GK_LM ? lm.out.pt : outs[k].pt;
  ph.push_back(lm);
  if (with_logits) {
    Phase tk{};
    tk.kind = PH_TOPK;
    tk.r_in = outs[GK_LM];
    tk.vocab = m->Vl;
    tk.vocab0 = m->rank * m->Vl;
    ph.push_back(tk);
    if (tp) {
      Phase mg{};
      mg.kind = PH_MERGE;
      ph.push_back(mg);
    }
  }
  // After a phase whose outputs are exchange words (tensor parallel o and down
  // partials) there is no barrier: the next phase's prologue polls the words.  After
  // the top-64 phase a cross-rank barrier; after every other phase a grid barrier.
  uint32_t ncross = 0, nlocal = 0;
  for (size_t i = 0; i + 1 < ph.size(); i++) {
    Phase &p = ph[i];
    p.nobar = (p.kind == PH_GEMV && p.out.push == 2) ? 1u : 0u;
    p.cross = (tp && p.kind == PH_TOPK) ? 1u : 0u;
    if (p.cross) ncross++;
    if (!p.nobar) nlocal++;
    p.gidx = ncross;
    p.lidx = nlocal;
  }
  *n_cross = ncross;
  *n_local = nlocal;
  *n_x = nx;
  CH_TRY(dmalloc(d_out, ph.size()));
  CH_CUDA(cudaMemcpy(*d_out, ph.data(), ph.size() * sizeof(Phase), cudaMemcpyHostToDevice));
  *n_out = (uint32_t)ph.size();
  std::vector<StreamDesc> st;
  for (const Phase &p : ph)
    if (p.kind == PH_GEMV) st.push_back(StreamDesc{p.tiles, p.out.pt});
  CH_TRY(dmalloc(d_str, st.size()));
  CH_CUDA(cudaMemcpy(*d_str, st.data(), st.size() * sizeof(StreamDesc), cudaMemcpyHostToDevice));
  *n_str = (uint32_t)st.size();
  return CH_OK;
}

// attention splits per kv head in the decode-step kernel: at most one CTA per
// (kv head, split) and no more than its combine keeps in registers
static uint32_t mk_attn_splits(const ch_model *m) {
  return (uint32_t)std::min({m->mk_grid / (int)m->nkv_l, m->attn_splits, (int)kMkMaxSplits});
}

// The decode step runs as one persistent kernel (decode_step.cu) when the shape
// fits it; otherwise -- or with CH_DECODE_OPS=1, for A/B measurement -- as the
// captured graph of per-op kernels.  Both are GPU paths with the same results.
// A tensor-parallel shard always uses the persistent kernel (the per-op graph
// has no exchange step).
static int init_decode_step(ch_model *m) {
  m->mk_grid = std::min(num_sms(), 255);  // straddle lists hold CTA ids in 8 bits
  const bool tp = m->world > 1;
  const char *env = getenv("CH_DECODE_OPS");
  m->use_ops = !tp && env && env[0] == '1';
  const uint32_t ratio = m->nq / m->nkv;
  const uint32_t max_k = std::max({m->H, m->qd, m->I});
  m->mk_smem = mk_smem_bytes(max_k, m->H, ratio, mk_attn_splits(m), kSlots, (uint32_t)m->mk_grid);
  int co = 0;
  CH_CUDA(cudaDeviceGetAttribute(&co, cudaDevAttrCooperativeLaunch, m->ctx->device));
  const bool fits = co && m->H <= 4096 && m->D == 256 && (ratio == 1 || ratio == 2 || ratio == 4) &&
                    (m->Vl + m->mk_grid - 1) / m->mk_grid <= 4096 && m->mk_smem <= 226 * 1024;
  if (!fits) {
    if (tp) return fail(CH_EINVAL, "tensor-parallel decode needs the persistent decode kernel; shape does not fit it");
    m->use_ops = true;
  }
  if (m->use_ops) return CH_OK;
  const size_t part = (size_t)m->mk_grid * mk_warps() * 2 * 16;
  const uint32_t rows[5] = {m->qd_l + 2 * m->kvd_l, m->H, 2 * m->I, m->H, m->Vl};
  for (int k = 0; k < 5; k++) {
    CH_TRY(dmalloc(&m->gdir[k], rows[k]));
    CH_TRY(dmalloc(&m->gpart[k], part));
  }
  CH_TRY(dmalloc(&m->mk_arrive, 1));
  CH_TRY(dmalloc(&m->mk_base, 3));
  CH_CUDA(cudaMemset(m->mk_arrive, 0, 8));
  CH_CUDA(cudaMemset(m->mk_base, 0, 24));
  if (tp) {
    // exchange arena: arrival counter, the o and down exchange arrays
    // ([2 parities][world][H] {value, epoch} words), every rank's top-64 -- same
    // offsets on every rank
    auto take = [&](size_t bytes) {
      const size_t o = m->arena_bytes;
      m->arena_bytes += (bytes + 255) & ~(size_t)255;
      return o;
    };
    m->off_arrive = take(8);
    m->off_o = take((size_t)2 * m->world * m->H * 8);
    m->off_down = take((size_t)2 * m->world * m->H * 8);
    m->off_cand = take((size_t)m->world * 64 * 8);
    CH_TRY(dmalloc(&m->arena, m->arena_bytes));
    CH_CUDA(cudaMemset(m->arena, 0, m->arena_bytes));
  }
  CH_TRY(build_phases(m, true, &m->d_phases, &m->n_phases, &m->d_streams, &m->n_streams, &m->n_cross,
                      &m->n_local, &m->n_x, m->kpart[0]));
  CH_TRY(build_phases(m, false, &m->d_phases_nl, &m->n_phases_nl, &m->d_streams_nl, &m->n_streams_nl,
                      &m->n_cross_nl, &m->n_local_nl, &m->n_x_nl, m->kpart[1]));
  return CH_OK;
}

static MegaArgs mega_args(ch_model *m, bool logits, bool device_loop) {
  MegaArgs a{};
  a.phases = logits ? m->d_phases : m->d_phases_nl;
  a.nphases = logits ? m->n_phases : m->n_phases_nl;
  a.streams = logits ? m->d_streams : m->d_streams_nl;
  for (uint32_t k = 0; k < kKinds; k++) a.kpart[k] = m->kpart[logits ? 0 : 1][k];
  a.nstreams = logits ? m->n_streams : m->n_streams_nl;
  a.grid = (uint32_t)m->mk_grid;
  a.arrive = m->mk_arrive;
  a.base = m->mk_base;
  a.garrive = m->arena ? reinterpret_cast<unsigned long long *>(m->arena + m->off_arrive) : nullptr;
  a.ncross = logits ? m->n_cross : m->n_cross_nl;
  a.nlocal = logits ? m->n_local : m->n_local_nl;
  a.nx = logits ? m->n_x : m->n_x_nl;
  a.err = m->ctx->err;
  a.sp = m->sp;
  a.sp_rw = device_loop ? m->sp : nullptr;
  a.nq = m->nq_l;
  a.nkv = m->nkv_l;
  a.world = m->world;
  a.rank = m->rank;
  a.attn_q0 = m->rank * m->nq_l;
  a.attn_local = 1;
  for (uint32_t r = 0; r < m->world && r < kMaxWorld; r++) a.arena[r] = m->peer_arena[r];
  a.xcand = m->arena ? reinterpret_cast<uint64_t *>(m->arena + m->off_cand) : nullptr;
  a.rot = m->cfg.rotary_dim;
  a.attn_max_splits = mk_attn_splits(m);
  a.cache_slots = kSlots;
  a.eps = m->cfg.rms_norm_eps;
  a.attn_partial = m->attn_partial;
  a.attn_counters = m->attn_counters;
  a.topk_cand = m->topk_cand;
  a.topk_counter = m->topk_counter;
  a.ids = m->ids;
  a.vals = m->vals;
  a.token_out = m->token;
  a.token_hist = device_loop ? m->token_hist : nullptr;
  a.hist_cap = m->hist_cap;
  return a;
}

// upload quant.zig Q4 blocks of one matrix into a temp device buffer
static int upload_blocks(ch_model *m, const uint32_t *host, uint32_t rows, uint32_t cols, uint32_t *tmp) {
  if (!host) return fail(CH_EINVAL, "NULL weight pointer");
  CH_CUDA(cudaMemcpyAsync(tmp, host, (size_t)rows * (cols / 32) * 5 * 4, cudaMemcpyHostToDevice, m->ctx->stream));
  return CH_OK;
}

extern "C" int ch_model_create(ch_ctx *ctx, const ch_model_config *cfg, const ch_layer_weights *lw,
                               const uint32_t *lm_head_q8, const float *final_norm, const uint16_t *embed_bf16,
                               ch_model **out) {
  if (!ctx || !out || !lw || !lm_head_q8 || !final_norm) return fail(CH_EINVAL, "NULL argument");
  CH_TRY(check_cfg(cfg));
  CH_CUDA(cudaSetDevice(ctx->device));
  ch_model *m = new ch_model();
  m->ctx = ctx;
  m->cfg = *cfg;
  int r = alloc_model_buffers(m);
  if (r != CH_OK) {
    free_model(m);
    return r;
  }
  cudaStream_t s = ctx->stream;
  // temp block buffers sized for the largest matrix
  size_t max_words = std::max({(size_t)(m->qd + 2 * m->kvd) * (m->H / 32) * 5, (size_t)m->H * (m->qd / 32) * 5,
                               (size_t)m->I * (m->H / 32) * 5, (size_t)m->H * (m->I / 32) * 5});
  uint32_t *tA = nullptr, *tB = nullptr;
  auto bail = [&](int code) {
    cudaFree(tA);
    cudaFree(tB);
    free_model(m);
    return code;
  };
  if (dmalloc(&tA, max_words) != CH_OK || dmalloc(&tB, max_words) != CH_OK) return bail(CH_ENOMEM);
  const size_t qw = (size_t)m->qd * (m->H / 32) * 5, kw = (size_t)m->kvd * (m->H / 32) * 5;
  for (uint32_t l = 0; l < m->L; l++) {
    const ch_layer_weights &w = lw[l];
    DevLayer &dl = m->layers[l];
    if (!w.q_proj || !w.k_proj || !w.v_proj || !w.o_proj || !w.gate_proj || !w.up_proj || !w.down_proj ||
        !w.input_norm || !w.q_norm || !w.k_norm || !w.pre_ffn_norm)
      return bail(fail(CH_EINVAL, "layer " + std::to_string(l) + ": NULL weight"));
    // q|k|v concatenated rows
    if (upload_blocks(m, w.q_proj, m->qd, m->H, tA) || upload_blocks(m, w.k_proj, m->kvd, m->H, tA + qw) ||
        upload_blocks(m, w.v_proj, m->kvd, m->H, tA + qw + kw))
      return bail(CH_ECUDA);
    if (launch_repack_q4(tA, nullptr, m->qd + 2 * m->kvd, m->H, MAP_PLAIN, dl.qkv, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack qkv"));
    if (upload_blocks(m, w.o_proj, m->H, m->qd, tB)) return bail(CH_ECUDA);
    if (launch_repack_q4(tB, nullptr, m->H, m->qd, MAP_PLAIN, dl.o, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack o"));
    cudaStreamSynchronize(s);
    if (upload_blocks(m, w.gate_proj, m->I, m->H, tA) || upload_blocks(m, w.up_proj, m->I, m->H, tB))
      return bail(CH_ECUDA);
    if (launch_repack_q4(tA, tB, 2 * m->I, m->H, MAP_GATEUP, dl.gateup, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack gate/up"));
    cudaStreamSynchronize(s);
    if (upload_blocks(m, w.down_proj, m->H, m->I, tA)) return bail(CH_ECUDA);
    if (launch_repack_q4(tA, nullptr, m->H, m->I, MAP_PLAIN, dl.down, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack down"));
    auto up = [&](float **dst, const float *src, uint32_t n, bool optional) -> int {
      if (!src) {
        if (optional) return CH_OK;
        return fail(CH_EINVAL, "NULL norm");
      }
      if (!*dst && dmalloc(dst, n) != CH_OK) return CH_ENOMEM;
      CH_CUDA(cudaMemcpyAsync(*dst, src, n * 4, cudaMemcpyHostToDevice, s));
      return CH_OK;
    };
    if (up(&dl.input_norm, w.input_norm, m->H, false) || up(&dl.q_norm, w.q_norm, m->D, false) ||
        up(&dl.k_norm, w.k_norm, m->D, false) || up(&dl.pre_ffn, w.pre_ffn_norm, m->H, false) ||
        up(&dl.post_attn, w.post_attn_norm, m->H, true) || up(&dl.post_ffn, w.post_ffn_norm, m->H, true))
      return bail(CH_ECUDA);
    dl.scalar = w.layer_scalar;
    cudaStreamSynchronize(s);
  }
  cudaFree(tA);
  cudaFree(tB);
  tA = tB = nullptr;
  // LM head Q8_0 blocks: upload in row chunks, repack per chunk
  {
    const uint32_t chunk_rows = 16384;
    uint32_t *tq = nullptr;
    if (dmalloc(&tq, (size_t)chunk_rows * (m->H / 32) * 9) != CH_OK) return bail(CH_ENOMEM);
    for (uint32_t r0 = 0; r0 < m->V; r0 += chunk_rows) {
      uint32_t nr = std::min(chunk_rows, m->V - r0);
      cudaMemcpyAsync(tq, lm_head_q8 + (size_t)r0 * (m->H / 32) * 9, (size_t)nr * (m->H / 32) * 9 * 4,
                      cudaMemcpyHostToDevice, s);
      launch_repack_q8(tq, nr, m->H, m->lm + q8_tile_bytes(r0, m->H), s);
      cudaStreamSynchronize(s);
    }
    cudaFree(tq);
  }
  if (cudaMemcpyAsync(m->final_norm, final_norm, m->H * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
    return bail(fail(CH_ECUDA, "final norm upload"));
  if (embed_bf16) {
    if (dmalloc(&m->embed, (size_t)m->V * m->H) != CH_OK) return bail(CH_ENOMEM);
    if (cudaMemcpyAsync(m->embed, embed_bf16, (size_t)m->V * m->H * 2, cudaMemcpyHostToDevice, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "embed upload"));
  }
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return bail(fail(CH_ECUDA, std::string("model upload: ") + cudaGetErrorString(e)));
  if (int r2 = init_decode_step(m)) return bail(r2);
  *out = m;
  return CH_OK;
}

// GpuModelContext.init with quantize-on-load (src/gpu/model_gpu.zig:44-55,109-127,157):
// the caller hands over the bf16 weights it mapped from safetensors; every projection
// is uploaded and quantized to Q4_0 on the device (quantizeRowQ4_0, quant.zig:58-98 --
// the same kernel as ch_quantize_q4_rows, bit-exact with quant.zig), then repacked like
// ch_model_create's blocks; the tied embedding becomes the Q8_0 LM head
// (model_gpu.zig:157) and stays on the device for the embedding lookup.  Norms are
// bf16 -> f32 (createNormBuffer, model_gpu.zig:57-66): a NULL input / q / k / pre-FFN /
// final norm is all ones like a missing tensor there, a NULL post-attention / post-FFN
// norm means the layer has none (has_post_*_norm, model_dispatch.zig:35,41); a NULL
// v_proj takes k_proj (attention_k_eq_v, model_gpu.zig:114).
extern "C" int ch_model_create_bf16(ch_ctx *ctx, const ch_model_config *cfg, const ch_layer_weights_bf16 *lw,
                                    const uint16_t *embed_bf16, const uint16_t *final_norm_bf16, ch_model **out) {
  if (!ctx || !out || !lw || !embed_bf16) return fail(CH_EINVAL, "NULL argument (the tied embedding is required)");
  CH_TRY(check_cfg(cfg));
  CH_CUDA(cudaSetDevice(ctx->device));
  ch_model *m = new ch_model();
  m->ctx = ctx;
  m->cfg = *cfg;
  int r = alloc_model_buffers(m);
  if (r != CH_OK) {
    free_model(m);
    return r;
  }
  cudaStream_t s = ctx->stream;
  const size_t max_elems = std::max({(size_t)m->qd * m->H, (size_t)m->kvd * m->H, (size_t)m->I * m->H});
  size_t max_words = std::max({(size_t)(m->qd + 2 * m->kvd) * (m->H / 32) * 5, (size_t)m->H * (m->qd / 32) * 5,
                               (size_t)m->I * (m->H / 32) * 5, (size_t)m->H * (m->I / 32) * 5});
  uint32_t *tA = nullptr, *tB = nullptr;
  uint16_t *tb = nullptr;
  auto bail = [&](int code) {
    cudaFree(tA);
    cudaFree(tB);
    cudaFree(tb);
    free_model(m);
    return code;
  };
  if (dmalloc(&tA, max_words) != CH_OK || dmalloc(&tB, max_words) != CH_OK || dmalloc(&tb, max_elems) != CH_OK)
    return bail(CH_ENOMEM);
  // one bf16 matrix (rows x cols, row-major) -> quant.zig Q4 blocks at dst
  auto quant = [&](const uint16_t *host, uint32_t rows, uint32_t cols, uint32_t *dst) -> int {
    if (!host) return fail(CH_EINVAL, "NULL weight pointer");
    CH_CUDA(cudaMemcpyAsync(tb, host, (size_t)rows * cols * 2, cudaMemcpyHostToDevice, s));
    CH_CUDA(launch_quantize_q4_rows(tb, rows, cols, dst, s));
    CH_CUDA(cudaStreamSynchronize(s));  // tb is reused by the next matrix
    return CH_OK;
  };
  // bf16 norm -> f32 on the device; NULL: all ones, or (optional) no norm at all
  auto norm = [&](float **dst, const uint16_t *host, uint32_t n, bool optional) -> int {
    if (!host && optional) return CH_OK;
    if (!*dst) CH_TRY(dmalloc(dst, n));
    if (host) {
      CH_CUDA(cudaMemcpyAsync(tb, host, (size_t)n * 2, cudaMemcpyHostToDevice, s));
      CH_CUDA(launch_bf16_to_f32(tb, *dst, n, s));
    } else {
      const std::vector<float> ones(n, 1.0f);
      CH_CUDA(cudaMemcpyAsync(*dst, ones.data(), (size_t)n * 4, cudaMemcpyHostToDevice, s));
    }
    CH_CUDA(cudaStreamSynchronize(s));
    return CH_OK;
  };
  const size_t qw = (size_t)m->qd * (m->H / 32) * 5, kw = (size_t)m->kvd * (m->H / 32) * 5;
  for (uint32_t l = 0; l < m->L; l++) {
    const ch_layer_weights_bf16 &w = lw[l];
    DevLayer &dl = m->layers[l];
    int rc = CH_OK;
    auto lfail = [&](const char *what) { return bail(fail(rc, "layer " + std::to_string(l) + " " + what + ": " + g_err)); };
    if ((rc = quant(w.q_proj, m->qd, m->H, tA)) || (rc = quant(w.k_proj, m->kvd, m->H, tA + qw)) ||
        (rc = quant(w.v_proj ? w.v_proj : w.k_proj, m->kvd, m->H, tA + qw + kw)))
      return lfail("q|k|v");
    if (launch_repack_q4(tA, nullptr, m->qd + 2 * m->kvd, m->H, MAP_PLAIN, dl.qkv, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack qkv"));
    if ((rc = quant(w.o_proj, m->H, m->qd, tB))) return lfail("o_proj");
    if (launch_repack_q4(tB, nullptr, m->H, m->qd, MAP_PLAIN, dl.o, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack o"));
    CH_CUDA(cudaStreamSynchronize(s));
    if ((rc = quant(w.gate_proj, m->I, m->H, tA)) || (rc = quant(w.up_proj, m->I, m->H, tB))) return lfail("gate/up");
    if (launch_repack_q4(tA, tB, 2 * m->I, m->H, MAP_GATEUP, dl.gateup, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack gate/up"));
    CH_CUDA(cudaStreamSynchronize(s));
    if ((rc = quant(w.down_proj, m->H, m->I, tA))) return lfail("down_proj");
    if (launch_repack_q4(tA, nullptr, m->H, m->I, MAP_PLAIN, dl.down, s) != cudaSuccess)
      return bail(fail(CH_ECUDA, "repack down"));
    CH_CUDA(cudaStreamSynchronize(s));
    if ((rc = norm(&dl.input_norm, w.input_norm, m->H, false)) || (rc = norm(&dl.q_norm, w.q_norm, m->D, false)) ||
        (rc = norm(&dl.k_norm, w.k_norm, m->D, false)) || (rc = norm(&dl.pre_ffn, w.pre_ffn_norm, m->H, false)) ||
        (rc = norm(&dl.post_attn, w.post_attn_norm, m->H, true)) ||
        (rc = norm(&dl.post_ffn, w.post_ffn_norm, m->H, true)))
      return lfail("norms");
    dl.scalar = w.layer_scalar;
  }
  if (int rc = norm(&m->final_norm, final_norm_bf16, m->H, false)) return bail(rc);
  cudaFree(tA);
  cudaFree(tB);
  cudaFree(tb);
  tA = tB = nullptr;
  tb = nullptr;
  if (dmalloc(&m->embed, (size_t)m->V * m->H) != CH_OK) return bail(CH_ENOMEM);
  if (cudaMemcpyAsync(m->embed, embed_bf16, (size_t)m->V * m->H * 2, cudaMemcpyHostToDevice, s) != cudaSuccess)
    return bail(fail(CH_ECUDA, "embed upload"));
  {
    const uint32_t chunk_rows = 16384;
    uint32_t *tq = nullptr;
    if (dmalloc(&tq, (size_t)chunk_rows * (m->H / 32) * 9) != CH_OK) return bail(CH_ENOMEM);
    for (uint32_t r0 = 0; r0 < m->V; r0 += chunk_rows) {
      const uint32_t nr = std::min(chunk_rows, m->V - r0);
      launch_quantize_q8_rows(m->embed + (size_t)r0 * m->H, nr, m->H, tq, s);
      launch_repack_q8(tq, nr, m->H, m->lm + q8_tile_bytes(r0, m->H), s);
    }
    cudaStreamSynchronize(s);
    cudaFree(tq);
  }
  const cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return bail(fail(CH_ECUDA, std::string("bf16 model upload: ") + cudaGetErrorString(e)));
  if (int r2 = init_decode_step(m)) return bail(r2);
  *out = m;
  return CH_OK;
}

// tensor ids of the synthetic generator (shared with tests/ and the oracle driver)
enum : uint32_t {
  T_Q = 0, T_K = 1, T_V = 2, T_O = 3, T_GATE = 4, T_UP = 5, T_DOWN = 6,
  T_IN_NORM = 10, T_Q_NORM = 11, T_K_NORM = 12, T_POST_ATTN = 13, T_PRE_FFN = 14, T_POST_FFN = 15,
  T_EMBED = 20, T_FINAL_NORM = 21,
};

static uint64_t host_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
extern "C" uint64_t ch_tensor_seed(uint64_t seed, uint32_t layer, uint32_t tensor_id) {
  return host_mix64(host_mix64(seed) ^ (((uint64_t)layer << 16) | tensor_id));
}

static int gen_norm(ch_model *m, float **dst, uint32_t n, uint64_t tseed, uint16_t *tmp) {
  if (!*dst) CH_TRY(dmalloc(dst, n));
  if (launch_gen_bf16(tmp, n, tseed, 1.0f, 0.02f, m->ctx->stream) != cudaSuccess) return fail(CH_ECUDA, "gen norm");
  if (launch_bf16_to_f32(tmp, *dst, n, m->ctx->stream) != cudaSuccess) return fail(CH_ECUDA, "norm convert");
  return CH_OK;
}

// Synthetic weights of shard `rank` of `world`: every tensor is generated as rows
// [row0, row0 + rows) of the whole-model tensor, so the shards of a tensor-parallel
// model are exactly the rows of ch_model_create_synthetic's weights.
static int create_synthetic(ch_ctx *ctx, const ch_model_config *cfg, uint64_t seed, uint32_t rank, uint32_t world,
                            ch_model **out) {
  if (!ctx || !out) return fail(CH_EINVAL, "NULL argument");
  CH_TRY(check_cfg(cfg));
  if (world == 0 || world > kMaxWorld || rank >= world) return fail(CH_EINVAL, "rank must be < world <= 8");
  if (world > 1 && (cfg->num_key_value_heads % world || cfg->intermediate_size % (64 * world) ||
                    cfg->vocab_size % (16 * world) || (cfg->num_attention_heads / world * cfg->head_dim) % 64))
    return fail(CH_EINVAL, "tensor parallel: kv heads, intermediate/64, vocab/16 and the per-rank q width/64 must divide by world");
  CH_CUDA(cudaSetDevice(ctx->device));
  ch_model *m = new ch_model();
  m->ctx = ctx;
  m->cfg = *cfg;
  m->rank = rank;
  m->world = world;
  int r = alloc_model_buffers(m);
  if (r != CH_OK) {
    free_model(m);
    return r;
  }
  cudaStream_t s = ctx->stream;
  size_t max_words = std::max({(size_t)(m->qd + 2 * m->kvd) * (m->H / 32) * 5, (size_t)m->H * (m->qd / 32) * 5,
                               (size_t)m->I * (m->H / 32) * 5, (size_t)m->H * (m->I / 32) * 5});
  uint32_t *tA = nullptr, *tB = nullptr;
  uint16_t *tn = nullptr;
  auto bail = [&](int code) {
    cudaFree(tA);
    cudaFree(tB);
    cudaFree(tn);
    free_model(m);
    return code;
  };
  if (dmalloc(&tA, max_words) != CH_OK || dmalloc(&tB, max_words) != CH_OK || dmalloc(&tn, std::max(m->H, m->D)) != CH_OK)
    return bail(CH_ENOMEM);
  const float wstd = 0.02f;
  const size_t qw = (size_t)m->qd_l * (m->H / 32) * 5, kw = (size_t)m->kvd_l * (m->H / 32) * 5;
  const uint32_t rk = m->rank;
  for (uint32_t l = 0; l < m->L; l++) {
    DevLayer &dl = m->layers[l];
    // q | k | v rows of this rank's heads, o / down rows, gate / up rows
    bool ok =
        launch_gen_q4_rows(tA, rk * m->qd_l, m->qd_l, m->H, ch_tensor_seed(seed, l, T_Q), wstd, s) == cudaSuccess &&
        launch_gen_q4_rows(tA + qw, rk * m->kvd_l, m->kvd_l, m->H, ch_tensor_seed(seed, l, T_K), wstd, s) == cudaSuccess &&
        launch_gen_q4_rows(tA + qw + kw, rk * m->kvd_l, m->kvd_l, m->H, ch_tensor_seed(seed, l, T_V), wstd, s) ==
            cudaSuccess &&
        launch_repack_q4(tA, nullptr, m->qd_l + 2 * m->kvd_l, m->H, MAP_PLAIN, dl.qkv, s) == cudaSuccess &&
        launch_gen_q4_cols(tB, m->H, m->qd, rk * m->qd_l, m->qd_l, ch_tensor_seed(seed, l, T_O), wstd, s) ==
            cudaSuccess &&
        launch_repack_q4(tB, nullptr, m->H, m->qd_l, MAP_PLAIN, dl.o, s) == cudaSuccess &&
        launch_gen_q4_rows(tA, rk * m->Il, m->Il, m->H, ch_tensor_seed(seed, l, T_GATE), wstd, s) == cudaSuccess &&
        launch_gen_q4_rows(tB, rk * m->Il, m->Il, m->H, ch_tensor_seed(seed, l, T_UP), wstd, s) == cudaSuccess &&
        launch_repack_q4(tA, tB, 2 * m->Il, m->H, MAP_GATEUP, dl.gateup, s) == cudaSuccess &&
        launch_gen_q4_cols(tA, m->H, m->I, rk * m->Il, m->Il, ch_tensor_seed(seed, l, T_DOWN), wstd, s) ==
            cudaSuccess &&
        launch_repack_q4(tA, nullptr, m->H, m->Il, MAP_PLAIN, dl.down, s) == cudaSuccess;
    if (!ok) return bail(fail(CH_ECUDA, "synthetic layer generation"));
    if (gen_norm(m, &dl.input_norm, m->H, ch_tensor_seed(seed, l, T_IN_NORM), tn) ||
        gen_norm(m, &dl.q_norm, m->D, ch_tensor_seed(seed, l, T_Q_NORM), tn) ||
        gen_norm(m, &dl.k_norm, m->D, ch_tensor_seed(seed, l, T_K_NORM), tn) ||
        gen_norm(m, &dl.post_attn, m->H, ch_tensor_seed(seed, l, T_POST_ATTN), tn) ||
        gen_norm(m, &dl.pre_ffn, m->H, ch_tensor_seed(seed, l, T_PRE_FFN), tn) ||
        gen_norm(m, &dl.post_ffn, m->H, ch_tensor_seed(seed, l, T_POST_FFN), tn))
      return bail(CH_ECUDA);
    dl.scalar = 1.0f;
  }
  if (gen_norm(m, &m->final_norm, m->H, ch_tensor_seed(seed, 0, T_FINAL_NORM), tn)) return bail(CH_ECUDA);
  cudaFree(tA);
  cudaFree(tB);
  tA = tB = nullptr;
  // tied embedding bf16 N(0, 0.02), LM head = quantizeRowQ8_0 of it
  if (dmalloc(&m->embed, (size_t)m->V * m->H) != CH_OK) return bail(CH_ENOMEM);
  if (launch_gen_bf16(m->embed, (size_t)m->V * m->H, ch_tensor_seed(seed, 0, T_EMBED), 0.0f, 0.02f, s) != cudaSuccess)
    return bail(fail(CH_ECUDA, "gen embed"));
  {
    const uint32_t chunk_rows = 16384;
    uint32_t *tq = nullptr;
    if (dmalloc(&tq, (size_t)chunk_rows * (m->H / 32) * 9) != CH_OK) return bail(CH_ENOMEM);
    for (uint32_t r0 = 0; r0 < m->Vl; r0 += chunk_rows) {  // this rank's vocab rows of the tied embedding
      uint32_t nr = std::min(chunk_rows, m->Vl - r0);
      launch_quantize_q8_rows(m->embed + (size_t)(rk * m->Vl + r0) * m->H, nr, m->H, tq, s);
      launch_repack_q8(tq, nr, m->H, m->lm + q8_tile_bytes(r0, m->H), s);
    }
    cudaStreamSynchronize(s);
    cudaFree(tq);
  }
  cudaError_t e = cudaStreamSynchronize(s);
  cudaFree(tn);
  tn = nullptr;
  if (e != cudaSuccess) return bail(fail(CH_ECUDA, std::string("synthetic model: ") + cudaGetErrorString(e)));
  if (int r2 = init_decode_step(m)) return bail(r2);
  *out = m;
  return CH_OK;
}

extern "C" int ch_model_create_synthetic(ch_ctx *ctx, const ch_model_config *cfg, uint64_t seed, ch_model **out) {
  return create_synthetic(ctx, cfg, seed, 0, 1, out);
}
extern "C" int ch_model_create_synthetic_sharded(ch_ctx *ctx, const ch_model_config *cfg, uint64_t seed, uint32_t rank,
                                                 uint32_t world, ch_model **out) {
  return create_synthetic(ctx, cfg, seed, rank, world, out);
}

// ---------------------------------------------------------------------------
// tensor parallel: the exchange arena is shared between the ranks' processes
// with CUDA IPC; every rank maps every other rank's arena.
extern "C" int ch_model_exchange_handle(ch_model *m, void *handle) {
  if (!m || !handle) return fail(CH_EINVAL, "NULL argument");
  if (m->world <= 1 || !m->arena) return fail(CH_ESTATE, "not a tensor-parallel model");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  cudaIpcMemHandle_t h;
  CH_CUDA(cudaIpcGetMemHandle(&h, m->arena));
  static_assert(sizeof(cudaIpcMemHandle_t) == CH_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return CH_OK;
}
extern "C" int ch_model_attach_peers(ch_model *m, const void *handles) {
  if (!m || !handles) return fail(CH_EINVAL, "NULL argument");
  if (m->world <= 1 || !m->arena) return fail(CH_ESTATE, "not a tensor-parallel model");
  if (m->peers_ready) return fail(CH_ESTATE, "peers already attached");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  const uint8_t *hb = static_cast<const uint8_t *>(handles);
  for (uint32_t r = 0; r < m->world; r++) {
    if (r == m->rank) {
      m->peer_arena[r] = m->arena;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return fail(CH_ECOMM, "cudaIpcOpenMemHandle(rank " + std::to_string(r) + "): " + cudaGetErrorString(e));
    m->peer_arena[r] = static_cast<uint8_t *>(p);
  }
  m->peers_ready = true;
  return CH_OK;
}

extern "C" void ch_model_destroy(ch_model *m) { free_model(m); }

extern "C" int ch_model_weight_tiles(ch_model *m, uint32_t layer, int which, void **tiles, uint32_t *rows,
                                     uint32_t *cols) {
  if (!m || !tiles || !rows || !cols || layer >= m->L) return fail(CH_EINVAL, "bad argument");
  const DevLayer &l = m->layers[layer];
  switch (which) {
    case 0: *tiles = l.qkv, *rows = m->qd_l + 2 * m->kvd_l, *cols = m->H; break;  // this rank's shard
    case 1: *tiles = l.o, *rows = m->H, *cols = m->qd_l; break;  // this rank's columns
    case 2: *tiles = l.gateup, *rows = 2 * m->Il, *cols = m->H; break;
    case 3: *tiles = l.down, *rows = m->H, *cols = m->Il; break;
    case 4: *tiles = m->lm, *rows = m->Vl, *cols = m->H; break;
    default: return fail(CH_EINVAL, "which must be 0..4");
  }
  return CH_OK;
}

extern "C" int ch_model_zero_state(ch_model *m) {
  if (!m) return fail(CH_EINVAL, "model is NULL");
  cudaStream_t s = m->ctx->stream;
  for (auto &l : m->layers) {
    CH_CUDA(cudaMemsetAsync(l.kc, 0, (size_t)kSlots * m->kvd_l * 2, s));
    CH_CUDA(cudaMemsetAsync(l.vc, 0, (size_t)kSlots * m->kvd_l * 2, s));
  }
  CH_CUDA(cudaMemsetAsync(m->X[0], 0, m->H * 4, s));
  CH_CUDA(cudaMemsetAsync(m->X[1], 0, m->H * 4, s));
  CH_CUDA(cudaMemsetAsync(m->normed, 0, m->H * 4, s));
  if (m->mk_arrive) CH_CUDA(cudaMemsetAsync(m->mk_arrive, 0, 8, s));
  if (m->mk_base) CH_CUDA(cudaMemsetAsync(m->mk_base, 0, 24, s));
  if (m->arena) {
    CH_CUDA(cudaMemsetAsync(m->arena + m->off_arrive, 0, 8, s));
    // exchange words restart at epoch 1: no word of an earlier run may carry it
    CH_CUDA(cudaMemsetAsync(m->arena + m->off_o, 0, (size_t)2 * m->world * m->H * 8, s));
    CH_CUDA(cudaMemsetAsync(m->arena + m->off_down, 0, (size_t)2 * m->world * m->H * 8, s));
  }
  CH_CUDA(cudaStreamSynchronize(s));
  return CH_OK;
}

// ---------------------------------------------------------------------------
// the decode step (model_dispatch.zig:10-45 order; norms fused into GEMV prologues)
static cudaError_t enqueue_decode(ch_model *m, cudaStream_t s, bool logits, bool device_loop) {
  cudaError_t e;
  const bool pdl = m->pdl;
  GemvArgs base;
  base.partial = m->gemv_partial;
  base.counters = m->gemv_counters;
  base.err = m->ctx->err;
  base.eps = m->cfg.rms_norm_eps;
  if (device_loop) {
    StepBeginArgs sb{m->embed,      m->H,         sqrtf((float)m->H), m->token,      m->X[0],
                     m->sp,         m->plan,      m->plan_steps,      m->ctx->err,   m->inv_freq_s,
                     m->inv_freq_f, m->rope_cs,   m->cfg.rotary_dim / 2};
    if ((e = launch_step_begin(sb, s, pdl)) != cudaSuccess) return e;
  }
  for (uint32_t l = 0; l < m->L; l++) {
    DevLayer &dl = m->layers[l];
    // q|k|v projections; prologue = layer-0 input norm, or the previous layer's
    // post-FFN norm + residual add + this layer's input norm (model_gpu.zig:160-163)
    {
      GemvArgs a = base;
      GemvPlan p;
      a.tiles = dl.qkv;
      a.row_tiles = (m->qd + 2 * m->kvd) / 16;
      a.k_tiles = m->H / 64;
      a.K = m->H;
      a.norm_w = dl.input_norm;
      a.normed_out = m->normed;
      a.y = m->qkv;
      if (l == 0) {
        p.pro = PRO_RMSNORM;
        a.x = m->X[0];
      } else {
        const DevLayer &pl = m->layers[l - 1];
        p.pro = PRO_ADD_RMSNORM;
        a.x = m->X[1];
        a.r = m->down_out;
        a.post_w = pl.post_ffn;
        a.scalar = pl.scalar;
        a.x_out = m->X[0];
      }
      if ((e = launch_gemv(p, a, s, pdl)) != cudaSuccess) return e;
    }
    {
      AttnArgs a{};
      a.qkv = m->qkv;
      a.q_norm_w = dl.q_norm;
      a.k_norm_w = dl.k_norm;
      a.rope_cs = m->rope_cs + (dl.full ? m->cfg.rotary_dim / 2 : 0);
      a.k_cache = dl.kc;
      a.v_cache = dl.vc;
      a.sp = m->sp;
      a.is_sliding = dl.full ? 0 : 1;
      a.nq = m->nq;
      a.nkv = m->nkv;
      a.D = m->D;
      a.rot = m->cfg.rotary_dim;
      a.eps = m->cfg.rms_norm_eps;
      a.scale = 1.0f;  // Gemma-style: q/k norms replace 1/sqrt(d) (forward.zig:85)
      a.out = m->attn;
      a.partial = m->attn_partial;
      a.counters = m->attn_counters;
      a.err = m->ctx->err;
      a.cache_slots = kSlots;
      if ((e = launch_decode_attn(a, m->attn_splits, s, pdl)) != cudaSuccess) return e;
    }
    {
      GemvArgs a = base;
      GemvPlan p;
      a.tiles = dl.o;
      a.row_tiles = m->H / 16;
      a.k_tiles = m->qd / 64;
      a.K = m->qd;
      a.x = m->attn;
      a.y = m->o_out;
      if ((e = launch_gemv(p, a, s, pdl)) != cudaSuccess) return e;
    }
    {
      GemvArgs a = base;
      GemvPlan p;
      p.epi = EPI_GELU_MUL;
      p.pro = PRO_ADD_RMSNORM;
      a.tiles = dl.gateup;
      a.row_tiles = 2 * m->I / 16;
      a.k_tiles = m->H / 64;
      a.K = m->H;
      a.x = m->X[0];
      a.r = m->o_out;
      a.post_w = dl.post_attn;
      a.scalar = 1.0f;
      a.norm_w = dl.pre_ffn;
      a.x_out = m->X[1];
      a.normed_out = m->normed;
      a.y = m->act;
      if ((e = launch_gemv(p, a, s, pdl)) != cudaSuccess) return e;
    }
    {
      GemvArgs a = base;
      GemvPlan p;
      a.tiles = dl.down;
      a.row_tiles = m->H / 16;
      a.k_tiles = m->I / 64;
      a.K = m->I;
      a.x = m->act;
      a.y = m->down_out;
      if ((e = launch_gemv(p, a, s, pdl)) != cudaSuccess) return e;
    }
  }
  const DevLayer &last = m->layers[m->L - 1];
  if (logits) {
    GemvArgs a = base;
    GemvPlan p;
    p.fmt = FMT_Q8;
    p.pro = PRO_ADD_RMSNORM;
    a.tiles = m->lm;
    a.row_tiles = m->V / 16;
    a.k_tiles = m->H / 32;
    a.K = m->H;
    a.x = m->X[1];
    a.r = m->down_out;
    a.post_w = last.post_ffn;
    a.scalar = last.scalar;
    a.norm_w = m->final_norm;
    a.x_out = m->X[0];
    a.normed_out = m->normed;
    a.y = m->logits;
    if ((e = launch_gemv(p, a, s, pdl)) != cudaSuccess) return e;
    TopkArgs t{};
    t.logits = m->logits;
    t.V = m->V;
    t.cand = m->topk_cand;
    t.counter = m->topk_counter;
    t.ids = m->ids;
    t.vals = m->vals;
    t.token_out = m->token;
    t.token_hist = device_loop ? m->token_hist : nullptr;
    t.hist_cap = m->hist_cap;
    t.sp = device_loop ? m->sp : nullptr;
    t.err = m->ctx->err;
    if ((e = launch_topk64(t, s, pdl)) != cudaSuccess) return e;
  } else {
    // no-logits variant: still fold the last residual add so read_x matches the logits path
    if (last.post_ffn &&
        (e = launch_rmsnorm_rows(m->down_out, last.post_ffn, m->down_out, 1, m->H, m->cfg.rms_norm_eps, s)) !=
            cudaSuccess)
      return e;
    if ((e = launch_add_rmsnorm_rows(m->X[1], m->down_out, m->final_norm, m->normed, 1, m->H, m->cfg.rms_norm_eps,
                                     last.scalar, s)) != cudaSuccess)
      return e;
    if ((e = cudaMemcpyAsync(m->X[0], m->X[1], m->H * 4, cudaMemcpyDeviceToDevice, s)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

static int capture(ch_model *m, bool logits, bool device_loop, cudaGraphExec_t *out) {
  cudaStream_t s = m->ctx->stream;
  for (int attempt = 0; attempt < 2; attempt++) {
    cudaGraph_t g = nullptr;
    CH_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_decode(m, s, logits, device_loop);
    cudaError_t e2 = cudaStreamEndCapture(s, &g);
    if (e == cudaSuccess && e2 == cudaSuccess) {
      cudaError_t e3 = cudaGraphInstantiate(out, g, 0);
      cudaGraphDestroy(g);
      if (e3 == cudaSuccess) return CH_OK;
      e = e3;
    }
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    if (!m->pdl) return fail(CH_ECUDA, std::string("graph capture: ") + cudaGetErrorString(e != cudaSuccess ? e : e2));
    m->pdl = false;  // retry without programmatic dependent launch
  }
  return fail(CH_ECUDA, "graph capture failed");
}

// (cos, sin) of clock * inv_freq[i] for the RoPE of one step: angle in f32 as the
// shaders form it (qkv_rope.wgsl:74-78), cos/sin in double rounded once
static void rope_table(const std::vector<float> &inv, uint32_t clock, float2 *out) {
  for (size_t i = 0; i < inv.size(); i++) {
    const float ang = (float)clock * inv[i];
    out[i] = make_float2((float)cos((double)ang), (float)sin((double)ang));
  }
}

static int check_lists(const uint32_t *l, uint32_t n) {
  if (n > kSlots) return fail(CH_EINVAL, "slot list longer than 4096");
  if (n && !l) return fail(CH_EINVAL, "NULL slot list");
  for (uint32_t i = 0; i < n; i++)
    if (l[i] >= kSlots) return fail(CH_EINVAL, "slot list entry >= 4096");
  return CH_OK;
}

extern "C" int ch_forward_token(ch_model *m, const float *x, uint32_t clock, uint32_t slot, const uint32_t *active,
                                uint32_t n_active, const uint32_t *sliding, uint32_t n_sliding, ch_topk *topk_out,
                                uint32_t *token_out) {
  if (!m || !x) return fail(CH_EINVAL, "NULL argument");
  if (slot >= kSlots) return fail(CH_EINVAL, "slot >= 4096");
  CH_TRY(check_lists(active, n_active));
  CH_TRY(check_lists(sliding, n_sliding));
  if (m->world > 1 && !m->peers_ready) return fail(CH_ESTATE, "tensor parallel: ch_model_attach_peers first");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  const bool logits = topk_out || token_out;
  cudaGraphExec_t *g = logits ? &m->g_host_logits : &m->g_host_nologits;
  if (m->use_ops && !*g) CH_TRY(capture(m, logits, false, g));
  cudaStream_t s = m->ctx->stream;
  memcpy(m->h_x, x, m->H * 4);
  m->h_sp->clock = clock;
  m->h_sp->slot = slot;
  m->h_sp->n_active = n_active;
  m->h_sp->n_sliding = n_sliding;
  m->h_sp->active = m->active;
  m->h_sp->sliding = m->sliding;
  m->h_sp->step = 0;
  m->h_sp->next = 0;
  m->h_sp->force = 0;
  m->h_sp->pad = 0;
  if (n_active) memcpy(m->h_lists, active, n_active * 4);
  if (n_sliding) memcpy(m->h_lists + kSlots, sliding, n_sliding * 4);
  const uint32_t rh = m->cfg.rotary_dim / 2;
  rope_table(m->h_inv_s, clock, m->h_rope);
  rope_table(m->h_inv_f, clock, m->h_rope + rh);
  CH_CUDA(cudaMemcpyAsync(m->X[0], m->h_x, m->H * 4, cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->sp, m->h_sp, sizeof(StepParams), cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->rope_cs, m->h_rope, 2 * rh * sizeof(float2), cudaMemcpyHostToDevice, s));
  if (n_active) CH_CUDA(cudaMemcpyAsync(m->active, m->h_lists, n_active * 4, cudaMemcpyHostToDevice, s));
  if (n_sliding) CH_CUDA(cudaMemcpyAsync(m->sliding, m->h_lists + kSlots, n_sliding * 4, cudaMemcpyHostToDevice, s));
  if (m->use_ops)
    CH_CUDA(cudaGraphLaunch(*g, s));
  else
    CH_CUDA(launch_decode_step(mega_args(m, logits, false), m->mk_smem, s));
  if (logits) {
    CH_CUDA(cudaMemcpyAsync(m->h_ids, m->ids, 64 * 4, cudaMemcpyDeviceToHost, s));
    CH_CUDA(cudaMemcpyAsync(m->h_vals, m->vals, 64 * 4, cudaMemcpyDeviceToHost, s));
  }
  // the step's device status (a bounded wait that gave up, a bad slot) comes back with
  // the results, and is cleared for the next call
  CH_CUDA(cudaMemcpyAsync(m->h_status, m->ctx->err, 4, cudaMemcpyDeviceToHost, s));
  CH_CUDA(cudaMemsetAsync(m->ctx->err, 0, 4, s));
  CH_CUDA(cudaStreamSynchronize(s));
  if (const int rc = status_from_flags(*m->h_status)) return rc;
  if (topk_out)
    for (int i = 0; i < 64; i++) topk_out[i] = ch_topk{m->h_ids[i], m->h_vals[i]};
  if (token_out) *token_out = m->h_ids[0];
  return CH_OK;
}

// ---------------------------------------------------------------------------
// device-resident greedy loop
extern "C" int ch_decode_plan(ch_model *m, const ch_step_desc *steps, uint32_t n_steps) {
  if (!m || (!steps && n_steps)) return fail(CH_EINVAL, "NULL argument");
  if (!m->embed) return fail(CH_ESTATE, "device decode loop needs the device embedding table");
  size_t total = 0;
  for (uint32_t i = 0; i < n_steps; i++) {
    if (steps[i].slot >= kSlots) return fail(CH_EINVAL, "slot >= 4096");
    CH_TRY(check_lists(steps[i].active, steps[i].n_active));
    CH_TRY(check_lists(steps[i].sliding, steps[i].n_sliding));
    total += steps[i].n_active + steps[i].n_sliding;
  }
  CH_CUDA(cudaSetDevice(m->ctx->device));
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  cudaFree(m->plan);
  cudaFree(m->plan_lists);
  m->plan = nullptr;
  m->plan_lists = nullptr;
  CH_TRY(dmalloc(&m->plan, std::max<uint32_t>(n_steps, 1)));
  CH_TRY(dmalloc(&m->plan_lists, std::max<size_t>(total, 1)));
  std::vector<StepParams> hp(n_steps);
  std::vector<uint32_t> hl(total);
  size_t off = 0;
  for (uint32_t i = 0; i < n_steps; i++) {
    hp[i].clock = steps[i].clock;
    hp[i].slot = steps[i].slot;
    hp[i].n_active = steps[i].n_active;
    hp[i].n_sliding = steps[i].n_sliding;
    if (steps[i].n_active) memcpy(&hl[off], steps[i].active, steps[i].n_active * 4);
    hp[i].active = m->plan_lists + off;
    off += steps[i].n_active;
    if (steps[i].n_sliding) memcpy(&hl[off], steps[i].sliding, steps[i].n_sliding * 4);
    hp[i].sliding = m->plan_lists + off;
    off += steps[i].n_sliding;
    hp[i].step = i;
    hp[i].next = 0;
    hp[i].force = 0;
    hp[i].pad = 0;
  }
  if (n_steps) CH_CUDA(cudaMemcpy(m->plan, hp.data(), n_steps * sizeof(StepParams), cudaMemcpyHostToDevice));
  if (total) CH_CUDA(cudaMemcpy(m->plan_lists, hl.data(), total * 4, cudaMemcpyHostToDevice));
  if (m->hist_cap < n_steps) {
    cudaFree(m->token_hist);
    m->token_hist = nullptr;
    CH_TRY(dmalloc(&m->token_hist, n_steps));
    m->hist_cap = n_steps;
  }
  if (n_steps == 0) return fail(CH_EINVAL, "empty plan");
  m->plan_steps = n_steps;
  // the loop graph bakes in plan / token_hist pointers and the plan length: recapture
  if (m->g_loop) {
    cudaGraphExecDestroy(m->g_loop);
    m->g_loop = nullptr;
  }
  if (m->use_ops) CH_TRY(capture(m, true, true, &m->g_loop));
  m->loop_ready = true;
  return CH_OK;
}

static cudaError_t launch_loop_sample(ch_model *m, cudaStream_t s);
static int launch_loop_steps(ch_model *m, uint32_t n_steps) {
  cudaStream_t s = m->ctx->stream;
  if (m->use_ops) {
    for (uint32_t i = 0; i < n_steps; i++) CH_CUDA(cudaGraphLaunch(m->g_loop, s));
    return CH_OK;
  }
  StepBeginArgs sb{m->embed,      m->H,       sqrtf((float)m->H), m->token,    m->X[0],
                   m->sp,         m->plan,    m->plan_steps,      m->ctx->err, m->inv_freq_s,
                   m->inv_freq_f, m->rope_cs, m->cfg.rotary_dim / 2};
  const MegaArgs a = mega_args(m, true, true);
  for (uint32_t i = 0; i < n_steps; i++) {
    CH_CUDA(launch_step_begin(sb, s, false));
    CH_CUDA(launch_decode_step(a, m->mk_smem, s));
    if (m->sampler) CH_CUDA(launch_loop_sample(m, s));
  }
  return CH_OK;
}

extern "C" int ch_decode_run(ch_model *m, uint32_t first_token, uint32_t n_steps) {
  if (!m) return fail(CH_EINVAL, "model is NULL");
  if (!m->loop_ready || n_steps > m->plan_steps) return fail(CH_ESTATE, "ch_decode_plan must cover n_steps first");
  if (m->world > 1 && !m->peers_ready) return fail(CH_ESTATE, "tensor parallel: ch_model_attach_peers first");
  if (first_token >= m->V) return fail(CH_EINVAL, "first_token >= vocab");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  cudaStream_t s = m->ctx->stream;
  CH_CUDA(cudaStreamSynchronize(s));  // previous run may still read the staging words
  m->h_run[0] = 0;
  m->h_run[1] = first_token;
  CH_CUDA(cudaMemcpyAsync(&m->sp->next, &m->h_run[0], 4, cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->token, &m->h_run[1], 4, cudaMemcpyHostToDevice, s));
  CH_TRY(launch_loop_steps(m, n_steps));
  m->loop_pos = n_steps;
  return CH_OK;
}

extern "C" int ch_decode_continue(ch_model *m, uint32_t n_steps) {
  if (!m) return fail(CH_EINVAL, "model is NULL");
  if (!m->loop_ready) return fail(CH_ESTATE, "ch_decode_plan and ch_decode_run come first");
  if ((uint64_t)m->loop_pos + n_steps > m->plan_steps) return fail(CH_EINVAL, "more steps than planned");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  CH_TRY(launch_loop_steps(m, n_steps));
  m->loop_pos += n_steps;
  return CH_OK;
}

// ---------------------------------------------------------------------------
// Device sampler (sampler.cu): Sampler.sampleTopK with its generator state on the device
struct ch_sampler {
  ch_ctx *ctx = nullptr;
  SamplerParams p{};
  uint64_t *prng = nullptr;      // [4]
  uint32_t *recent = nullptr;    // [cap]
  uint32_t *n_recent = nullptr;  // [1]
  uint32_t cap = 0;
};
static_assert(sizeof(SamplerParams) == sizeof(ch_sampler_params), "sampler params layout");
extern "C" int ch_sampler_create(ch_ctx *ctx, const ch_sampler_params *params, uint64_t seed, uint32_t recent_cap,
                                 ch_sampler **out) {
  if (!ctx || !params || !out) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaSetDevice(ctx->device));
  ch_sampler *s = new ch_sampler();
  s->ctx = ctx;
  memcpy(&s->p, params, sizeof(SamplerParams));
  s->cap = recent_cap;
  if (dmalloc(&s->prng, 4) != CH_OK || dmalloc(&s->recent, std::max(recent_cap, 1u)) != CH_OK ||
      dmalloc(&s->n_recent, 1) != CH_OK) {
    cudaFree(s->prng);
    cudaFree(s->recent);
    cudaFree(s->n_recent);
    delete s;
    return fail(CH_ENOMEM, "sampler allocation");
  }
  // Xoshiro256.init(seed): the state words are four SplitMix64 outputs (Zig std/Random/Xoshiro256.zig)
  uint64_t st[4], z0 = seed;
  for (int i = 0; i < 4; i++) {
    z0 += 0x9e3779b97f4a7c15ull;
    uint64_t z = z0;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    st[i] = z ^ (z >> 31);
  }
  const uint32_t zero = 0;
  if (cudaMemcpy(s->prng, st, sizeof(st), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(s->n_recent, &zero, 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(s->prng);
    cudaFree(s->recent);
    cudaFree(s->n_recent);
    delete s;
    return fail(CH_ECUDA, "sampler upload");
  }
  *out = s;
  return CH_OK;
}
extern "C" void ch_sampler_destroy(ch_sampler *s) {
  if (!s) return;
  cudaSetDevice(s->ctx->device);
  cudaStreamSynchronize(s->ctx->stream);
  cudaFree(s->prng);
  cudaFree(s->recent);
  cudaFree(s->n_recent);
  delete s;
}
extern "C" int ch_sampler_set_recent(ch_sampler *s, const uint32_t *recent, uint32_t n) {
  if (!s || (!recent && n)) return fail(CH_EINVAL, "NULL argument");
  if (n > s->cap) return fail(CH_EINVAL, "more recent tokens than the sampler's capacity");
  CH_CUDA(cudaSetDevice(s->ctx->device));
  CH_CUDA(cudaStreamSynchronize(s->ctx->stream));
  if (n) CH_CUDA(cudaMemcpy(s->recent, recent, (size_t)n * 4, cudaMemcpyHostToDevice));
  CH_CUDA(cudaMemcpy(s->n_recent, &n, 4, cudaMemcpyHostToDevice));
  return CH_OK;
}
extern "C" int ch_sampler_sample_topk(ch_sampler *s, const uint32_t *ids, const float *vals, uint32_t n,
                                      const uint32_t *recent, uint32_t n_recent, uint32_t *token) {
  if (!s || !ids || !vals || !token) return fail(CH_EINVAL, "NULL argument");
  if (n > 64) return fail(CH_EINVAL, "at most 64 candidates");
  CH_CUDA(cudaSetDevice(s->ctx->device));
  SampleArgs a;
  a.ids = ids;
  a.vals = vals;
  a.n = n;
  a.recent = recent;
  a.n_recent = recent ? n_recent : 0;
  a.p = s->p;
  a.prng = s->prng;
  a.token_out = token;
  CH_CUDA(launch_sample_topk(a, s->ctx->stream));
  return CH_OK;
}
extern "C" int ch_model_set_sampler(ch_model *m, ch_sampler *s) {
  if (!m) return fail(CH_EINVAL, "NULL model");
  if (s && s->ctx->device != m->ctx->device) return fail(CH_EINVAL, "sampler and model on different devices");
  if (s && m->use_ops) return fail(CH_ESTATE, "the device sampler runs with the persistent decode kernel");
  m->sampler = s;
  return CH_OK;
}
// the sampling launch of one device-loop step (after the decode step wrote the top-64)
static cudaError_t launch_loop_sample(ch_model *m, cudaStream_t s) {
  ch_sampler *sm = m->sampler;
  SampleArgs a;
  a.ids = m->ids;
  a.vals = m->vals;
  a.n = 64;
  a.recent = sm->recent;
  a.n_recent_dev = sm->n_recent;
  a.recent_w = sm->recent;
  a.recent_cap = sm->cap;
  a.p = sm->p;
  a.prng = sm->prng;
  a.token_out = m->token;
  a.sp = m->sp;
  a.token_hist = m->token_hist;
  a.hist_cap = m->hist_cap;
  return launch_sample_topk(a, s);
}

// ---------------------------------------------------------------------------
// Device-side ring lists (ring_dev.cu): a device copy of a ring's layer-0 metadata
// and the decode loop that builds every step's lists from it on the device.
namespace ch {
bool ring_export_layer0(const ch_ring *r, RingDevState *out);
}
struct ch_ring_dev {
  ch_ctx *ctx = nullptr;
  RingDevState *d = nullptr;
  RingDevState *h = nullptr;  // pinned staging
};
extern "C" int ch_ring_dev_create(ch_ctx *ctx, ch_ring_dev **out) {
  if (!ctx || !out) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaSetDevice(ctx->device));
  ch_ring_dev *r = new ch_ring_dev();
  r->ctx = ctx;
  if (cudaMalloc(&r->d, sizeof(RingDevState)) != cudaSuccess ||
      cudaMallocHost(&r->h, sizeof(RingDevState)) != cudaSuccess) {
    cudaFree(r->d);
    cudaFreeHost(r->h);
    delete r;
    return fail(CH_ENOMEM, "ring_dev allocation");
  }
  memset(r->h, 0, sizeof(RingDevState));
  CH_CUDA(cudaMemset(r->d, 0, sizeof(RingDevState)));
  *out = r;
  return CH_OK;
}
extern "C" void ch_ring_dev_destroy(ch_ring_dev *r) {
  if (!r) return;
  cudaSetDevice(r->ctx->device);
  cudaStreamSynchronize(r->ctx->stream);
  cudaFree(r->d);
  cudaFreeHost(r->h);
  delete r;
}
extern "C" int ch_ring_dev_upload(ch_ring_dev *r, const ch_ring *host) {
  if (!r || !host) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaSetDevice(r->ctx->device));
  CH_CUDA(cudaStreamSynchronize(r->ctx->stream));  // the staging copy may still be in flight
  if (!ring_export_layer0(host, r->h)) return fail(CH_EINVAL, "ring clock does not fit 32 bits");
  CH_CUDA(cudaMemcpyAsync(r->d, r->h, sizeof(RingDevState), cudaMemcpyHostToDevice, r->ctx->stream));
  CH_CUDA(cudaStreamSynchronize(r->ctx->stream));
  return CH_OK;
}
extern "C" int ch_ring_dev_lists(ch_ring_dev *r, uint32_t clock, int activate, size_t sliding_window, uint32_t *slot_dev,
                                 uint32_t *active_dev, uint32_t *n_active_dev, uint32_t *sliding_dev,
                                 uint32_t *n_sliding_dev) {
  if (!r || !active_dev || !n_active_dev || !sliding_dev || !n_sliding_dev) return fail(CH_EINVAL, "NULL argument");
  if (sliding_window > 0xFFFFFFFFull) return fail(CH_EINVAL, "sliding_window does not fit 32 bits");
  CH_CUDA(cudaSetDevice(r->ctx->device));
  RingStepArgs a;
  a.ring = r->d;
  a.clock = clock;
  a.sliding_window = (uint32_t)sliding_window;
  a.activate = activate ? 1 : 0;
  a.slot_out = slot_dev;
  a.active_out = active_dev;
  a.n_active_out = n_active_dev;
  a.sliding_out = sliding_dev;
  a.n_sliding_out = n_sliding_dev;
  CH_CUDA(launch_ring_step(a, r->ctx->stream));
  return CH_OK;
}
extern "C" int ch_ring_dev_prefill_prev(ch_ring_dev *r, uint32_t start_clock, uint32_t chunk_len, uint32_t *out_dev,
                                        uint32_t *n_dev) {
  if (!r || !out_dev || !n_dev) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaSetDevice(r->ctx->device));
  if (start_clock == 0 || chunk_len == 0) {  // ring_buffer.zig:344
    CH_CUDA(cudaMemsetAsync(n_dev, 0, 4, r->ctx->stream));
    return CH_OK;
  }
  RingStepArgs a;
  a.ring = r->d;
  a.clock = start_clock;
  a.chunk_len = chunk_len;
  a.prev = 1;
  a.active_out = out_dev;
  a.n_active_out = n_dev;
  CH_CUDA(launch_ring_step(a, r->ctx->stream));
  return CH_OK;
}
extern "C" int ch_decode_run_ring(ch_model *m, ch_ring_dev *r, ch_ring *host, uint32_t first_token,
                                  uint32_t first_clock, uint32_t n_steps) {
  if (!m || !r) return fail(CH_EINVAL, "NULL argument");
  if (!m->embed) return fail(CH_ESTATE, "device decode loop needs the device embedding table");
  if (r->ctx->device != m->ctx->device) return fail(CH_EINVAL, "ring_dev and model on different devices");
  if (m->world > 1 && !m->peers_ready) return fail(CH_ESTATE, "tensor parallel: ch_model_attach_peers first");
  if (first_token >= m->V) return fail(CH_EINVAL, "first_token >= vocab");
  if (n_steps == 0) return fail(CH_EINVAL, "n_steps == 0");
  if ((uint64_t)first_clock + n_steps > 0xFFFFFFFFull) return fail(CH_EINVAL, "clock overflow");
  if (m->use_ops) return fail(CH_ESTATE, "device ring loop runs on the persistent decode kernel");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  cudaStream_t s = m->ctx->stream;
  CH_CUDA(cudaStreamSynchronize(r->ctx->stream));
  CH_CUDA(cudaStreamSynchronize(s));  // a previous run may still read the staging words
  if (m->hist_cap < n_steps) {
    cudaFree(m->token_hist);
    m->token_hist = nullptr;
    m->hist_cap = 0;
    CH_TRY(dmalloc(&m->token_hist, n_steps));
    m->hist_cap = n_steps;
  }
  r->h->next_clock = first_clock;
  r->h->step = 0;
  m->h_run[1] = first_token;
  CH_CUDA(cudaMemcpyAsync(&r->d->next_clock, &r->h->next_clock, 8, cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->token, &m->h_run[1], 4, cudaMemcpyHostToDevice, s));
  RingStepArgs ra;
  ra.ring = r->d;
  ra.sliding_window = m->cfg.sliding_window;
  ra.activate = 1;
  ra.loop = 1;
  ra.active_out = m->active;
  ra.sliding_out = m->sliding;
  ra.sp = m->sp;
  StepBeginArgs sb{m->embed,      m->H,       sqrtf((float)m->H), m->token,    m->X[0],
                   m->sp,         nullptr,    0,                  m->ctx->err, m->inv_freq_s,
                   m->inv_freq_f, m->rope_cs, m->cfg.rotary_dim / 2};
  const MegaArgs a = mega_args(m, true, true);
  for (uint32_t i = 0; i < n_steps; i++) {
    CH_CUDA(launch_ring_step(ra, s));
    CH_CUDA(launch_step_begin(sb, s, false));
    CH_CUDA(launch_decode_step(a, m->mk_smem, s));
    if (m->sampler) CH_CUDA(launch_loop_sample(m, s));
  }
  // the host ring takes the same activations (the caller's ring stays the source of truth)
  if (host)
    for (uint32_t i = 0; i < n_steps; i++) ch_ring_activate_slot(host, 0, (size_t)first_clock + i);
  m->loop_ready = false;  // the plan's step counter no longer matches the device state
  return CH_OK;
}

extern "C" int ch_decode_tokens(ch_model *m, uint32_t *tokens, uint32_t n) {
  if (!m || (!tokens && n)) return fail(CH_EINVAL, "NULL argument");
  if (n > m->hist_cap) return fail(CH_EINVAL, "more tokens than planned steps");
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  if (n) CH_CUDA(cudaMemcpy(tokens, m->token_hist, n * 4, cudaMemcpyDeviceToHost));
  uint32_t f = 0;
  CH_TRY(ch_ctx_device_status(m->ctx, &f));
  return status_from_flags(f);
}

// ---------------------------------------------------------------------------
// state access
extern "C" int ch_read_x(ch_model *m, float *x) {
  if (!m || !x) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  CH_CUDA(cudaMemcpy(x, m->X[0], m->H * 4, cudaMemcpyDeviceToHost));
  return CH_OK;
}
extern "C" int ch_read_normed_x(ch_model *m, float *x) {
  if (!m || !x) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  CH_CUDA(cudaMemcpy(x, m->normed, m->H * 4, cudaMemcpyDeviceToHost));
  return CH_OK;
}
// k / v hold kv_dim = num_key_value_heads * head_dim floats (every kv head).  A
// tensor-parallel shard holds kv heads [rank * n_kv / world, (rank + 1) * n_kv / world):
// ch_kv_read fills that range of k / v and leaves the rest as it was, ch_kv_write
// stores only that range -- the full row is each rank's call over the same row.
extern "C" int ch_kv_read(ch_model *m, uint32_t layer, uint32_t slot, float *k, float *v) {
  if (!m || layer >= m->L || slot >= kSlots) return fail(CH_EINVAL, "bad layer / slot");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  const uint32_t w = m->kvd_l, c0 = m->rank * w;
  std::vector<__half> hk(w), hv(w);
  CH_CUDA(cudaMemcpy(hk.data(), m->layers[layer].kc + (size_t)slot * w, w * 2, cudaMemcpyDeviceToHost));
  CH_CUDA(cudaMemcpy(hv.data(), m->layers[layer].vc + (size_t)slot * w, w * 2, cudaMemcpyDeviceToHost));
  for (uint32_t i = 0; i < w; i++) {
    if (k) k[c0 + i] = __half2float(hk[i]);
    if (v) v[c0 + i] = __half2float(hv[i]);
  }
  return CH_OK;
}
extern "C" int ch_kv_write(ch_model *m, uint32_t layer, uint32_t slot, const float *k, const float *v) {
  if (!m || layer >= m->L || slot >= kSlots || !k || !v) return fail(CH_EINVAL, "bad argument");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  const uint32_t w = m->kvd_l, c0 = m->rank * w;
  std::vector<__half> hk(w), hv(w);
  for (uint32_t i = 0; i < w; i++) {
    hk[i] = __float2half_rn(k[c0 + i]);
    hv[i] = __float2half_rn(v[c0 + i]);
  }
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  CH_CUDA(cudaMemcpy(m->layers[layer].kc + (size_t)slot * w, hk.data(), w * 2, cudaMemcpyHostToDevice));
  CH_CUDA(cudaMemcpy(m->layers[layer].vc + (size_t)slot * w, hv.data(), w * 2, cudaMemcpyHostToDevice));
  return CH_OK;
}

// ---------------------------------------------------------------------------
// batched prefill (batch_dispatch.zig:55-151 order)
static int ensure_prefill(ch_model *m) {
  const uint32_t N = m->cfg.max_prefill_tokens ? m->cfg.max_prefill_tokens : 1024;
  if (m->pf_cap >= N) return CH_OK;
  CH_TRY(dmalloc(&m->pX, (size_t)N * m->H));
  CH_TRY(dmalloc(&m->pNX, (size_t)N * m->H));
  CH_TRY(dmalloc(&m->pQKV, (size_t)N * (m->qd + 2 * m->kvd)));
  CH_TRY(dmalloc(&m->pQO, (size_t)N * m->qd));
  CH_TRY(dmalloc(&m->pA, (size_t)N * m->qd));
  CH_TRY(dmalloc(&m->pMO, (size_t)N * m->H));
  CH_TRY(dmalloc(&m->pACT, (size_t)N * m->I));
  CH_TRY(dmalloc(&m->pSlots, (size_t)N + kSlots));
  CH_TRY(dmalloc(&m->pTok, (size_t)N));
  {
    const uint32_t qkvd = m->qd + 2 * m->kvd;
    size_t need = tc_gemm_scratch_bytes(N, qkvd, m->H);
    need = std::max(need, tc_gemm_scratch_bytes(N, m->H, m->qd));
    need = std::max(need, tc_gemm_scratch_bytes(N, 2 * m->I, m->H));
    need = std::max(need, tc_gemm_scratch_bytes(N, m->H, m->I));
    CH_TRY(dmalloc(&m->pXS, need));
    m->pXS_n = need;
    CH_CUDA(cudaMemset(m->pXS, 0, 16384));  // split-K tile counters start at zero
  }
  m->pf_cap = N;
  return CH_OK;
}

// Tensor-parallel prefill: the prompt runs through the persistent decode kernel one
// token at a time (plan entries with forced tokens; the LM head only for the last),
// every rank in lock step.  Token t attends to slots[0 .. num_prev + t] (its sliding
// list is the last 1024 of them, batch_causal_attn.wgsl:53), like the batched path.
static int prefill_tp(ch_model *m, const uint32_t *tokens, uint32_t n, const uint32_t *slots, uint32_t start_clock,
                      uint32_t num_prev, ch_topk *topk_out, ch_progress_fn progress_fn, void *progress_ctx) {
  if (!m->peers_ready) return fail(CH_ESTATE, "tensor parallel: ch_model_attach_peers first");
  if (!m->embed) return fail(CH_ESTATE, "tensor-parallel prefill embeds on the device: no device embedding table");
  cudaStream_t s = m->ctx->stream;
  CH_CUDA(cudaStreamSynchronize(s));
  cudaFree(m->pplan);
  cudaFree(m->pplan_lists);
  m->pplan = nullptr;
  m->pplan_lists = nullptr;
  CH_TRY(dmalloc(&m->pplan, n));
  CH_TRY(dmalloc(&m->pplan_lists, num_prev + n));
  CH_CUDA(cudaMemcpy(m->pplan_lists, slots, (size_t)(num_prev + n) * 4, cudaMemcpyHostToDevice));
  std::vector<StepParams> hp(n);
  for (uint32_t t = 0; t < n; t++) {
    const uint32_t na = num_prev + t + 1, ns = std::min<uint32_t>(na, 1024);
    hp[t] = StepParams{start_clock + t, slots[num_prev + t], na, ns, m->pplan_lists, m->pplan_lists + (na - ns),
                       t, 0, tokens[t] + 1, 0};
  }
  CH_CUDA(cudaMemcpy(m->pplan, hp.data(), n * sizeof(StepParams), cudaMemcpyHostToDevice));
  m->h_run[0] = 0;
  CH_CUDA(cudaMemcpyAsync(&m->sp->next, &m->h_run[0], 4, cudaMemcpyHostToDevice, s));
  StepBeginArgs sb{m->embed,      m->H,       sqrtf((float)m->H), m->token,    m->X[0],
                   m->sp,         m->pplan,   n,                  m->ctx->err, m->inv_freq_s,
                   m->inv_freq_f, m->rope_cs, m->cfg.rotary_dim / 2};
  const MegaArgs a_nl = mega_args(m, false, false), a_lg = mega_args(m, true, false);
  for (uint32_t t = 0; t < n; t++) {
    CH_CUDA(launch_step_begin(sb, s, false));
    CH_CUDA(launch_decode_step(t + 1 < n ? a_nl : a_lg, m->mk_smem, s));
  }
  if (topk_out) {
    CH_CUDA(cudaMemcpyAsync(m->h_ids, m->ids, 256, cudaMemcpyDeviceToHost, s));
    CH_CUDA(cudaMemcpyAsync(m->h_vals, m->vals, 256, cudaMemcpyDeviceToHost, s));
  }
  CH_CUDA(cudaStreamSynchronize(s));
  if (topk_out)
    for (int i = 0; i < 64; i++) topk_out[i] = ch_topk{m->h_ids[i], m->h_vals[i]};
  if (progress_fn) progress_fn(m->L, m->L, progress_ctx);
  uint32_t f = 0;
  CH_TRY(ch_ctx_device_status(m->ctx, &f));
  return status_from_flags(f);
}

// stream < 0: the model's own KV cache; else that stream's (ch_streams_init)
static int prefill_impl(ch_model *m, const uint32_t *tokens, uint32_t n, const uint16_t *embed_bf16,
                        const uint32_t *slots, uint32_t start_clock, uint32_t num_prev, ch_topk *topk_out,
                        float *logits_out, size_t logits_len, ch_progress_fn progress_fn, void *progress_ctx,
                        int stream) {
  if (!m || !tokens || !slots) return fail(CH_EINVAL, "NULL argument");
  if (logits_out && logits_len > m->V) return fail(CH_EINVAL, "logits_out longer than the vocabulary");
  if (!logits_out) logits_len = 0;
  if (logits_len && m->world > 1)
    return fail(CH_ESTATE, "tensor parallel: each rank holds only its vocab rows' logits");
  const uint32_t cap = m->cfg.max_prefill_tokens ? m->cfg.max_prefill_tokens : 1024;
  if (n == 0 || n > cap) return fail(CH_EBATCH, "BatchTooLarge: n_tokens must be 1..max_prefill_tokens");
  if (num_prev + n > kSlots) return fail(CH_EINVAL, "num_prev_slots + n_tokens > 4096");
  CH_TRY(check_lists(slots, num_prev + n));
  for (uint32_t i = 0; i < n; i++)
    if (tokens[i] >= m->V) return fail(CH_EINVAL, "token id >= vocab");
  if (!embed_bf16 && !m->embed) return fail(CH_ESTATE, "no embedding table (host or device)");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  if (m->world > 1) return prefill_tp(m, tokens, n, slots, start_clock, num_prev, topk_out, progress_fn, progress_ctx);
  CH_TRY(ensure_prefill(m));
  const size_t soff = stream < 0 ? 0 : (size_t)stream * kSlots * m->kvd;  // the stream's cache within the layer's
  auto kc_of = [&](uint32_t l) { return stream < 0 ? m->layers[l].kc : m->skc[l] + soff; };
  auto vc_of = [&](uint32_t l) { return stream < 0 ? m->layers[l].vc : m->svc[l] + soff; };
  cudaStream_t s = m->ctx->stream;
  const float scale = sqrtf((float)m->H);
  if (embed_bf16) {
    // host expand like expandEmbeddings (batch_dispatch.zig:14-23)
    std::vector<float> hx((size_t)n * m->H);
    for (uint32_t t = 0; t < n; t++) {
      const uint16_t *row = embed_bf16 + (size_t)tokens[t] * m->H;
      for (uint32_t i = 0; i < m->H; i++) {
        uint32_t u = (uint32_t)row[i] << 16;
        float f;
        memcpy(&f, &u, 4);
        hx[(size_t)t * m->H + i] = f * scale;
      }
    }
    CH_CUDA(cudaMemcpyAsync(m->pX, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice, s));
    CH_CUDA(cudaStreamSynchronize(s));
  } else {
    CH_CUDA(cudaMemcpyAsync(m->pTok, tokens, n * 4, cudaMemcpyHostToDevice, s));
    CH_CUDA(launch_embed_rows(m->embed, m->pTok, n, m->H, scale, m->pX, s));
  }
  CH_CUDA(cudaMemcpyAsync(m->pSlots, slots, (num_prev + n) * 4, cudaMemcpyHostToDevice, s));
  const float eps = m->cfg.rms_norm_eps;
  const uint32_t qkvd = m->qd + 2 * m->kvd;
  uint32_t *err = m->ctx->err;
  for (uint32_t l = 0; l < m->L; l++) {
    DevLayer &dl = m->layers[l];
    if (l == 0) CH_CUDA(launch_rmsnorm_rows(m->pX, dl.input_norm, m->pNX, n, m->H, eps, s));
    CH_CUDA(launch_batch_gemm_q4_tc(BatchGemmArgs{dl.qkv, qkvd, m->H, n, m->pNX, m->pQKV, EPI_STORE}, m->pXS, m->pXS_n, err, s));
    BatchQkvRopeArgs r{};
    r.q = m->pQKV;
    r.k = m->pQKV + m->qd;
    r.v = m->pQKV + m->qd + m->kvd;
    r.q_stride = qkvd;
    r.kv_stride = qkvd;
    r.q_norm_w = dl.q_norm;
    r.k_norm_w = dl.k_norm;
    r.inv_freq = dl.full ? m->inv_freq_f : m->inv_freq_s;
    r.q_out = m->pQO;
    r.k_cache = kc_of(l);
    r.v_cache = vc_of(l);
    r.slots = m->pSlots;
    r.slot_offset = num_prev;
    r.start_clock = start_clock;
    r.N = n;
    r.nq = m->nq;
    r.nkv = m->nkv;
    r.D = m->D;
    r.rot = m->cfg.rotary_dim;
    r.eps = eps;
    r.k_eq_v = 0;
    CH_CUDA(launch_batch_qkv_rope(r, s));
    BatchAttnArgs at{m->pQO, kc_of(l), vc_of(l), m->pSlots, n, num_prev, m->nq, m->nkv, m->D, 1.0f, dl.full ? 0 : 1, m->pA};
    CH_CUDA(launch_batch_causal_attn(at, s));
    CH_CUDA(launch_batch_gemm_q4_tc(BatchGemmArgs{dl.o, m->H, m->qd, n, m->pA, m->pMO, EPI_STORE}, m->pXS, m->pXS_n, err, s));
    if (dl.post_attn) CH_CUDA(launch_rmsnorm_rows(m->pMO, dl.post_attn, m->pMO, n, m->H, eps, s));
    CH_CUDA(launch_add_rmsnorm_rows(m->pX, m->pMO, dl.pre_ffn, m->pNX, n, m->H, eps, 1.0f, s));
    CH_CUDA(launch_batch_gemm_q4_tc(BatchGemmArgs{dl.gateup, 2 * m->I, m->H, n, m->pNX, m->pACT, EPI_GELU_MUL}, m->pXS,
                                    m->pXS_n, err, s));
    CH_CUDA(launch_batch_gemm_q4_tc(BatchGemmArgs{dl.down, m->H, m->I, n, m->pACT, m->pMO, EPI_STORE}, m->pXS, m->pXS_n, err, s));
    if (dl.post_ffn) CH_CUDA(launch_rmsnorm_rows(m->pMO, dl.post_ffn, m->pMO, n, m->H, eps, s));
    const float *next = (l + 1 < m->L) ? m->layers[l + 1].input_norm : m->final_norm;
    CH_CUDA(launch_add_rmsnorm_rows(m->pX, m->pMO, next, m->pNX, n, m->H, eps, dl.scalar, s));
    if (progress_fn && ((l + 1) % 4 == 0 || l + 1 == m->L)) {
      CH_CUDA(cudaStreamSynchronize(s));
      progress_fn(l + 1, m->L, progress_ctx);
    }
  }
  // decode-visible state = last token's residual / normed hidden
  CH_CUDA(cudaMemcpyAsync(m->X[0], m->pX + (size_t)(n - 1) * m->H, m->H * 4, cudaMemcpyDeviceToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->normed, m->pNX + (size_t)(n - 1) * m->H, m->H * 4, cudaMemcpyDeviceToDevice, s));
  if (topk_out || logits_len) {  // LM head + top-64 of the last token (batch_dispatch.zig:145-150)
    GemvArgs a;
    GemvPlan p;
    p.fmt = FMT_Q8;
    a.tiles = m->lm;
    a.row_tiles = m->V / 16;
    a.k_tiles = m->H / 32;
    a.K = m->H;
    a.x = m->normed;
    a.y = m->logits;
    a.partial = m->gemv_partial;
    a.counters = m->gemv_counters;
    a.err = m->ctx->err;
    CH_CUDA(launch_gemv(p, a, s, false));
    TopkArgs t{};
    t.logits = m->logits;
    t.V = m->V;
    t.cand = m->topk_cand;
    t.counter = m->topk_counter;
    t.ids = m->ids;
    t.vals = m->vals;
    t.token_out = m->token;
    t.err = m->ctx->err;
    CH_CUDA(launch_topk64(t, s, false));
    CH_CUDA(cudaMemcpyAsync(m->h_ids, m->ids, 256, cudaMemcpyDeviceToHost, s));
    CH_CUDA(cudaMemcpyAsync(m->h_vals, m->vals, 256, cudaMemcpyDeviceToHost, s));
  }
  // the reference copies the first logits_out.len raw logits (batch_dispatch.zig:168-170)
  if (logits_len) CH_CUDA(cudaMemcpyAsync(logits_out, m->logits, logits_len * 4, cudaMemcpyDeviceToHost, s));
  CH_CUDA(cudaStreamSynchronize(s));
  if (topk_out)
    for (int i = 0; i < 64; i++) topk_out[i] = ch_topk{m->h_ids[i], m->h_vals[i]};
  uint32_t f = 0;
  CH_TRY(ch_ctx_device_status(m->ctx, &f));
  return status_from_flags(f);
}

extern "C" int ch_prefill(ch_model *m, const uint32_t *tokens, uint32_t n, const uint16_t *embed_bf16,
                          const uint32_t *slots, uint32_t start_clock, uint32_t num_prev, ch_topk *topk_out,
                          float *logits_out, size_t logits_len, ch_progress_fn progress_fn, void *progress_ctx) {
  return prefill_impl(m, tokens, n, embed_bf16, slots, start_clock, num_prev, topk_out, logits_out, logits_len,
                      progress_fn, progress_ctx, -1);
}

// ---------------------------------------------------------------------------
// Multi-stream greedy decode.  Every stream has its own
// 4,096-slot KV cache per layer.  One step takes one token from each of up to
// ms_cap streams and runs the layers as a batch: the row norms and tcgen05 Q4 GEMMs
// of the prefill path on B tokens, then decode attention with one token per stream
// -- each against its own stream's cache and slot lists, at its own clock (RoPE) --
// and the Q8 LM head and greedy argmax per token.  The weights are read once per
// step for all B streams.  The reference serves one stream (server_queue.zig:9-145,
// server.zig:259-281); this batching is new.
static void free_streams(ch_model *m) {
  for (auto g : m->ms_exec)
    if (g) cudaGraphExecDestroy(g);
  m->ms_exec.clear();
  for (auto *p : m->skc) cudaFree(p);
  for (auto *p : m->svc) cudaFree(p);
  m->skc.clear();
  m->svc.clear();
  void *dev[] = {m->ms_logits, m->ms_tok, m->ms_stream, m->ms_ids, m->ms_lists, m->ms_sp, m->ms_rope,
                 m->ms_partial, m->ms_counters, m->ms_xf, m->ms_skp};
  for (void *p : dev) cudaFree(p);
  void *host[] = {m->h_ms_u32, m->h_ms_sp, m->h_ms_rope};
  for (void *p : host) cudaFreeHost(p);
  m->ms_logits = nullptr, m->ms_tok = m->ms_stream = m->ms_ids = m->ms_lists = nullptr, m->ms_sp = nullptr;
  m->ms_rope = nullptr, m->ms_partial = nullptr, m->ms_counters = nullptr, m->ms_xf = nullptr, m->ms_skp = nullptr;
  m->h_ms_u32 = nullptr, m->h_ms_sp = nullptr, m->h_ms_rope = nullptr;
  m->ms_n = m->ms_cap = 0;
}

static int init_streams(ch_model *m, uint32_t n_streams, uint32_t max_batch) {
  CH_TRY(ensure_prefill(m));
  const size_t per = (size_t)n_streams * kSlots * m->kvd;
  m->skc.assign(m->L, nullptr);
  m->svc.assign(m->L, nullptr);
  for (uint32_t l = 0; l < m->L; l++) {
    CH_TRY(dmalloc(&m->skc[l], per));
    CH_TRY(dmalloc(&m->svc[l], per));
    CH_CUDA(cudaMemset(m->skc[l], 0, per * sizeof(__half)));
    CH_CUDA(cudaMemset(m->svc[l], 0, per * sizeof(__half)));
  }
  const uint32_t rh = m->cfg.rotary_dim / 2, R = m->nq / m->nkv;
  CH_TRY(dmalloc(&m->ms_logits, (size_t)max_batch * m->V));
  CH_TRY(dmalloc(&m->ms_tok, max_batch));
  CH_TRY(dmalloc(&m->ms_stream, max_batch));
  CH_TRY(dmalloc(&m->ms_ids, max_batch));
  CH_TRY(dmalloc(&m->ms_lists, (size_t)max_batch * 2 * kSlots));
  CH_TRY(dmalloc(&m->ms_sp, max_batch));
  CH_TRY(dmalloc(&m->ms_rope, (size_t)2 * max_batch * rh));
  CH_TRY(dmalloc(&m->ms_partial, (size_t)max_batch * attn_partial_floats(m->nkv, R, m->D, m->attn_splits)));
  CH_TRY(dmalloc(&m->ms_counters, (size_t)max_batch * m->nkv));
  CH_CUDA(cudaMemset(m->ms_counters, 0, (size_t)max_batch * m->nkv * 4));
  CH_TRY(dmalloc(&m->ms_xf, skinny_x_words(max_batch, std::max({m->H, m->qd, m->I}))));
  {
    const uint32_t qkvd = m->qd + 2 * m->kvd;
    size_t p = skinny_partial_floats(max_batch, qkvd / 16, m->H);
    p = std::max(p, skinny_partial_floats(max_batch, m->H / 16, m->qd));
    p = std::max(p, skinny_partial_floats(max_batch, 2 * m->I / 16, m->H));
    p = std::max(p, skinny_partial_floats(max_batch, m->H / 16, m->I));
    CH_TRY(dmalloc(&m->ms_skp, p));
  }
  CH_CUDA(cudaMallocHost(&m->h_ms_u32, ((size_t)3 * max_batch + (size_t)max_batch * 2 * kSlots) * 4));
  CH_CUDA(cudaMallocHost(&m->h_ms_sp, max_batch * sizeof(StepParams)));
  CH_CUDA(cudaMallocHost(&m->h_ms_rope, (size_t)2 * max_batch * rh * sizeof(float2)));
  m->ms_n = n_streams;
  m->ms_cap = max_batch;
  return CH_OK;
}

extern "C" int ch_streams_init(ch_model *m, uint32_t n_streams, uint32_t max_batch) {
  if (!m) return fail(CH_EINVAL, "NULL model");
  if (m->world > 1)
    return fail(CH_ESTATE, "multi-stream decode runs on one GPU (across GPUs: one replica per GPU)");
  if (!m->embed) return fail(CH_ESTATE, "multi-stream decode embeds on the device: the model needs its embedding");
  if (m->ms_n) return fail(CH_ESTATE, "streams already initialised");
  const uint32_t cap = m->cfg.max_prefill_tokens ? m->cfg.max_prefill_tokens : 1024;
  if (n_streams == 0 || max_batch == 0 || max_batch > n_streams || max_batch > cap || max_batch > 64)
    return fail(CH_EINVAL, "streams: 1 <= max_batch <= n_streams, max_batch <= 64 and <= max_prefill_tokens");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  const int rc = init_streams(m, n_streams, max_batch);
  if (rc != CH_OK) {
    const std::string msg = g_err;
    free_streams(m);
    return fail(rc, msg);
  }
  return CH_OK;
}

extern "C" int ch_stream_prefill(ch_model *m, uint32_t stream, const uint32_t *tokens, uint32_t n,
                                 const uint32_t *slots, uint32_t start_clock, uint32_t num_prev, uint32_t *token_out) {
  if (!m) return fail(CH_EINVAL, "NULL model");
  if (stream >= m->ms_n) return fail(CH_EINVAL, "stream index >= the streams initialised");
  ch_topk top[64];
  CH_TRY(prefill_impl(m, tokens, n, nullptr, slots, start_clock, num_prev, token_out ? top : nullptr, nullptr, 0,
                      nullptr, nullptr,
                      (int)stream));
  if (token_out) *token_out = top[0].id;
  return CH_OK;
}

// The device work of one batched step once its inputs are staged: embedding, the layers,
// the LM head and the argmax -- about 17 launches per layer, captured into a CUDA graph
// per batch size (their arguments depend only on the batch size and the model).
#define SK_TRY(x)                         \
  do {                                    \
    const cudaError_t e_ = (x);           \
    if (e_ != cudaSuccess) return e_;     \
  } while (0)
static cudaError_t enqueue_streams_step(ch_model *m, uint32_t n, cudaStream_t s) {
  const uint32_t cap = m->ms_cap, rh = m->cfg.rotary_dim / 2, qkvd = m->qd + 2 * m->kvd;
  SK_TRY(launch_embed_rows(m->embed, m->ms_tok, n, m->H, sqrtf((float)m->H), m->pX, s));
  const float eps = m->cfg.rms_norm_eps;
  uint32_t *err = m->ctx->err;
  // 17-64 tokens (the tcgen05 skinny GEMMs): the o and down epilogues run fused
  const bool fuse = n >= kSkinnyTcMinTokens && m->H % 64 == 0 && m->H <= 4096;
  for (uint32_t l = 0; l < m->L; l++) {
    DevLayer &dl = m->layers[l];
    if (l == 0) SK_TRY(launch_rmsnorm_rows(m->pX, dl.input_norm, m->pNX, n, m->H, eps, s));
    SK_TRY(launch_skinny_q4(dl.qkv, qkvd / 16, m->H, m->pNX, m->H, n, EPI_STORE, m->pQKV, qkvd, m->ms_xf, m->ms_skp,
                            err, s, fuse && l > 0));
    AttnArgs a{};
    a.qkv = m->pQKV;
    a.qkv_stride = qkvd;
    a.q_norm_w = dl.q_norm;
    a.k_norm_w = dl.k_norm;
    a.rope_cs = m->ms_rope + (dl.full ? (size_t)cap * rh : 0);
    a.rope_stride = rh;
    a.k_cache = m->skc[l];
    a.v_cache = m->svc[l];
    a.stream = m->ms_stream;
    a.cache_stride = (size_t)kSlots * m->kvd;
    a.sp = m->ms_sp;
    a.is_sliding = dl.full ? 0 : 1;
    a.nq = m->nq;
    a.nkv = m->nkv;
    a.D = m->D;
    a.rot = m->cfg.rotary_dim;
    a.eps = eps;
    a.scale = 1.0f;  // Gemma-style: q/k norms replace 1/sqrt(d) (forward.zig:85)
    a.out = m->pA;
    a.out_stride = m->qd;
    a.partial = m->ms_partial;
    a.counters = m->ms_counters;
    a.err = err;
    a.cache_slots = kSlots;
    a.n_tok = n;
    // splits per (token, kv head): about 8 CTAs per SM over the whole batch (64 streams x 8
    // kv heads need 3; a single token keeps the model's split count)
    const uint32_t want = (8u * (uint32_t)num_sms() + n * m->nkv - 1) / (n * m->nkv);
    const int splits = (int)std::max(1u, std::min((uint32_t)m->attn_splits, want));
    SK_TRY(launch_decode_attn(a, splits, s, false));
    const float *next = (l + 1 < m->L) ? m->layers[l + 1].input_norm : m->final_norm;
    if (fuse) {
      // o and down end in one kernel each: split sum, post norm, residual add, the next
      // norm and the next GEMM's activation blocks (same operations, same order)
      uint8_t *xs = reinterpret_cast<uint8_t *>(m->ms_xf);
      uint32_t sk = 0;
      SK_TRY(launch_skinny_q4_tc(dl.o, m->H / 16, m->qd, m->pA, m->qd, n, xs, m->ms_skp, err, &sk, s));
      SK_TRY(launch_skinny_tail(m->ms_skp, sk, n, m->H, dl.post_attn, m->pX, dl.pre_ffn, m->pNX, eps, 1.0f, xs, s));
      SK_TRY(launch_skinny_q4(dl.gateup, 2 * m->I / 16, m->H, m->pNX, m->H, n, EPI_GELU_MUL, m->pACT, m->I, m->ms_xf,
                              m->ms_skp, err, s, true));
      SK_TRY(launch_skinny_q4_tc(dl.down, m->H / 16, m->I, m->pACT, m->I, n, xs, m->ms_skp, err, &sk, s));
      SK_TRY(launch_skinny_tail(m->ms_skp, sk, n, m->H, dl.post_ffn, m->pX, next, m->pNX, eps, dl.scalar,
                                l + 1 < m->L ? xs : nullptr, s));
      continue;
    }
    SK_TRY(launch_skinny_q4(dl.o, m->H / 16, m->qd, m->pA, m->qd, n, EPI_STORE, m->pMO, m->H, m->ms_xf, m->ms_skp,
                             err, s));
    if (dl.post_attn) SK_TRY(launch_rmsnorm_rows(m->pMO, dl.post_attn, m->pMO, n, m->H, eps, s));
    SK_TRY(launch_add_rmsnorm_rows(m->pX, m->pMO, dl.pre_ffn, m->pNX, n, m->H, eps, 1.0f, s));
    SK_TRY(launch_skinny_q4(dl.gateup, 2 * m->I / 16, m->H, m->pNX, m->H, n, EPI_GELU_MUL, m->pACT, m->I, m->ms_xf,
                             m->ms_skp, err, s));
    SK_TRY(launch_skinny_q4(dl.down, m->H / 16, m->I, m->pACT, m->I, n, EPI_STORE, m->pMO, m->H, m->ms_xf,
                             m->ms_skp, err, s));
    if (dl.post_ffn) SK_TRY(launch_rmsnorm_rows(m->pMO, dl.post_ffn, m->pMO, n, m->H, eps, s));
    SK_TRY(launch_add_rmsnorm_rows(m->pX, m->pMO, next, m->pNX, n, m->H, eps, dl.scalar, s));
  }
  {  // Q8 LM head of every token's final-normed state, the head read once for the batch
    LmHeadArgs h{};
    h.tiles = m->lm;
    h.row_tiles = m->V / 16;
    h.K = m->H;
    h.V = m->V;
    h.B = n;
    h.logits = m->ms_logits;
    h.err = err;
    SK_TRY(launch_lmhead_q8(m->pNX, m->H, h, m->ms_xf, s));
  }
  SK_TRY(launch_argmax_rows(m->ms_logits, n, m->V, m->ms_ids, s));
  return cudaSuccess;
}
#undef SK_TRY

extern "C" int ch_streams_decode(ch_model *m, const ch_stream_step *steps, uint32_t n, uint32_t *tokens_out) {
  if (!m || !steps || !tokens_out) return fail(CH_EINVAL, "NULL argument");
  if (!m->ms_n) return fail(CH_ESTATE, "ch_streams_init first");
  if (n == 0 || n > m->ms_cap) return fail(CH_EBATCH, "BatchTooLarge: 1..max_batch tokens per step");
  std::vector<uint8_t> seen(m->ms_n, 0);
  for (uint32_t b = 0; b < n; b++) {
    const ch_stream_step &st = steps[b];
    if (st.stream >= m->ms_n) return fail(CH_EINVAL, "stream index >= the streams initialised");
    if (seen[st.stream]++) return fail(CH_EINVAL, "a stream appears twice in one step");
    if (st.token >= m->V) return fail(CH_EINVAL, "token id >= vocab");
    if (st.slot >= kSlots) return fail(CH_EINVAL, "slot >= 4096");
    CH_TRY(check_lists(st.active, st.n_active));
    CH_TRY(check_lists(st.sliding, st.n_sliding));
  }
  CH_CUDA(cudaSetDevice(m->ctx->device));
  cudaStream_t s = m->ctx->stream;
  const uint32_t cap = m->ms_cap, rh = m->cfg.rotary_dim / 2;
  uint32_t *h_tok = m->h_ms_u32, *h_str = h_tok + cap, *h_ids = h_str + cap, *h_lists = h_ids + cap;
  for (uint32_t b = 0; b < n; b++) {
    const ch_stream_step &st = steps[b];
    h_tok[b] = st.token;
    h_str[b] = st.stream;
    uint32_t *la = h_lists + (size_t)b * 2 * kSlots;
    if (st.n_active) memcpy(la, st.active, st.n_active * 4);
    if (st.n_sliding) memcpy(la + kSlots, st.sliding, st.n_sliding * 4);
    StepParams &sp = m->h_ms_sp[b];
    sp = StepParams{};
    sp.clock = st.clock;
    sp.slot = st.slot;
    sp.n_active = st.n_active;
    sp.n_sliding = st.n_sliding;
    sp.active = m->ms_lists + (size_t)b * 2 * kSlots;
    sp.sliding = m->ms_lists + (size_t)b * 2 * kSlots + kSlots;
    rope_table(m->h_inv_s, st.clock, m->h_ms_rope + (size_t)b * rh);
    rope_table(m->h_inv_f, st.clock, m->h_ms_rope + ((size_t)cap + b) * rh);
  }
  CH_CUDA(cudaMemcpyAsync(m->ms_tok, h_tok, n * 4, cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->ms_stream, h_str, n * 4, cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->ms_lists, h_lists, (size_t)n * 2 * kSlots * 4, cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->ms_sp, m->h_ms_sp, n * sizeof(StepParams), cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->ms_rope, m->h_ms_rope, (size_t)n * rh * sizeof(float2), cudaMemcpyHostToDevice, s));
  CH_CUDA(cudaMemcpyAsync(m->ms_rope + (size_t)cap * rh, m->h_ms_rope + (size_t)cap * rh, (size_t)n * rh * sizeof(float2),
                          cudaMemcpyHostToDevice, s));
  if (m->ms_exec.size() <= n) m->ms_exec.resize(n + 1, nullptr);
  if (!m->ms_exec[n]) {
    cudaGraph_t g = nullptr;
    CH_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_streams_step(m, n, s);
    const cudaError_t e2 = cudaStreamEndCapture(s, &g);
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&m->ms_exec[n], g, 0);
    if (g) cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      m->ms_exec[n] = nullptr;
      cudaGetLastError();
      return fail(CH_ECUDA, std::string("streams step capture: ") + cudaGetErrorString(e));
    }
  }
  CH_CUDA(cudaGraphLaunch(m->ms_exec[n], s));
  CH_CUDA(cudaMemcpyAsync(h_ids, m->ms_ids, n * 4, cudaMemcpyDeviceToHost, s));
  CH_CUDA(cudaStreamSynchronize(s));
  memcpy(tokens_out, h_ids, n * 4);
  uint32_t f = 0;
  CH_TRY(ch_ctx_device_status(m->ctx, &f));
  return status_from_flags(f);
}

// State of the last ch_streams_decode step, token b = the step's b-th entry: the
// final-normed hidden state each token's LM head read, and its raw (pre-softcap) logits.
extern "C" int ch_streams_read_normed_x(ch_model *m, uint32_t n, float *out) {
  if (!m || !out) return fail(CH_EINVAL, "NULL argument");
  if (!m->ms_n) return fail(CH_ESTATE, "ch_streams_init first");
  if (n == 0 || n > m->ms_cap) return fail(CH_EINVAL, "1..max_batch rows");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  CH_CUDA(cudaMemcpy(out, m->pNX, (size_t)n * m->H * 4, cudaMemcpyDeviceToHost));
  return CH_OK;
}
extern "C" int ch_streams_read_logits(ch_model *m, uint32_t n, float *out) {
  if (!m || !out) return fail(CH_EINVAL, "NULL argument");
  if (!m->ms_n) return fail(CH_ESTATE, "ch_streams_init first");
  if (n == 0 || n > m->ms_cap) return fail(CH_EINVAL, "1..max_batch rows");
  CH_CUDA(cudaSetDevice(m->ctx->device));
  CH_CUDA(cudaStreamSynchronize(m->ctx->stream));
  CH_CUDA(cudaMemcpy(out, m->ms_logits, (size_t)n * m->V * 4, cudaMemcpyDeviceToHost));
  return CH_OK;
}

// ---------------------------------------------------------------------------
// op-level entry points
extern "C" size_t ch_q4_tile_bytes(uint32_t rows, uint32_t cols) { return q4_tile_bytes(rows, cols); }
extern "C" size_t ch_q8_tile_bytes(uint32_t rows, uint32_t cols) { return q8_tile_bytes(rows, cols); }
extern "C" int ch_q4_pack(ch_ctx *c, const uint32_t *blocks, uint32_t rows, uint32_t cols, void *tiles) {
  if (!c || !blocks || !tiles || rows % 16 || cols % 64) return fail(CH_EINVAL, "q4_pack: rows % 16, cols % 64");
  CH_CUDA(launch_repack_q4(blocks, nullptr, rows, cols, MAP_PLAIN, (uint8_t *)tiles, c->stream));
  return CH_OK;
}
extern "C" int ch_q4_pack_gateup(ch_ctx *c, const uint32_t *gate, const uint32_t *up, uint32_t rows, uint32_t cols,
                                 void *tiles) {
  if (!c || !gate || !up || !tiles || rows % 8 || cols % 64) return fail(CH_EINVAL, "q4_pack_gateup: rows % 8, cols % 64");
  CH_CUDA(launch_repack_q4(gate, up, 2 * rows, cols, MAP_GATEUP, (uint8_t *)tiles, c->stream));
  return CH_OK;
}
extern "C" int ch_q8_pack(ch_ctx *c, const uint32_t *blocks, uint32_t rows, uint32_t cols, void *tiles) {
  if (!c || !blocks || !tiles || rows % 16 || cols % 32) return fail(CH_EINVAL, "q8_pack: rows % 16, cols % 32");
  CH_CUDA(launch_repack_q8(blocks, rows, cols, (uint8_t *)tiles, c->stream));
  return CH_OK;
}
static int op_gemv(ch_ctx *c, int fmt, int epi, const void *tiles, uint32_t rows_tiles16, uint32_t cols,
                   const float *x, float *y) {
  CH_TRY(ctx_ensure_gemv(c, rows_tiles16));
  GemvArgs a;
  GemvPlan p;
  p.fmt = fmt;
  p.epi = epi;
  a.tiles = (const uint8_t *)tiles;
  a.row_tiles = rows_tiles16;
  a.k_tiles = fmt == FMT_Q4 ? cols / 64 : cols / 32;
  a.K = cols;
  a.x = x;
  a.y = y;
  a.partial = c->gemv_partial;
  a.counters = c->gemv_counters;
  a.err = c->err;
  // programmatic dependent launch: the weight stream starts while the previous
  // kernel on the stream finishes; x and the scratch are read after it completes
  CH_CUDA(launch_gemv(p, a, c->stream, true));
  return CH_OK;
}
extern "C" int ch_gemv_q4(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x, float *y) {
  if (!c || !tiles || !x || !y || rows % 16 || cols % 64 || rows == 0) return fail(CH_EINVAL, "gemv_q4 arguments");
  return op_gemv(c, FMT_Q4, EPI_STORE, tiles, rows / 16, cols, x, y);
}
extern "C" int ch_fused_mlp_q4(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x, float *act) {
  if (!c || !tiles || !x || !act || rows % 8 || cols % 64 || rows == 0) return fail(CH_EINVAL, "fused_mlp_q4 arguments");
  return op_gemv(c, FMT_Q4, EPI_GELU_MUL, tiles, 2 * rows / 16, cols, x, act);
}
extern "C" int ch_gemv_q8(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x, float *y) {
  if (!c || !tiles || !x || !y || rows % 16 || cols % 32 || rows == 0) return fail(CH_EINVAL, "gemv_q8 arguments");
  return op_gemv(c, FMT_Q8, EPI_STORE, tiles, rows / 16, cols, x, y);
}
extern "C" int ch_rmsnorm(ch_ctx *c, const float *x, const float *w, float *y, uint32_t n, uint32_t h, float eps) {
  if (!c || !x || !w || !y) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(launch_rmsnorm_rows(x, w, y, n, h, eps, c->stream));
  return CH_OK;
}
extern "C" int ch_add_rmsnorm(ch_ctx *c, float *x, const float *r, const float *w, float *y, uint32_t n, uint32_t h,
                              float eps, float scalar) {
  if (!c || !x || !r || !w || !y) return fail(CH_EINVAL, "NULL argument");
  CH_CUDA(launch_add_rmsnorm_rows(x, r, w, y, n, h, eps, scalar, c->stream));
  return CH_OK;
}
// batch_causal_attn.wgsl:25-223 on its own: token t of the batch attends to
// slots[0 .. num_prev + t + 1) (the last 1,024 of them on a sliding layer)
extern "C" int ch_batch_causal_attention(ch_ctx *c, const float *q, const void *k_cache, const void *v_cache,
                                         const uint32_t *slots, uint32_t n_tokens, uint32_t num_prev, uint32_t nq,
                                         uint32_t nkv, uint32_t head_dim, float scale, int is_sliding, float *out) {
  if (!c || !q || !k_cache || !v_cache || !slots || !out) return fail(CH_EINVAL, "NULL argument");
  if (head_dim != 256 || nkv == 0 || nq % nkv || n_tokens == 0 || num_prev + n_tokens > kSlots)
    return fail(CH_EINVAL, "batch_causal_attention: head_dim 256, nq % nkv == 0, 1 <= num_prev + n <= 4096");
  BatchAttnArgs a{q, static_cast<const __half *>(k_cache), static_cast<const __half *>(v_cache), slots, n_tokens,
                  num_prev, nq, nkv, head_dim, scale, is_sliding ? 1 : 0, out};
  CH_CUDA(launch_batch_causal_attn(a, c->stream));
  return CH_OK;
}
extern "C" int ch_decode_attention(ch_ctx *c, const float *qkv, const float *q_norm, const float *k_norm, void *k_cache,
                                   void *v_cache, const uint32_t *slots_dev, uint32_t n_slots, uint32_t clock,
                                   uint32_t slot, uint32_t nq, uint32_t nkv, uint32_t head_dim, uint32_t rot, float theta,
                                   float eps, float scale, float *out) {
  if (!c || !qkv || !q_norm || !k_norm || !k_cache || !v_cache || !out || (n_slots && !slots_dev))
    return fail(CH_EINVAL, "NULL argument");
  if (head_dim != 256 || nkv == 0 || nq % nkv || n_slots > kSlots || slot >= kSlots || rot > head_dim || (rot & 1))
    return fail(CH_EINVAL, "decode_attention shape");
  const uint32_t R = nq / nkv;
  if (R != 1 && R != 2 && R != 4 && R != 8) return fail(CH_EINVAL, "GQA ratio must be 1, 2, 4 or 8");
  const int splits = attn_default_splits(nkv);
  const size_t need = attn_partial_floats(nkv, R, head_dim, splits);
  if (c->attn_partial_n < need) {
    cudaFree(c->attn_partial);
    c->attn_partial = nullptr;
    CH_TRY(dmalloc(&c->attn_partial, need));
    c->attn_partial_n = need;
  }
  if (c->attn_counters_n < nkv) {
    cudaFree(c->attn_counters);
    c->attn_counters = nullptr;
    CH_TRY(dmalloc(&c->attn_counters, nkv));
    c->attn_counters_n = nkv;
    CH_CUDA(cudaMemsetAsync(c->attn_counters, 0, nkv * 4, c->stream));
  }
  if (c->attn_rope_n < rot / 2) {
    cudaFree(c->attn_rope);
    c->attn_rope = nullptr;
    CH_TRY(dmalloc(&c->attn_rope, 128));
    c->attn_rope_n = 128;
  }
  std::vector<float> f(rot / 2);
  for (uint32_t i = 0; i < rot / 2; i++) {
    float e = (2.0f * (float)i) / (float)rot;
    f[i] = (float)(1.0 / pow((double)theta, (double)e));
  }
  std::vector<float2> cs(rot / 2);
  rope_table(f, clock, cs.data());
  StepParams sp{clock, slot, n_slots, n_slots, slots_dev, slots_dev, 0, 0};
  CH_CUDA(cudaMemcpyAsync(c->attn_rope, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice, c->stream));
  CH_CUDA(cudaMemcpyAsync(c->op_sp, &sp, sizeof(sp), cudaMemcpyHostToDevice, c->stream));
  AttnArgs a{};
  a.qkv = qkv;
  a.q_norm_w = q_norm;
  a.k_norm_w = k_norm;
  a.rope_cs = c->attn_rope;
  a.k_cache = (__half *)k_cache;
  a.v_cache = (__half *)v_cache;
  a.sp = c->op_sp;
  a.is_sliding = 0;
  a.nq = nq;
  a.nkv = nkv;
  a.D = head_dim;
  a.rot = rot;
  a.eps = eps;
  a.scale = scale;
  a.out = out;
  a.partial = c->attn_partial;
  a.counters = c->attn_counters;
  a.err = c->err;
  a.cache_slots = kSlots;
  CH_CUDA(launch_decode_attn(a, splits, c->stream, false));
  // host staging above is synchronous-by-contract: wait so the stack copies stay valid
  CH_CUDA(cudaStreamSynchronize(c->stream));
  return CH_OK;
}
extern "C" int ch_topk64(ch_ctx *c, const float *logits, uint32_t V, uint32_t *ids, float *vals) {
  if (!c || !logits || !ids || !vals || V == 0 || V > 262144) return fail(CH_EINVAL, "topk64 arguments");
  TopkArgs t{};
  t.logits = logits;
  t.V = V;
  t.cand = c->topk_cand;
  t.counter = c->topk_counter;
  t.ids = ids;
  t.vals = vals;
  t.err = c->err;
  CH_CUDA(launch_topk64(t, c->stream, false));
  return CH_OK;
}
// 17..64 tokens: the skinny tcgen05 GEMM of the multi-stream decode step (skinny_tc.cu),
// whose cost does not depend on the token count; scratch: after the prefill GEMM's split-K
// counters (the first 16 KB, which stay zero), its token blocks, then the split-K partials
static int batch_gemm_skinny(ch_ctx *c, const void *tiles, uint32_t M, uint32_t K, const float *x, uint32_t n, int epi,
                             float *y, uint32_t ldy) {
  const size_t x0 = 16384, xw = (skinny_x_words(n, K) * 4 + 255) & ~(size_t)255;
  CH_TRY(ctx_ensure_xs(c, x0 + xw + skinny_partial_floats(n, M / 16, K) * sizeof(float)));
  CH_CUDA(launch_skinny_q4((const uint8_t *)tiles, M / 16, K, x, K, n, epi, y, ldy,
                           reinterpret_cast<uint32_t *>(c->xs + x0), reinterpret_cast<float *>(c->xs + x0 + xw), c->err,
                           c->stream));
  return CH_OK;
}
extern "C" int ch_batch_gemm_q4(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x, uint32_t n,
                                float *y) {
  if (!c || !tiles || !x || !y || rows % 16 || cols % 64) return fail(CH_EINVAL, "batch_gemm_q4 arguments");
  if (n == 0) return CH_OK;
  if (n >= kSkinnyTcMinTokens && n <= 64) return batch_gemm_skinny(c, tiles, rows, cols, x, n, EPI_STORE, y, rows);
  CH_TRY(ctx_ensure_xs(c, tc_gemm_scratch_bytes(n, rows, cols)));
  CH_CUDA(launch_batch_gemm_q4_tc(BatchGemmArgs{(const uint8_t *)tiles, rows, cols, n, x, y, EPI_STORE}, c->xs, c->xs_n, c->err,
                                  c->stream));
  return CH_OK;
}
extern "C" int ch_batch_fused_mlp_q4(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x,
                                     uint32_t n, float *act) {
  if (!c || !tiles || !x || !act || rows % 8 || cols % 64) return fail(CH_EINVAL, "batch_fused_mlp_q4 arguments");
  if (n == 0) return CH_OK;
  if (n >= kSkinnyTcMinTokens && n <= 64)
    return batch_gemm_skinny(c, tiles, 2 * rows, cols, x, n, EPI_GELU_MUL, act, rows);
  CH_TRY(ctx_ensure_xs(c, tc_gemm_scratch_bytes(n, 2 * rows, cols)));
  CH_CUDA(launch_batch_gemm_q4_tc(BatchGemmArgs{(const uint8_t *)tiles, 2 * rows, cols, n, x, act, EPI_GELU_MUL}, c->xs,
                                  c->xs_n, c->err, c->stream));
  return CH_OK;
}
// the same two GEMMs on the legacy mma.sync tensor path, kept as the measured baseline
extern "C" int ch_batch_gemm_q4_mma(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x,
                                    uint32_t n, float *y) {
  if (!c || !tiles || !x || !y || rows % 16 || cols % 64) return fail(CH_EINVAL, "batch_gemm_q4 arguments");
  CH_CUDA(launch_batch_gemm_q4(BatchGemmArgs{(const uint8_t *)tiles, rows, cols, n, x, y, EPI_STORE}, c->stream));
  return CH_OK;
}
extern "C" int ch_batch_fused_mlp_q4_mma(ch_ctx *c, const void *tiles, uint32_t rows, uint32_t cols, const float *x,
                                         uint32_t n, float *act) {
  if (!c || !tiles || !x || !act || rows % 8 || cols % 64) return fail(CH_EINVAL, "batch_fused_mlp_q4 arguments");
  CH_CUDA(launch_batch_gemm_q4(BatchGemmArgs{(const uint8_t *)tiles, 2 * rows, cols, n, x, act, EPI_GELU_MUL}, c->stream));
  return CH_OK;
}
extern "C" int ch_gen_q4_blocks(ch_ctx *c, uint32_t *dst, uint32_t rows, uint32_t cols, uint64_t tseed, float sstd) {
  if (!c || !dst || cols % 32) return fail(CH_EINVAL, "gen_q4_blocks arguments");
  CH_CUDA(launch_gen_q4_blocks(dst, rows, cols, tseed, sstd, c->stream));
  return CH_OK;
}
extern "C" int ch_gen_bf16(ch_ctx *c, uint16_t *dst, size_t n, uint64_t tseed, float mean, float std) {
  if (!c || !dst) return fail(CH_EINVAL, "gen_bf16 arguments");
  CH_CUDA(launch_gen_bf16(dst, n, tseed, mean, std, c->stream));
  return CH_OK;
}
extern "C" int ch_quantize_q8_rows(ch_ctx *c, const uint16_t *src, uint32_t rows, uint32_t cols, uint32_t *dst) {
  if (!c || !src || !dst || cols % 32) return fail(CH_EINVAL, "quantize_q8_rows arguments");
  CH_CUDA(launch_quantize_q8_rows(src, rows, cols, dst, c->stream));
  return CH_OK;
}
extern "C" int ch_quantize_q4_rows(ch_ctx *c, const uint16_t *src, uint32_t rows, uint32_t cols, uint32_t *dst) {
  if (!c || !src || !dst || cols % 32) return fail(CH_EINVAL, "quantize_q4_rows arguments");
  CH_CUDA(launch_quantize_q4_rows(src, rows, cols, dst, c->stream));
  return CH_OK;
}
