// Host side of the verify pass: the shard object behind the C ABI of include/potpori_b200.h.
//
// A shard owns, on one device: the packed BF16 weights of its layers (QKV concatenated,
// gate/up interleaved in 64-row blocks, rows padded to 128 and K to 64 with zeros so every
// TMA box is in bounds), F32 norms, the F32 KV cache in head-major [n_kv][capacity][128]
// layout, a RoPE table [capacity][head_dim/2] of (cos, sin) computed once in double precision,
// activation buffers for up to 8 rows, and the scratch of the stream-K GEMV and split-KV
// attention. One step is a fixed sequence of kernels that reads pos/m/tokens from a device
// header, so it is captured once per chunk width into a CUDA graph and replayed; kernels are
// chained with programmatic dependent launch so each GEMV streams its weights while the
// previous kernel drains.
#include <cuda.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/potpori_b200.h"
#include "pp_attn.cuh"
#include "pp_common.cuh"
#include "pp_decode.cuh"
#include "pp_gemv.cuh"
#include "pp_misc.cuh"
#include "pp_prefill_rows.cuh"

using namespace pp;

namespace {

thread_local std::string g_create_error;

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

typedef CUresult (*StreamWriteValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

StreamWriteValue32Fn write_value_fn() {
  static StreamWriteValue32Fn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (StreamWriteValue32Fn)p;
  }
  return fn;
}

// Bytes of one inbox slot: the step header (padded to 256) and kMaxRows hidden rows.
inline size_t inbox_slot_bytes(int64_t Hp) { return 256 + (size_t)kMaxRows * Hp * 4; }

inline float bits_to_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint64_t mix64h(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
uint64_t fnv1a(const char* s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (const unsigned char* p = (const unsigned char*)s; *p; ++p) {
    h ^= *p;
    h *= 0x100000001b3ull;
  }
  return h;
}
uint64_t tensor_key(uint64_t seed, const char* name) {
  return mix64h(seed * 0x9E3779B97F4A7C15ull ^ fnv1a(name));
}

enum MatId { M_Q, M_K, M_V, M_O, M_G, M_U, M_D, M_COUNT };
enum NormId { N_ATTN, N_QN, N_KN, N_FFN, N_COUNT };
const char* kMatNames[M_COUNT] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                                  "self_attn.o_proj", "mlp.gate_proj",    "mlp.up_proj",
                                  "mlp.down_proj"};
const char* kNormNames[N_COUNT] = {"input_layernorm", "self_attn.q_norm", "self_attn.k_norm",
                                   "post_attention_layernorm"};

struct LayerDev {
  uint16_t* wqkv = nullptr;  // [qkv_rows][Hp]
  uint16_t* wo = nullptr;    // [o_rows][Qp]
  uint16_t* wgu = nullptr;   // [gu_rows][Hp]
  uint16_t* wd = nullptr;    // [d_rows][Ip]
  float* norm[N_COUNT] = {};
  uint8_t* kc = nullptr;  // [n_kv][capacity] rows of kv_row_bytes(hd)
  uint8_t* vc = nullptr;
  bool mat_set[M_COUNT] = {};
  bool norm_set[N_COUNT] = {};
};

constexpr int kVariants = 5;  // chunk widths 1, 2, 4, 8, 16
constexpr int kRing = 64;     // in-flight headers / results per shard
inline int variant_of(int m) { return m <= 1 ? 0 : m <= 2 ? 1 : m <= 4 ? 2 : m <= 8 ? 3 : 4; }

}  // namespace

struct pp_shard {
  pp_shard_desc d;
  int H, Q, KV, I, hd, V, nh, nkv, G;
  int64_t Hp, Qp, Ip, Vp;
  int64_t qkv_rows, o_rows, gu_rows, d_rows;
  int first, last, nl;
  int dev = 0, num_sms = 148, smem_optin = 0;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  uint64_t bytes = 0;
  std::vector<LayerDev> L;
  uint16_t* embed = nullptr;  // [Vp][Hp]
  float* final_norm = nullptr;
  bool embed_set = false, final_norm_set = false;
  float2* rope = nullptr;
  float* x = nullptr;      // [kMaxRows][Hp]
  float* qbuf = nullptr;   // [kMaxRows][Q]
  uint8_t* attn_split = nullptr;  // attention output, split BF16 blocks (Qp / 64 x 4 KB)
  uint8_t* act_split = nullptr;   // SwiGLU output, split BF16 blocks (Ip / 64 x 4 KB)
  // Normalised GEMV operands split(x * w) (Hp / 64 x 4 KB) and the per-tile sums of squares
  // of x [ss_tiles][kMaxRows] they are scaled with: the attention input (QKV, and the vocab
  // head after the last layer) and the MLP input (gate/up).
  uint8_t* xw_attn = nullptr;
  uint8_t* xw_ffn = nullptr;
  float* ss_attn = nullptr;
  float* ss_ffn = nullptr;
  int ss_tiles = 1;
  float* logits = nullptr; // [kMaxRows][V]
  float* apart = nullptr;
  float* gpart = nullptr;
  uint32_t* tile_cnt = nullptr;
  ArgRec* recs = nullptr;
  uint32_t* done = nullptr;
  int32_t* d_decode = nullptr;  // [kDecodeMax + 1] greedy-decode picks and error bits
  int32_t* h_decode = nullptr;  // pinned copy
  StepDesc* d_desc = nullptr;
  StepResult* d_res = nullptr;
  StepDesc* h_desc = nullptr;      // pinned ring of kRing headers
  StepResult* h_res = nullptr;     // pinned: result of the host-synchronous path
  StepResult* h_slots = nullptr;   // pinned ring of kRing results (asynchronous path)
  cudaEvent_t desc_ev[kRing] = {};
  cudaEvent_t slot_ev[kRing] = {};
  cudaEvent_t handoff_ev = nullptr, handoff_done_ev = nullptr;
  // Cross-process link (pp_shard_inbox_export / pp_shard_outbox_open): this shard's inbox of
  // chunk slots (header + hidden rows) that the previous stage's process writes, and the next
  // stage's inbox opened through CUDA IPC.
  uint8_t* inbox = nullptr;
  uint32_t inbox_slots = 0;
  uint8_t* outbox = nullptr;
  uint32_t outbox_slots = 0;
  float* pf_peer = nullptr;  // the next stage's prefill rows, opened through CUDA IPC
  uint32_t desc_next = 0;
  float* h_stage = nullptr;  // pinned [kMaxRows][H]
  int splits = 1, nq_max = 1;
  int max_grid = 148;
  // Weight stages per GEMV CTA (16 KB each): 6 to 8 in flight per SM already stream the
  // vocabulary head at the measured HBM copy rate in a chain of launches; 12 is slightly
  // slower. PP_GEMV_STAGES overrides it (2..12).
  int gemv_max_stages = 8;
  int attn_per_sm = kAttnSplitsPerSm;  // attention key splits per KV head and SM of the budget
  bool use_graphs = true, use_pdl = true;
  cudaGraphExec_t exec[kVariants] = {};
  // Single-token decode kernel (pp_shard_set_decode_kernel): row-major weight copies and the
  // per-layer table on the device, its scratch, and whether the copies match the weights.
  bool dec_on = false, dec_stale = true;
  bool dec_graph = true;  // false once capturing the cooperative launch into a graph failed
  std::vector<uint16_t*> dec_w;  // [nl][4]: QKV, O, gate/up pairs, down
  DecodeLayer* dec_layers = nullptr;
  float *dec_qkv = nullptr, *dec_attn = nullptr, *dec_act = nullptr, *dec_part = nullptr;
  float* dec_opart = nullptr;  // [n_kv][H] each KV head's share of the O projection
  uint32_t* dec_sync = nullptr;
  int dec_vec = 0;
  size_t dec_budget = 0;  // dynamic shared memory the decode kernel may use
  uint64_t dec_wait_ns = kDecBarrierNs;  // barrier time limit (pp_shard_set_wait_test)
  int32_t dec_unreachable = 0;           // 1: the grid barriers wait for one CTA too many
  // Prompt prefill (pp_shard_prefill): F32 row buffers for up to kPrefillMax rows, the
  // projections' activation blocks (work) and error word, the prompt's tokens.
  struct {
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *gu = nullptr;
    void* work = nullptr;
    uint64_t work_bytes = 0;
    uint32_t* err = nullptr;
    int32_t* tokens = nullptr;
  } pf;
  // Tapped layers (pp_shard_set_taps): model layer numbers, ascending, and their output rows
  // [n_taps][kMaxRows][H] F32 written by every step.
  std::vector<int> taps;
  float* d_taps = nullptr;
  int taps_cap = 0;  // taps the buffer holds
  uint32_t launches = 0;                 // kernels of the step being enqueued
  std::vector<cudaEvent_t>* prof_events = nullptr;  // kernel-by-kernel timing (profile mode)
  std::vector<int>* prof_kinds = nullptr;
  uint32_t variant_launches[kVariants] = {};
  int last_variant = 0;
  std::string err;
};

namespace {

// Whether 1-row steps run on the persistent decode kernel (it does not write tapped outputs).
inline bool use_decode(const pp_shard* s) { return s->dec_on && s->taps.empty(); }

void drop_graphs(pp_shard* s) {
  for (auto& e : s->exec)
    if (e) {
      cudaGraphExecDestroy(e);
      e = nullptr;
    }
}

pp_status fail(pp_shard* s, pp_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (s)
    s->err = buf;
  else
    g_create_error = buf;
  return st;
}

#define CK(call)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(s, e_ == cudaErrorMemoryAllocation ? PP_E_OOM : PP_E_CUDA, "%s: %s", #call, \
                  cudaGetErrorString(e_));                                               \
  } while (0)

template <typename T>
pp_status dalloc(pp_shard* s, T** p, size_t bytes) {
  void* q = nullptr;
  CK(cudaMalloc(&q, bytes ? bytes : 16));
  CK(cudaMemsetAsync(q, 0, bytes ? bytes : 16, s->stream));
  s->allocs.push_back(q);
  s->bytes += bytes;
  *p = (T*)q;
  return PP_OK;
}

// ---- kernel table ---------------------------------------------------------------------------
pp_status after_launch(pp_shard* s, cudaStream_t st, int kind) {
  ++s->launches;
  if (s->prof_events) {
    cudaEvent_t e;
    CK(cudaEventCreate(&e));
    // External: a real event record node in the captured graph (timing works on replay).
    CK(cudaEventRecordWithFlags(e, st, cudaEventRecordExternal));
    s->prof_events->push_back(e);
    s->prof_kinds->push_back(kind);
  }
  return PP_OK;
}

template <int MT, int XM>
int gemv_stages(int64_t kp, size_t budget, int max_stages) {
  using Lay = GemvSmem<MT, XM>;
  int ns = max_stages;
  while (ns > 2 && Lay::total(ns, (int)kp) > budget) --ns;
  return ns;
}

// Dynamic shared memory a kernel may use: the opt-in limit minus its static shared memory.
template <typename K>
size_t dyn_smem_limit(pp_shard* s, K kern) {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return 0;
  return (size_t)s->smem_optin > fa.sharedSizeBytes ? (size_t)s->smem_optin - fa.sharedSizeBytes : 0;
}

template <int MT, int XM, int EPI>
pp_status launch_gemv(pp_shard* s, cudaStream_t st, const uint16_t* w, GemvArgs a) {
  a.w = w;
  using Lay = GemvSmem<MT, XM>;
  auto kern = pp_gemv_kernel<MT, XM, EPI>;
  const size_t budget = dyn_smem_limit(s, kern);
  a.nstages = gemv_stages<MT, XM>(a.kp, budget, s->gemv_max_stages);
  const size_t smem = Lay::total(a.nstages, a.kp);
  if (smem > budget)
    return fail(s, PP_E_UNSUPPORTED, "GEMV with K=%d needs %zu bytes of shared memory", a.k, smem);
  const int64_t T = (int64_t)a.tiles * a.kchunks;
  const int grid = (int)(T < s->max_grid ? T : s->max_grid);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = s->use_pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, kern, a));
  return after_launch(s, st, EPI == EPI_QKV      ? PP_K_QKV
                             : EPI == EPI_SWIGLU ? PP_K_GATE_UP
                             : EPI == EPI_ARGMAX ? PP_K_HEAD
                             : a.k == s->Q       ? PP_K_O
                                                 : PP_K_DOWN);
}

template <typename... KArgs, typename... Args>
pp_status launch_plain(pp_shard* s, cudaStream_t st, int kind, bool pdl, dim3 grid, dim3 block,
                       size_t smem, void (*kern)(KArgs...), Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (pdl && s->use_pdl) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, kern, args...));
  return after_launch(s, st, kind);
}

}  // namespace

// Validates the step header on the device, clears the result and stops every later kernel
// of a malformed step (a header that came from a peer instead of the host checks).
__global__ void pp_step_begin_kernel(const StepDesc* desc, StepResult* res, int32_t capacity,
                                  int32_t max_rows, int32_t vocab, int32_t first) {
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const int t = threadIdx.x;
  if (t < kMaxRows) {
    res->argmax[t] = -1;
    res->top1[t] = 0.f;
    res->top2[t] = 0.f;
  }
  if (t == 0) {
    res->nonfinite_rows = 0;
    res->n_accepted = 0;
    res->correction = -1;
    const StepDesc d = *desc;
    bool bad = d.pos < 0 || d.m < 1 || d.m > max_rows || (int64_t)d.pos + d.m > capacity ||
               d.n_drafts < 0 || d.n_drafts > kMaxRows;
    if (first && !bad)
      for (int r = 0; r < d.m; ++r) bad |= d.tokens[r] < 0 || d.tokens[r] >= vocab;
    res->status = bad ? ST_BAD_STEP : 0;
  }
}

// Greedy decode on the device (pp_shard_decode_greedy): after 1-row step i, record its pick
// and, if another step follows, make it the next step's token at the next position. Errors
// of the step (status bits, a non-finite row) accumulate in out[kDecodeMax].
constexpr int kDecodeMax = 64;
__global__ void pp_decode_feed_kernel(StepDesc* desc, const StepResult* res, int32_t* out,
                                   int32_t i, int32_t feed) {
  const int32_t t = res->argmax[0];
  out[i] = t;
  out[kDecodeMax] |= res->status | (t < 0 ? ST_NONFINITE_OUT : 0);
  if (feed) {
    desc->pos += 1;
    desc->tokens[0] = t < 0 ? 0 : t;  // keep later steps well-formed; the error is recorded
  }
}

namespace {

// Final norm + vocabulary projection + argmax/top-2/accept of a last shard (stream-K GEMV
// over the tied embedding, operand split(x * final_norm) in xw_attn).
template <int MT>
pp_status launch_head(pp_shard* s, cudaStream_t st) {
  GemvArgs h = {};
  h.desc = s->d_desc;
  h.res = s->d_res;
  h.partials = s->gpart;
  h.tile_cnt = s->tile_cnt;
  h.recs = s->recs;
  h.done_cnt = s->done;
  h.eps = s->d.cfg.rms_norm_eps;
  h.capacity = (int32_t)s->d.capacity;
  h.n_out = s->V;
  h.n_packed = (int32_t)s->Vp;
  h.k = s->H;
  h.kp = (int32_t)s->Hp;
  h.tiles = (int32_t)(s->Vp / kTileRows);
  h.kchunks = (int32_t)(s->Hp / kChunkK);
  h.xsplit = s->xw_attn;
  h.ss_in = s->ss_attn;
  h.ss_tiles = s->ss_tiles;
  h.logits = s->logits;
  return launch_gemv<MT, X_STREAM, EPI_ARGMAX>(s, st, s->embed, h);
}

// The kernels of one step for chunk width MT, in stream order.
template <int MT>
pp_status enqueue_step(pp_shard* s, cudaStream_t st) {
  s->launches = 0;
  pp_status r;
  if ((r = launch_plain(s, st, PP_K_BEGIN, false, dim3(1), dim3(32), 0, pp_step_begin_kernel, s->d_desc, s->d_res,
                        (int32_t)s->d.capacity, (int32_t)MT, (int32_t)s->V, (int32_t)s->first)))
    return r;
  {
    // Input rows (embedding or received hidden) and the first GEMV's operand.
    const float* w0 = s->nl ? s->L[0].norm[N_ATTN] : s->final_norm;
    PrepArgs pa = {};
    pa.table = s->first ? s->embed : nullptr;
    pa.hidden = s->H;
    pa.kchunks = (int32_t)(s->Hp / kChunkK);
    pa.vocab = s->V;
    pa.x = s->x;
    pa.ldx = (int32_t)s->Hp;
    pa.norm_w = w0;
    pa.xw = s->xw_attn;
    pa.ss = s->ss_attn;
    pa.desc = s->d_desc;
    pa.res = s->d_res;
    if ((r = launch_plain(s, st, PP_K_EMBED, true, dim3(s->ss_tiles, MT), dim3(128), 0,
                          pp_input_prep_kernel<MT>, pa, (int32_t)s->d.capacity)))
      return r;
  }
  for (int l = 0; l < s->nl; ++l) {
    LayerDev& Ld = s->L[l];
    GemvArgs a = {};
    a.desc = s->d_desc;
    a.res = s->d_res;
    a.partials = s->gpart;
    a.tile_cnt = s->tile_cnt;
    a.recs = s->recs;
    a.done_cnt = s->done;
    a.eps = s->d.cfg.rms_norm_eps;
    a.capacity = (int32_t)s->d.capacity;
    a.q_dim = s->Q;
    a.kv_dim = s->KV;
    a.head_dim = s->hd;
    // QKV with the input norm, QK-norm, RoPE and KV write.
    GemvArgs q = a;
    q.n_out = s->Q + 2 * s->KV;
    q.n_packed = (int32_t)s->qkv_rows;
    q.k = s->H;
    q.kp = (int32_t)s->Hp;
    q.tiles = (int32_t)(s->qkv_rows / kTileRows);
    q.kchunks = (int32_t)(s->Hp / kChunkK);
    q.xsplit = s->xw_attn;
    q.ss_in = s->ss_attn;
    q.ss_tiles = s->ss_tiles;
    q.out = s->qbuf;
    q.ldo = s->Q;
    q.qn = Ld.norm[N_QN];
    q.kn = Ld.norm[N_KN];
    q.rope = s->rope;
    q.kcache = Ld.kc;
    q.vcache = Ld.vc;
    if ((r = launch_gemv<MT, X_STREAM, EPI_QKV>(s, st, Ld.wqkv, q))) return r;
    // Attention.
    AttnArgs at = {};
    at.q = s->qbuf;
    at.kcache = Ld.kc;
    at.vcache = Ld.vc;
    at.part = s->apart;
    at.out_split = s->attn_split;
    at.n_heads = s->nh;
    at.n_kv = s->nkv;
    at.head_dim = s->hd;
    at.capacity = (int32_t)s->d.capacity;
    at.splits = s->splits;
    at.q_dim = (int32_t)s->Qp;
    at.nq_max = s->nq_max;
    at.scale = sqrtf((float)s->hd);
    at.desc = s->d_desc;
    at.res = s->d_res;
    AttnArgs atq = at;
    atq.q_dim = s->Q;  // the query buffer is [rows][Q]
    {
      // Split kernel reads q with stride Q; combine writes attn with stride Qp.
      const int qpw = (s->G * MT + 7) / 8;  // query tiles of 8 (G * MT query vectors)
      const size_t smem = attn_smem_bytes(s->hd, qpw);
      const dim3 grid(s->nkv, s->splits), block(kAttnThreads);
      r = qpw <= 1   ? launch_plain(s, st, PP_K_ATTN, true, grid, block, smem, pp_attn_split_kernel<MT, 1>, atq)
          : qpw <= 2 ? launch_plain(s, st, PP_K_ATTN, true, grid, block, smem, pp_attn_split_kernel<MT, 2>, atq)
          : qpw <= 4 ? launch_plain(s, st, PP_K_ATTN, true, grid, block, smem, pp_attn_split_kernel<MT, 4>, atq)
                     : launch_plain(s, st, PP_K_ATTN, true, grid, block, smem, pp_attn_split_kernel<MT, 8>, atq);
      if (r) return r;
      const int tb = s->hd < 32 ? 32 : s->hd;
      if ((r = launch_plain(s, st, PP_K_ATTN_COMBINE, true, dim3(s->nh, MT), dim3(tb), 0,
                            pp_attn_combine_kernel<MT>, at)))
        return r;
    }
    // O projection + residual.
    GemvArgs o = a;
    o.n_out = s->H;
    o.n_packed = (int32_t)s->o_rows;
    o.k = s->Q;
    o.kp = (int32_t)s->Qp;
    o.tiles = (int32_t)(s->o_rows / kTileRows);
    o.kchunks = (int32_t)(s->Qp / kChunkK);
    o.xsplit = s->attn_split;
    o.out = s->x;
    o.ldo = (int32_t)s->Hp;
    o.xw_out = s->xw_ffn;
    o.wnext = Ld.norm[N_FFN];
    o.ss_out = s->ss_ffn;
    if ((r = launch_gemv<MT, X_STREAM, EPI_RESADD>(s, st, Ld.wo, o))) return r;
    // gate/up with the post-attention norm and SwiGLU.
    GemvArgs g = a;
    g.n_out = s->I;
    g.n_packed = (int32_t)s->gu_rows;
    g.k = s->H;
    g.kp = (int32_t)s->Hp;
    g.tiles = (int32_t)(s->gu_rows / kTileRows);
    g.kchunks = (int32_t)(s->Hp / kChunkK);
    g.xsplit = s->xw_ffn;
    g.ss_in = s->ss_ffn;
    g.ss_tiles = s->ss_tiles;
    g.out_split = s->act_split;
    if ((r = launch_gemv<MT, X_STREAM, EPI_SWIGLU>(s, st, Ld.wgu, g))) return r;
    // down + residual.
    GemvArgs dn = a;
    dn.n_out = s->H;
    dn.n_packed = (int32_t)s->d_rows;
    dn.k = s->I;
    dn.kp = (int32_t)s->Ip;
    dn.tiles = (int32_t)(s->d_rows / kTileRows);
    dn.kchunks = (int32_t)(s->Ip / kChunkK);
    dn.xsplit = s->act_split;
    dn.out = s->x;
    dn.ldo = (int32_t)s->Hp;
    // The next norm's operand: the next layer's input norm, the final norm after the last
    // layer of the model, none when the next layer lives on another shard.
    dn.wnext = l + 1 < s->nl ? s->L[l + 1].norm[N_ATTN] : s->last ? s->final_norm : nullptr;
    if (dn.wnext) {
      dn.xw_out = s->xw_attn;
      dn.ss_out = s->ss_attn;
    }
    if ((r = launch_gemv<MT, X_STREAM, EPI_RESADD>(s, st, Ld.wd, dn))) return r;
    // Tapped layer: keep its output rows (src/node.rs:152-157).
    for (size_t ti = 0; ti < s->taps.size(); ++ti)
      if (s->taps[ti] == (int)s->d.layer_begin + l)
        CK(cudaMemcpy2DAsync(s->d_taps + ti * (size_t)kMaxRows * s->H, (size_t)s->H * 4, s->x,
                             (size_t)s->Hp * 4, (size_t)s->H * 4, MT, cudaMemcpyDeviceToDevice, st));
  }
  if (s->last && (r = launch_head<MT>(s, st))) return r;
  return PP_OK;
}

// ---- single-token decode kernel ---------------------------------------------------------------
// Own residual rows of the smallest share of H a CTA of this grid gets, plus one.
inline int decode_own_cap(const pp_shard* s, int grid) { return (s->H + grid - 1) / grid + 1; }

pp_status decode_alloc(pp_shard* s) {
  if (s->dec_layers) return PP_OK;
  pp_status r;
  const int64_t H = s->H, Q = s->Q, KV = s->KV, I = s->I;
  s->dec_w.assign((size_t)s->nl * 4, nullptr);
  std::vector<DecodeLayer> tab(s->nl);
  const int64_t kH = dec_kpad(s->H), kI = dec_kpad(s->I);
  for (int l = 0; l < s->nl; ++l) {
    uint16_t** w = &s->dec_w[(size_t)l * 4];
    if ((r = dalloc(s, &w[0], (size_t)(Q + 2 * KV) * kH * 2))) return r;
    if ((r = dalloc(s, &w[1], (size_t)s->nkv * H * s->G * s->hd * 2))) return r;
    if ((r = dalloc(s, &w[2], (size_t)2 * I * kH * 2))) return r;
    if ((r = dalloc(s, &w[3], (size_t)H * kI * 2))) return r;
    const LayerDev& Ld = s->L[l];
    tab[l] = DecodeLayer{w[0], w[1], w[2], w[3], Ld.norm[N_ATTN], Ld.norm[N_QN], Ld.norm[N_KN],
                         Ld.norm[N_FFN], Ld.kc, Ld.vc};
  }
  if ((r = dalloc(s, &s->dec_layers, tab.size() * sizeof(DecodeLayer)))) return r;
  CK(cudaMemcpyAsync(s->dec_layers, tab.data(), tab.size() * sizeof(DecodeLayer),
                     cudaMemcpyHostToDevice, s->stream));
  const int max_splits = s->num_sms / s->nkv;
  if ((r = dalloc(s, &s->dec_qkv, (size_t)(Q + 2 * KV) * 4))) return r;
  if ((r = dalloc(s, &s->dec_attn, (size_t)Q * 4))) return r;
  if ((r = dalloc(s, &s->dec_act, (size_t)I * 4))) return r;
  if ((r = dalloc(s, &s->dec_opart, (size_t)s->nkv * H * 4))) return r;
  if ((r = dalloc(s, &s->dec_part, (size_t)s->nh * max_splits * (s->hd + 4) * 4))) return r;
  if ((r = dalloc(s, &s->dec_sync, (size_t)(2 + s->nkv) * 4))) return r;
  CK(cudaStreamSynchronize(s->stream));
  return PP_OK;
}

// Row-major copies of the packed weights (after any weight upload).
pp_status decode_rebuild(pp_shard* s) {
  const int64_t H = s->H, Q = s->Q, KV = s->KV, I = s->I;
  const int64_t kH = dec_kpad(s->H), kI = dec_kpad(s->I);
  for (int l = 0; l < s->nl; ++l) {
    uint16_t** w = &s->dec_w[(size_t)l * 4];
    const LayerDev& Ld = s->L[l];
    pp_untile_rows_kernel<<<1024, 256, 0, s->stream>>>(w[0], Ld.wqkv, Q + 2 * KV, H, kH, s->Hp / kChunkK, 0);
    pp_untile_o_heads_kernel<<<1024, 256, 0, s->stream>>>(w[1], Ld.wo, H, (int64_t)s->G * s->hd,
                                                          s->nkv, s->Qp / kChunkK);
    pp_untile_rows_kernel<<<1024, 256, 0, s->stream>>>(w[2], Ld.wgu, 2 * I, H, kH, s->Hp / kChunkK, 1);
    pp_untile_rows_kernel<<<1024, 256, 0, s->stream>>>(w[3], Ld.wd, H, I, kI, s->Ip / kChunkK, 0);
    CK(cudaGetLastError());
  }
  CK(cudaStreamSynchronize(s->stream));
  s->dec_stale = false;
  return PP_OK;
}

// A 1-row step of a whole-model shard: header check, one cooperative launch of the decode
// kernel over the shard's SM budget, the vocabulary head.
pp_status enqueue_decode_step(pp_shard* s, cudaStream_t st) {
  s->launches = 0;
  pp_status r;
  if ((r = launch_plain(s, st, PP_K_BEGIN, false, dim3(1), dim3(32), 0, pp_step_begin_kernel, s->d_desc, s->d_res,
                        (int32_t)s->d.capacity, (int32_t)1, (int32_t)s->V, (int32_t)s->first)))
    return r;
  CK(cudaMemsetAsync(s->dec_sync, 0, (size_t)(2 + s->nkv) * 4, st));
  const int grid = s->max_grid;
  // Ring slots: what the shared memory holds beside this grid's fixed part (at most 8).
  const size_t fixed = DecodeSmem(0, s->dec_vec, decode_own_cap(s, grid),
                                  decode_part_rows(s->H, s->Q, s->KV, s->I, s->nkv, grid))
                           .total();
  int ns = s->dec_budget > fixed ? (int)((s->dec_budget - fixed) / kDecSlot) : 0;
  ns = ns > 8 ? 8 : ns;
  if (ns < 2) return fail(s, PP_E_UNSUPPORTED, "the decode kernel's ring does not fit");
  DecodeArgs a = {};
  a.layers = s->dec_layers;
  a.nl = s->nl;
  a.H = s->H;
  a.Q = s->Q;
  a.KV = s->KV;
  a.I = s->I;
  a.hd = s->hd;
  a.nh = s->nh;
  a.nkv = s->nkv;
  a.G = s->G;
  a.V = s->V;
  a.capacity = (int32_t)s->d.capacity;
  a.embed_kchunks = (int32_t)(s->Hp / kChunkK);
  a.splits = grid / s->nkv;
  a.ss_tiles = s->ss_tiles;
  a.nslots = ns;
  a.kH = dec_kpad(s->H);
  a.kQ = dec_kpad(s->Q);
  a.kI = dec_kpad(s->I);
  a.kO = s->G * s->hd;
  a.vec_floats = s->dec_vec;
  a.eps = s->d.cfg.rms_norm_eps;
  a.inv_scale = 1.0f / sqrtf((float)s->hd);
  a.extra_arrivals = s->dec_unreachable;
  a.wait_ns = s->dec_wait_ns;
  a.embed = s->embed;
  a.final_norm = s->final_norm;
  a.rope = s->rope;
  a.qkv = s->dec_qkv;
  a.x = s->x;
  a.attn = s->dec_attn;
  a.act = s->dec_act;
  a.opart = s->dec_opart;
  a.part = s->dec_part;
  a.sync = s->dec_sync;
  a.xw_out = s->xw_attn;
  a.ss_out = s->ss_attn;
  a.desc = s->d_desc;
  a.res = s->d_res;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes =
      DecodeSmem(ns, s->dec_vec, decode_own_cap(s, grid),
                 decode_part_rows(s->H, s->Q, s->KV, s->I, s->nkv, grid)).total();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: they meet at grid barriers
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (s->G) {  // set_decode_kernel admits 1, 2 or 4 query heads per KV head
    case 1: CK(cudaLaunchKernelEx(&cfg, pp_decode_step_kernel<1>, a)); break;
    case 2: CK(cudaLaunchKernelEx(&cfg, pp_decode_step_kernel<2>, a)); break;
    default: CK(cudaLaunchKernelEx(&cfg, pp_decode_step_kernel<4>, a)); break;
  }
  if ((r = after_launch(s, st, PP_K_DECODE))) return r;
  return launch_head<1>(s, st);
}


// ---- prompt prefill ------------------------------------------------------------------------
constexpr int kPrefillMax = 2048;  // rows of one pp_shard_prefill call

pp_status prefill_alloc(pp_shard* s) {
  if (s->pf.x) return PP_OK;
  pp_status r;
  const size_t T = kPrefillMax;
  if ((r = dalloc(s, &s->pf.x, T * s->H * 4))) return r;
  if ((r = dalloc(s, &s->pf.qkv, T * (s->Q + 2 * s->KV) * 4))) return r;
  if ((r = dalloc(s, &s->pf.q, T * s->Q * 4))) return r;
  if ((r = dalloc(s, &s->pf.gu, T * s->gu_rows * 4))) return r;
  uint64_t wb = pp_rows_gemm_work_bytes((uint32_t)T, (uint32_t)s->H);
  const uint64_t cand[2] = {pp_rows_gemm_work_bytes((uint32_t)T, (uint32_t)s->Q),
                            pp_rows_gemm_work_bytes((uint32_t)T, (uint32_t)s->I)};
  for (uint64_t c : cand) wb = c > wb ? c : wb;
  uint8_t* w = nullptr;
  if ((r = dalloc(s, &w, wb + 1024))) return r;
  s->pf.work = (void*)(((uintptr_t)w + 1023) & ~(uintptr_t)1023);
  s->pf.work_bytes = wb;
  if ((r = dalloc(s, &s->pf.err, 16))) return r;
  if ((r = dalloc(s, &s->pf.tokens, T * 4))) return r;
  return PP_OK;
}

// y[t][n] (row stride ldy) = or += (accumulate) x . W^T on the tensor cores, x being the
// activation blocks in the shard's prefill work area.
pp_status prefill_gemm(pp_shard* s, const uint16_t* w, int n, int k, int t, float* y, int ldy,
                       bool accumulate) {
  const pp_status st = rows_gemm_blocks(w, (uint32_t)n, (uint32_t)k, (const uint8_t*)s->pf.work,
                                        (uint32_t)t, y, (uint32_t)ldy, accumulate, s->pf.err,
                                        s->stream);
  if (st) {
    char msg[256];
    pp_last_error(nullptr, msg, sizeof msg);
    return fail(s, st, "prompt projection: %s", msg);
  }
  return PP_OK;
}

// Every layer of a shard over t prompt rows at positions pos.. (embedding on the first shard,
// else the input rows already in pf.x; per layer RMSNorm into activation blocks, tcgen05 QKV,
// QK-norm + RoPE + K/V rows into the cache, flash-style causal attention over the whole chunk
// into activation blocks, tcgen05 O added to the residual rows, RMSNorm into blocks, tcgen05
// gate/up, SwiGLU into blocks, tcgen05 down added to the residual rows; the model's last
// layer stops after its K/V rows, which is all a prefill leaves behind, and a shard before
// the last leaves its output rows in pf.x for the next stage).
pp_status enqueue_prefill(pp_shard* s, uint32_t pos, int t) {
  cudaStream_t st = s->stream;
  const int H = s->H, Q = s->Q, KV = s->KV, I = s->I, hd = s->hd;
  const int kcH = (H + kChunkK - 1) / kChunkK, kcI = (I + kChunkK - 1) / kChunkK;
  const float eps = s->d.cfg.rms_norm_eps;
  uint8_t* xs = (uint8_t*)s->pf.work;
  pp_status r;
  CK(cudaMemsetAsync(s->pf.err, 0, 4, st));
  CK(cudaMemsetAsync(s->d_res, 0, sizeof(StepResult), st));
  if (s->first) {  // a later stage finds its input rows in pf.x
    pp_pre_embed_kernel<<<t, 256, 0, st>>>(s->embed, (int32_t)(s->Hp / kChunkK), s->pf.tokens, H, s->pf.x);
    CK(cudaGetLastError());
  }
  const int bq = (s->G <= 4 ? 64 : 128) / s->G;  // prompt rows per attention CTA
  const int64_t swiglu_units = (int64_t)t * kcI * 8;
  const int swiglu_grid = (int)((swiglu_units + 255) / 256 < 4096 ? (swiglu_units + 255) / 256 : 4096);
  for (int l = 0; l < s->nl; ++l) {
    LayerDev& Ld = s->L[l];
    pp_pre_norm_split_kernel<<<t, 256, 0, st>>>(s->pf.x, Ld.norm[N_ATTN], H, eps, kcH, xs);
    CK(cudaGetLastError());
    if ((r = prefill_gemm(s, Ld.wqkv, Q + 2 * KV, H, t, s->pf.qkv, Q + 2 * KV, false))) return r;
    pp_pre_qkv_kernel<<<dim3(t, (s->nh + 2 * s->nkv + 3) / 4), 256, 0, st>>>(
        s->pf.qkv, t, (int32_t)pos, s->nh, s->nkv, hd, eps, Ld.norm[N_QN], Ld.norm[N_KN], s->rope,
        Ld.kc, Ld.vc, (int32_t)s->d.capacity, s->pf.q);
    CK(cudaGetLastError());
    if (l + 1 == s->nl && s->last) break;  // the model's last layer: its K/V rows are all
    const dim3 fgrid(s->nkv, (t + bq - 1) / bq);
    if (s->G <= 4)
      pp_pre_flash_kernel<4, 2><<<fgrid, 128, flash_smem_bytes(4, 2), st>>>(
          s->pf.q, Ld.kc, Ld.vc, (int32_t)s->d.capacity, s->nh, s->nkv, (int32_t)pos, t,
          sqrtf((float)hd), xs, s->d_res);
    else
      pp_pre_flash_kernel<8, 3><<<fgrid, 256, flash_smem_bytes(8, 3), st>>>(
          s->pf.q, Ld.kc, Ld.vc, (int32_t)s->d.capacity, s->nh, s->nkv, (int32_t)pos, t,
          sqrtf((float)hd), xs, s->d_res);
    CK(cudaGetLastError());
    if ((r = prefill_gemm(s, Ld.wo, H, Q, t, s->pf.x, H, true))) return r;
    pp_pre_norm_split_kernel<<<t, 256, 0, st>>>(s->pf.x, Ld.norm[N_FFN], H, eps, kcH, xs);
    CK(cudaGetLastError());
    if ((r = prefill_gemm(s, Ld.wgu, (int)s->gu_rows, H, t, s->pf.gu, (int)s->gu_rows, false))) return r;
    pp_pre_swiglu_split_kernel<<<swiglu_grid, 256, 0, st>>>(s->pf.gu, (int32_t)s->gu_rows, I, t, kcI, xs);
    CK(cudaGetLastError());
    if ((r = prefill_gemm(s, Ld.wd, H, I, t, s->pf.x, H, true))) return r;
  }
  return PP_OK;
}

template <typename K>
pp_status set_max_smem(pp_shard* s, K kern) {
  const size_t lim = dyn_smem_limit(s, kern);
  if (!lim) return fail(s, PP_E_CUDA, "cudaFuncGetAttributes failed");
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim));
  return PP_OK;
}

template <int MT>
pp_status set_attrs_mt(pp_shard* s) {
  pp_status r;
  if ((r = set_max_smem(s, pp_gemv_kernel<MT, X_STREAM, EPI_QKV>)) ||
      (r = set_max_smem(s, pp_gemv_kernel<MT, X_STREAM, EPI_RESADD>)) ||
      (r = set_max_smem(s, pp_gemv_kernel<MT, X_STREAM, EPI_SWIGLU>)) ||
      (r = set_max_smem(s, pp_gemv_kernel<MT, X_STREAM, EPI_ARGMAX>)) ||
      (r = set_max_smem(s, pp_attn_split_kernel<MT, 1>)) ||
      (r = set_max_smem(s, pp_attn_split_kernel<MT, 2>)) ||
      (r = set_max_smem(s, pp_attn_split_kernel<MT, 4>)) ||
      (r = set_max_smem(s, pp_attn_split_kernel<MT, 8>)))
    return r;
  return PP_OK;
}

pp_status set_attrs(pp_shard* s) {
  pp_status r;
  if ((r = set_attrs_mt<1>(s)) || (r = set_attrs_mt<2>(s)) || (r = set_attrs_mt<4>(s)) ||
      (r = set_attrs_mt<8>(s)) || (r = set_attrs_mt<16>(s)) ||
      (r = set_max_smem(s, pp_decode_step_kernel<1>)) || (r = set_max_smem(s, pp_decode_step_kernel<2>)) ||
      (r = set_max_smem(s, pp_decode_step_kernel<4>)) ||
      (r = set_max_smem(s, pp_pre_flash_kernel<4, 2>)) ||
      (r = set_max_smem(s, pp_pre_flash_kernel<8, 3>)))
    return r;
  return PP_OK;
}

pp_status enqueue_variant(pp_shard* s, int vi, cudaStream_t st) {
  pp_status r;
  switch (vi) {
    case 0: r = use_decode(s) ? enqueue_decode_step(s, st) : enqueue_step<1>(s, st); break;
    case 1: r = enqueue_step<2>(s, st); break;
    case 2: r = enqueue_step<4>(s, st); break;
    case 3: r = enqueue_step<8>(s, st); break;
    default: r = enqueue_step<16>(s, st); break;
  }
  s->variant_launches[vi] = s->launches;
  return r;
}

// Launch one step of width variant vi on stream st: graph replay, or direct launches.
pp_status run_step(pp_shard* s, int vi, cudaStream_t st) {
  if (pp_shard_missing(s, nullptr, 0))
    return fail(s, PP_E_MISSING, "parameters missing; see pp_shard_missing");
  s->last_variant = vi;
  const bool dec = vi == 0 && use_decode(s);
  if (dec && s->dec_stale) {
    pp_status r = decode_rebuild(s);
    if (r) return r;
  }
  if (!s->use_graphs || (dec && !s->dec_graph)) return enqueue_variant(s, vi, st);
  if (!s->exec[vi]) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    pp_status r = enqueue_variant(s, vi, s->stream);
    cudaError_t e = cudaStreamEndCapture(s->stream, &g);
    const char* what = "graph capture";
    if (e == cudaSuccess && !r) {
      what = "graph instantiate";
      e = cudaGraphInstantiate(&s->exec[vi], g, 0);
      if (e != cudaSuccess) s->exec[vi] = nullptr;
    }
    if (g) cudaGraphDestroy(g);
    if (dec && (r || e != cudaSuccess)) {
      // A runtime that cannot capture the cooperative launch: launch the step directly.
      cudaGetLastError();
      s->err.clear();
      s->dec_graph = false;
      return enqueue_variant(s, vi, st);
    }
    if (r) return r;
    if (e != cudaSuccess) return fail(s, PP_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  CK(cudaGraphLaunch(s->exec[vi], st));
  s->last_variant = vi;
  return PP_OK;
}

pp_status status_of(pp_shard* s, const StepResult& r) {
  if (r.status & ST_TIMEOUT) return fail(s, PP_E_TIMEOUT, "a bounded device wait expired");
  if (r.status & ST_BAD_STEP) return fail(s, PP_E_INVALID, "invalid step header");
  if (r.status & ST_NONFINITE_IN) return fail(s, PP_E_INVALID, "invalid hidden input");
  if (r.status & ST_NONFINITE_OUT)
    return fail(s, PP_E_NONFINITE, "the shard produced missing or non-finite logits");
  return PP_OK;
}

void fill_verify(pp_shard* s, uint32_t m, pp_verify_out* v) {
  const StepResult& r = *s->h_res;
  for (uint32_t i = 0; i < m; ++i) {
    if (v->argmax) v->argmax[i] = r.argmax[i];
    if (v->top1) v->top1[i] = r.top1[i];
    if (v->top2) v->top2[i] = r.top2[i];
  }
  v->n_accepted = r.n_accepted;
  v->correction = r.correction;
  v->nonfinite_rows = r.nonfinite_rows;
}

// Next pinned header slot; waits (host) until its previous upload has been consumed.
StepDesc* next_desc(pp_shard* s, int* slot) {
  const int i = (int)(s->desc_next++ % kRing);
  cudaEventSynchronize(s->desc_ev[i]);
  *slot = i;
  return &s->h_desc[i];
}

pp_status upload_desc(pp_shard* s, int slot, cudaStream_t st) {
  CK(cudaMemcpyAsync(s->d_desc, &s->h_desc[slot], sizeof(StepDesc), cudaMemcpyHostToDevice, st));
  CK(cudaEventRecord(s->desc_ev[slot], st));
  return PP_OK;
}

pp_status check_step(pp_shard* s, uint32_t pos, uint32_t m) {
  // src/qwen/model.rs:373-381
  if (m == 0 || (uint64_t)pos + m > s->d.capacity)
    return fail(s, PP_E_INVALID, "chunk exceeds KV capacity");
  if (s->d.chunk != 0 && m != 1 && m != s->d.chunk)
    return fail(s, PP_E_INVALID, "unsupported verify chunk size");
  if (m > (uint32_t)kMaxRows) return fail(s, PP_E_UNSUPPORTED, "chunks above 16 rows are not built");
  if (m > 8 && s->G > 4)
    return fail(s, PP_E_UNSUPPORTED, "16-row chunks need at most 4 query heads per KV head");
  return PP_OK;
}

// Common tail of the host-buffer forwards: enqueue, copy out, synchronise, report.
pp_status finish_host_step(pp_shard* s, uint32_t m, float* out_hidden, pp_verify_out* verify) {
  const int vi = variant_of((int)m);
  pp_status r = run_step(s, vi, s->stream);
  if (r) return r;
  if (!s->last && out_hidden)
    CK(cudaMemcpy2DAsync(s->h_stage, (size_t)s->H * 4, s->x, (size_t)s->Hp * 4, (size_t)s->H * 4, m,
                         cudaMemcpyDeviceToHost, s->stream));
  CK(cudaMemcpyAsync(s->h_res, s->d_res, sizeof(StepResult), cudaMemcpyDeviceToHost, s->stream));
  if (s->last && verify && verify->logits)
    CK(cudaMemcpyAsync(verify->logits, s->logits, (size_t)m * s->V * 4, cudaMemcpyDeviceToHost,
                       s->stream));
  CK(cudaStreamSynchronize(s->stream));
  if (!s->last && out_hidden) memcpy(out_hidden, s->h_stage, (size_t)m * s->H * 4);
  if (s->last && verify) fill_verify(s, m, verify);
  return status_of(s, *s->h_res);
}

// ---- minimal safetensors header reader ---------------------------------------------------
struct StEntry {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;
};

struct JsonCursor {
  const char* p;
  const char* e;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) ++p;
      out.push_back(*p++);
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool num(int64_t& v) {
    ws();
    char* end = nullptr;
    v = strtoll(p, &end, 10);
    if (end == p) return false;
    p = end;
    return true;
  }
  bool skip() {  // skip any value
    ws();
    if (p >= e) return false;
    if (*p == '"') {
      std::string t;
      return str(t);
    }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      int depth = 0;
      bool in_str = false;
      for (; p < e; ++p) {
        if (in_str) {
          if (*p == '\\') ++p;
          else if (*p == '"') in_str = false;
        } else if (*p == '"') in_str = true;
        else if (*p == open) ++depth;
        else if (*p == close && --depth == 0) {
          ++p;
          return true;
        }
      }
      return false;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
  bool lit(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
};

bool parse_entry(JsonCursor& j, StEntry& out) {
  if (!j.lit('{')) return false;
  while (true) {
    std::string key;
    if (!j.str(key) || !j.lit(':')) return false;
    if (key == "dtype") {
      if (!j.str(out.dtype)) return false;
    } else if (key == "shape") {
      if (!j.lit('[')) return false;
      if (!j.lit(']')) {
        while (true) {
          int64_t v;
          if (!j.num(v)) return false;
          out.shape.push_back(v);
          if (j.lit(']')) break;
          if (!j.lit(',')) return false;
        }
      }
    } else if (key == "data_offsets") {
      if (!j.lit('[') || !j.num(out.begin) || !j.lit(',') || !j.num(out.end) || !j.lit(']'))
        return false;
    } else if (!j.skip()) {
      return false;
    }
    if (j.lit('}')) return true;
    if (!j.lit(',')) return false;
  }
}

bool parse_header(const char* p, size_t n, std::map<std::string, StEntry>& out) {
  JsonCursor j{p, p + n};
  if (!j.lit('{')) return false;
  if (j.lit('}')) return true;
  while (true) {
    std::string name;
    if (!j.str(name) || !j.lit(':')) return false;
    if (name == "__metadata__") {
      if (!j.skip()) return false;
    } else {
      StEntry en;
      if (!parse_entry(j, en)) return false;
      out[name] = en;
    }
    if (j.lit('}')) return true;
    if (!j.lit(',')) return false;
  }
}

}  // namespace

namespace pp {
// Message for pp_last_error(NULL, ...) from entry points that have no handle.
void set_global_error(const char* msg) { g_create_error = msg; }
}  // namespace pp

// =========================================================================== C ABI
extern "C" {

const char* pp_version(void) { return "potpori_b200 0.1 (sm_100a)"; }

size_t pp_last_error(const pp_shard* s, char* buf, size_t len) {
  const std::string& e = s ? s->err : g_create_error;
  if (buf && len) {
    size_t n = e.size() < len - 1 ? e.size() : len - 1;
    memcpy(buf, e.data(), n);
    buf[n] = 0;
  }
  return e.size();
}

void pp_shard_destroy(pp_shard* s) {
  if (!s) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(s->dev);
  if (s->stream) cudaStreamSynchronize(s->stream);
  for (auto& e : s->exec)
    if (e) cudaGraphExecDestroy(e);
  if (s->outbox) cudaIpcCloseMemHandle(s->outbox);
  if (s->pf_peer) cudaIpcCloseMemHandle(s->pf_peer);
  if (s->inbox) cudaFree(s->inbox);
  for (void* p : s->allocs) cudaFree(p);
  if (s->h_desc) cudaFreeHost(s->h_desc);
  if (s->h_res) cudaFreeHost(s->h_res);
  if (s->h_slots) cudaFreeHost(s->h_slots);
  for (int i = 0; i < kRing; ++i) {
    if (s->desc_ev[i]) cudaEventDestroy(s->desc_ev[i]);
    if (s->slot_ev[i]) cudaEventDestroy(s->slot_ev[i]);
  }
  if (s->handoff_ev) cudaEventDestroy(s->handoff_ev);
  if (s->handoff_done_ev) cudaEventDestroy(s->handoff_done_ev);
  if (s->h_stage) cudaFreeHost(s->h_stage);
  if (s->h_decode) cudaFreeHost(s->h_decode);
  if (s->stream) cudaStreamDestroy(s->stream);
  cudaSetDevice(prev);
  delete s;
}

static pp_status create_impl(const pp_shard_desc* desc, pp_shard* s) {
  const pp_config& c = desc->cfg;
  s->d = *desc;
  s->H = c.hidden;
  s->nh = c.n_heads;
  s->nkv = c.n_kv_heads;
  s->hd = c.head_dim;
  s->Q = c.n_heads * c.head_dim;
  s->KV = c.n_kv_heads * c.head_dim;
  s->I = c.intermediate;
  s->V = c.vocab_size;
  s->G = c.n_heads / c.n_kv_heads;
  s->first = desc->layer_begin == 0;
  s->last = desc->layer_end == c.layers;
  s->nl = desc->layer_end - desc->layer_begin;
  s->Hp = round_up(s->H, kChunkK);
  s->Qp = round_up(s->Q, kChunkK);
  s->Ip = round_up(s->I, kChunkK);
  s->Vp = round_up(s->V, kTileRows);
  s->qkv_rows = round_up(s->Q + 2 * s->KV, kTileRows);
  s->o_rows = round_up(s->H, kTileRows);
  s->gu_rows = round_up(s->I, kTileRows / 2) * 2;
  s->d_rows = round_up(s->H, kTileRows);
  s->dev = desc->cuda_device;
  CK(cudaSetDevice(s->dev));
  CK(cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, s->dev));
  CK(cudaDeviceGetAttribute(&s->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, s->dev));
  s->max_grid = s->num_sms;
  if (const char* e = getenv("PP_GEMV_STAGES")) {
    const int v = atoi(e);
    if (v >= 2 && v <= 12) s->gemv_max_stages = v;
  }
  if (const char* e = getenv("PP_ATTN_SPLITS_PER_SM")) {
    const int v = atoi(e);
    if (v >= 1 && v <= kAttnSplitsPerSm) s->attn_per_sm = v;
  }
  CK(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  pp_status r0 = set_attrs(s);
  if (r0) return r0;
  s->splits = s->attn_per_sm * s->num_sms / s->nkv > 0 ? s->attn_per_sm * s->num_sms / s->nkv : 1;
  if (s->splits > 256) s->splits = 256;  // the combine kernel holds up to 256 splits
  s->nq_max = s->G * kMaxRows;
  pp_status r;
  s->L.resize(s->nl);
  for (int l = 0; l < s->nl; ++l) {
    LayerDev& Ld = s->L[l];
    if ((r = dalloc(s, &Ld.wqkv, (size_t)s->qkv_rows * s->Hp * 2))) return r;
    if ((r = dalloc(s, &Ld.wo, (size_t)s->o_rows * s->Qp * 2))) return r;
    if ((r = dalloc(s, &Ld.wgu, (size_t)s->gu_rows * s->Hp * 2))) return r;
    if ((r = dalloc(s, &Ld.wd, (size_t)s->d_rows * s->Ip * 2))) return r;
    if ((r = dalloc(s, &Ld.norm[N_ATTN], (size_t)s->H * 4))) return r;
    if ((r = dalloc(s, &Ld.norm[N_QN], (size_t)s->hd * 4))) return r;
    if ((r = dalloc(s, &Ld.norm[N_KN], (size_t)s->hd * 4))) return r;
    if ((r = dalloc(s, &Ld.norm[N_FFN], (size_t)s->H * 4))) return r;
    if ((r = dalloc(s, &Ld.kc, (size_t)s->nkv * desc->capacity * kv_row_bytes(s->hd)))) return r;
    if ((r = dalloc(s, &Ld.vc, (size_t)s->nkv * desc->capacity * kv_row_bytes(s->hd)))) return r;
  }
  if (s->first || s->last) {
    if ((r = dalloc(s, &s->embed, (size_t)s->Vp * s->Hp * 2))) return r;
  }
  if (s->last && (r = dalloc(s, &s->final_norm, (size_t)s->H * 4))) return r;
  // RoPE table, src/qwen/model.rs:397-402 / tiny.rs:29-30: angle = pos * theta^(-2i/d).
  {
    const int half = s->hd / 2;
    std::vector<float2> tab((size_t)desc->capacity * half);
    for (uint32_t p = 0; p < desc->capacity; ++p)
      for (int i = 0; i < half; ++i) {
        const double ang = (double)p * pow((double)c.rope_theta, -2.0 * i / (double)s->hd);
        tab[(size_t)p * half + i] = make_float2((float)cos(ang), (float)sin(ang));
      }
    if ((r = dalloc(s, &s->rope, tab.size() * sizeof(float2)))) return r;
    CK(cudaMemcpyAsync(s->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice,
                       s->stream));
    CK(cudaStreamSynchronize(s->stream));
  }
  if ((r = dalloc(s, &s->x, (size_t)kMaxRows * s->Hp * 4))) return r;
  if ((r = dalloc(s, &s->qbuf, (size_t)kMaxRows * s->Q * 4))) return r;
  if ((r = dalloc(s, &s->attn_split, (size_t)(s->Qp / kChunkK) * SplitRows<16>::kBlock))) return r;
  if ((r = dalloc(s, &s->act_split, (size_t)(s->Ip / kChunkK) * SplitRows<16>::kBlock))) return r;
  s->ss_tiles = (int)(s->o_rows / kTileRows);
  if ((r = dalloc(s, &s->xw_attn, (size_t)(s->Hp / kChunkK) * SplitRows<16>::kBlock))) return r;
  if ((r = dalloc(s, &s->xw_ffn, (size_t)(s->Hp / kChunkK) * SplitRows<16>::kBlock))) return r;
  if ((r = dalloc(s, &s->ss_attn, (size_t)s->ss_tiles * kMaxRows * 4))) return r;
  if ((r = dalloc(s, &s->ss_ffn, (size_t)s->ss_tiles * kMaxRows * 4))) return r;
  if (s->last && (r = dalloc(s, &s->logits, (size_t)kMaxRows * s->V * 4))) return r;
  if ((r = dalloc(s, &s->apart, (size_t)s->nkv * s->splits * s->nq_max * (s->hd + 4) * 4))) return r;
  if ((r = dalloc(s, &s->gpart, (size_t)s->max_grid * 2 * kTileRows * kMaxRows * 4))) return r;
  {
    int64_t max_tiles = s->Vp / kTileRows;
    const int64_t cand[4] = {s->qkv_rows, s->o_rows, s->gu_rows, s->d_rows};
    for (int64_t v : cand) max_tiles = v / kTileRows > max_tiles ? v / kTileRows : max_tiles;
    if ((r = dalloc(s, &s->tile_cnt, (size_t)max_tiles * 4))) return r;
  }
  if ((r = dalloc(s, &s->recs, (size_t)s->max_grid * kMaxRows * sizeof(ArgRec)))) return r;
  if ((r = dalloc(s, &s->done, 64))) return r;
  if ((r = dalloc(s, &s->d_decode, (kDecodeMax + 1) * 4))) return r;
  CK(cudaMallocHost(&s->h_decode, (kDecodeMax + 1) * 4));
  if ((r = dalloc(s, &s->d_desc, sizeof(StepDesc)))) return r;
  if ((r = dalloc(s, &s->d_res, sizeof(StepResult)))) return r;
  CK(cudaMallocHost(&s->h_desc, sizeof(StepDesc) * kRing));
  CK(cudaMallocHost(&s->h_res, sizeof(StepResult)));
  CK(cudaMallocHost(&s->h_slots, sizeof(StepResult) * kRing));
  for (int i = 0; i < kRing; ++i) {
    CK(cudaEventCreateWithFlags(&s->desc_ev[i], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&s->slot_ev[i], cudaEventDisableTiming));
  }
  CK(cudaEventCreateWithFlags(&s->handoff_ev, cudaEventDisableTiming));
  CK(cudaEventCreateWithFlags(&s->handoff_done_ev, cudaEventDisableTiming));
  CK(cudaMallocHost(&s->h_stage, (size_t)kMaxRows * s->H * 4));
  memset(s->h_desc, 0, sizeof(StepDesc) * kRing);
  CK(cudaStreamSynchronize(s->stream));
  return PP_OK;
}

pp_status pp_shard_create(const pp_shard_desc* desc, pp_shard** out) {
  pp_shard* s = nullptr;
  if (!desc || !out) return fail(nullptr, PP_E_INVALID, "null argument");
  *out = nullptr;
  const pp_config& c = desc->cfg;
  // src/qwen/model.rs:206-217
  if (!(desc->layer_begin < desc->layer_end && desc->layer_end <= c.layers))
    return fail(nullptr, PP_E_INVALID, "invalid shard layer range");
  if (!(desc->capacity > 0 && desc->capacity <= 0x7fffffffu && desc->chunk <= desc->capacity))
    return fail(nullptr, PP_E_INVALID, "invalid cache/chunk capacity");
  if (c.n_kv_heads == 0 || c.n_heads % c.n_kv_heads || c.head_dim % 4 || c.head_dim > 128 ||
      c.hidden % 4 || c.intermediate % 4 ||
      128 % c.head_dim || c.hidden == 0 || c.intermediate == 0 || c.vocab_size == 0)
    return fail(nullptr, PP_E_UNSUPPORTED, "unsupported geometry");
  if (c.n_heads / c.n_kv_heads > 8)
    return fail(nullptr, PP_E_UNSUPPORTED, "more than 8 query heads per KV head");
  if (desc->chunk > (uint32_t)kMaxRows)
    return fail(nullptr, PP_E_UNSUPPORTED, "chunks above 16 rows are not built");
  if (desc->chunk > 8 && c.n_heads / c.n_kv_heads > 4)
    return fail(nullptr, PP_E_UNSUPPORTED, "16-row chunks need at most 4 query heads per KV head");
  if (!encode_fn()) return fail(nullptr, PP_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
  s = new pp_shard();
  int prev = 0;
  cudaGetDevice(&prev);
  pp_status r = create_impl(desc, s);
  if (r) {
    g_create_error = s->err;
    pp_shard_destroy(s);
    cudaSetDevice(prev);
    return r;
  }
  *out = s;
  return PP_OK;
}

int32_t pp_shard_missing(const pp_shard* s, char* buf, size_t len) {
  int n = 0;
  std::string names;
  auto miss = [&](const std::string& nm) {
    ++n;
    names += nm + ";";
  };
  if ((s->first || s->last) && !s->embed_set) miss("model.embed_tokens.weight");
  if (s->last && !s->final_norm_set) miss("model.norm.weight");
  for (int l = 0; l < s->nl; ++l) {
    const int gl = (int)s->d.layer_begin + l;
    for (int m = 0; m < M_COUNT; ++m)
      if (!s->L[l].mat_set[m]) miss("model.layers." + std::to_string(gl) + "." + kMatNames[m] + ".weight");
    for (int m = 0; m < N_COUNT; ++m)
      if (!s->L[l].norm_set[m]) miss("model.layers." + std::to_string(gl) + "." + kNormNames[m] + ".weight");
  }
  if (buf && len) {
    size_t k = names.size() < len - 1 ? names.size() : len - 1;
    memcpy(buf, names.data(), k);
    buf[k] = 0;
  }
  return n;
}

// Resolve a checkpoint name to this shard's destination.
struct Target {
  bool mine = false;
  bool is_norm = false;
  uint16_t* mat = nullptr;
  float* norm = nullptr;
  int64_t rows = 0, cols = 0, kchunks = 0;
  RowMap map{1, 0, 0};
  bool* flag = nullptr;
};

static pp_status resolve(pp_shard* s, const char* name, Target& t) {
  const int64_t H = s->H, Q = s->Q, KV = s->KV, I = s->I;
  if (!strcmp(name, "model.embed_tokens.weight")) {
    if (!(s->first || s->last)) return PP_OK;
    t = Target{true, false, s->embed, nullptr, s->V, H, s->Hp / kChunkK, RowMap{(int32_t)s->V, 0, 0}, &s->embed_set};
    return PP_OK;
  }
  if (!strcmp(name, "model.norm.weight")) {
    if (!s->last) return PP_OK;
    t = Target{true, true, nullptr, s->final_norm, 1, H, H, RowMap{1, 0, 0}, &s->final_norm_set};
    return PP_OK;
  }
  int layer = -1, off = 0;
  if (sscanf(name, "model.layers.%d.%n", &layer, &off) != 1 || off == 0)
    return fail(s, PP_E_INVALID, "unknown parameter %s", name);
  if (layer < (int)s->d.layer_begin || layer >= (int)s->d.layer_end) {
    if (layer < 0 || layer >= (int)s->d.cfg.layers)
      return fail(s, PP_E_INVALID, "unknown parameter %s", name);
    return PP_OK;
  }
  LayerDev& Ld = s->L[layer - s->d.layer_begin];
  const char* rest = name + off;
  for (int m = 0; m < M_COUNT; ++m) {
    std::string full = std::string(kMatNames[m]) + ".weight";
    if (full != rest) continue;
    t.mine = true;
    t.flag = &Ld.mat_set[m];
    switch (m) {
      case M_Q: t.mat = Ld.wqkv; t.rows = Q; t.cols = H; t.kchunks = s->Hp / kChunkK; t.map = RowMap{(int32_t)Q, 0, 0}; break;
      case M_K: t.mat = Ld.wqkv; t.rows = KV; t.cols = H; t.kchunks = s->Hp / kChunkK; t.map = RowMap{(int32_t)KV, 0, (int32_t)Q}; break;
      case M_V: t.mat = Ld.wqkv; t.rows = KV; t.cols = H; t.kchunks = s->Hp / kChunkK; t.map = RowMap{(int32_t)KV, 0, (int32_t)(Q + KV)}; break;
      case M_O: t.mat = Ld.wo; t.rows = H; t.cols = Q; t.kchunks = s->Qp / kChunkK; t.map = RowMap{(int32_t)H, 0, 0}; break;
      case M_G: t.mat = Ld.wgu; t.rows = I; t.cols = H; t.kchunks = s->Hp / kChunkK; t.map = RowMap{kTileRows / 2, kTileRows, 0}; break;
      case M_U: t.mat = Ld.wgu; t.rows = I; t.cols = H; t.kchunks = s->Hp / kChunkK; t.map = RowMap{kTileRows / 2, kTileRows, kTileRows / 2}; break;
      default: t.mat = Ld.wd; t.rows = H; t.cols = I; t.kchunks = s->Ip / kChunkK; t.map = RowMap{(int32_t)H, 0, 0}; break;
    }
    return PP_OK;
  }
  for (int m = 0; m < N_COUNT; ++m) {
    std::string full = std::string(kNormNames[m]) + ".weight";
    if (full != rest) continue;
    t.mine = true;
    t.is_norm = true;
    t.flag = &Ld.norm_set[m];
    t.norm = Ld.norm[m];
    t.rows = 1;
    t.cols = (m == N_QN || m == N_KN) ? s->hd : H;
    return PP_OK;
  }
  return fail(s, PP_E_INVALID, "unknown parameter %s", name);
}

pp_status pp_shard_set_tensor(pp_shard* s, const char* name, pp_dtype dtype, const void* data,
                              uint64_t elements) {
  if (!s || !name || !data) return fail(s, PP_E_INVALID, "null argument");
  CK(cudaSetDevice(s->dev));
  Target t;
  pp_status r = resolve(s, name, t);
  if (r || !t.mine) return r;
  if ((int64_t)elements != t.rows * t.cols)
    return fail(s, PP_E_INVALID, "shape mismatch for %s: %llu elements, want %lld", name,
                (unsigned long long)elements, (long long)(t.rows * t.cols));
  if (t.is_norm) {
    std::vector<float> v(elements);
    for (uint64_t i = 0; i < elements; ++i)
      v[i] = dtype == PP_F32 ? ((const float*)data)[i]
                             : bits_to_float((uint32_t)((const uint16_t*)data)[i] << 16);
    CK(cudaMemcpyAsync(t.norm, v.data(), elements * 4, cudaMemcpyHostToDevice, s->stream));
    CK(cudaStreamSynchronize(s->stream));
  } else {
    const size_t eb = dtype == PP_F32 ? 4 : 2;
    void* tmp = nullptr;
    CK(cudaMalloc(&tmp, elements * eb));
    cudaError_t e = cudaMemcpyAsync(tmp, data, elements * eb, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) {
      pp_pack_matrix_kernel<<<1024, 256, 0, s->stream>>>(t.mat, tmp, dtype == PP_F32, t.rows, t.cols,
                                                      t.kchunks, t.map);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail(s, PP_E_CUDA, "upload %s: %s", name, cudaGetErrorString(e));
  }
  *t.flag = true;
  s->dec_stale = true;
  return PP_OK;
}

pp_status pp_shard_init_random(pp_shard* s, uint64_t seed, float stdv) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  CK(cudaSetDevice(s->dev));
  std::vector<std::string> names;
  if (s->first || s->last) names.push_back("model.embed_tokens.weight");
  if (s->last) names.push_back("model.norm.weight");
  for (int l = 0; l < s->nl; ++l) {
    const std::string pre = "model.layers." + std::to_string(s->d.layer_begin + l) + ".";
    for (int m = 0; m < M_COUNT; ++m) names.push_back(pre + kMatNames[m] + ".weight");
    for (int m = 0; m < N_COUNT; ++m) names.push_back(pre + kNormNames[m] + ".weight");
  }
  const float scale = stdv * (1.0f / 65536.0f);
  for (const std::string& nm : names) {
    Target t;
    pp_status r = resolve(s, nm.c_str(), t);
    if (r) return r;
    if (t.is_norm) {
      pp_fill_f32_kernel<<<64, 256, 0, s->stream>>>(t.norm, t.cols, 1.0f);
    } else {
      pp_gen_matrix_kernel<<<2048, 256, 0, s->stream>>>(t.mat, t.rows, t.cols, t.kchunks, t.map,
                                                     tensor_key(seed, nm.c_str()), scale);
    }
    CK(cudaGetLastError());
    *t.flag = true;
  }
  s->dec_stale = true;
  CK(cudaStreamSynchronize(s->stream));
  return PP_OK;
}

pp_status pp_shard_load_safetensors(pp_shard* s, const char* path) {
  if (!s || !path) return fail(s, PP_E_INVALID, "null argument");
  int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(s, PP_E_INVALID, "cannot open %s", path);
  struct stat sb;
  fstat(fd, &sb);
  const size_t size = (size_t)sb.st_size;
  void* mp = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  close(fd);
  if (mp == MAP_FAILED) return fail(s, PP_E_INVALID, "cannot map %s", path);
  const uint8_t* base = (const uint8_t*)mp;
  pp_status r = PP_OK;
  uint64_t hlen = 0;
  std::map<std::string, StEntry> ents;
  if (size < 8) {
    r = fail(s, PP_E_INVALID, "%s: not a safetensors file", path);
  } else {
    memcpy(&hlen, base, 8);
    if (hlen > size - 8 || !parse_header((const char*)base + 8, hlen, ents))
      r = fail(s, PP_E_INVALID, "%s: bad safetensors header", path);
  }
  const uint8_t* data = base + 8 + hlen;
  const size_t dsize = size - 8 - (size_t)hlen;
  for (auto it = ents.begin(); r == PP_OK && it != ents.end(); ++it) {
    const std::string& nm = it->first;
    const StEntry& en = it->second;
    Target t;
    if ((r = resolve(s, nm.c_str(), t))) {
      if (nm.rfind("model.", 0) != 0) {  // not a model parameter (e.g. lm_head): ignore
        r = PP_OK;
        s->err.clear();
      }
      continue;
    }
    if (!t.mine) continue;
    // src/qwen/hf.rs:235: the stored shape must be the parameter's ([rows, cols], or [n] for a
    // norm), not only its element count.
    const std::vector<int64_t> want =
        t.is_norm ? std::vector<int64_t>{t.cols} : std::vector<int64_t>{t.rows, t.cols};
    if (en.shape != want) {
      r = fail(s, PP_E_INVALID, "shape mismatch for %s", nm.c_str());
      break;
    }
    int64_t n = 1;
    for (int64_t v : en.shape) n *= v;
    if (en.begin < 0 || en.end < en.begin || (size_t)en.end > dsize) {
      r = fail(s, PP_E_INVALID, "%s: bad data offsets", nm.c_str());
      break;
    }
    const uint8_t* src = data + en.begin;
    if (en.dtype == "BF16" && (en.end - en.begin) == n * 2) {
      r = pp_shard_set_tensor(s, nm.c_str(), PP_BF16, src, (uint64_t)n);
    } else if (en.dtype == "F32" && (en.end - en.begin) == n * 4) {
      r = pp_shard_set_tensor(s, nm.c_str(), PP_F32, src, (uint64_t)n);
    } else if (en.dtype == "F16" && (en.end - en.begin) == n * 2) {
      std::vector<float> f((size_t)n);
      for (int64_t i = 0; i < n; ++i) {
        uint16_t hbits;
        memcpy(&hbits, src + 2 * i, 2);
        const uint32_t sign = (uint32_t)(hbits >> 15) << 31, ex = (hbits >> 10) & 31, man = hbits & 1023;
        float v;
        if (ex == 0) v = ldexpf((float)man, -24);
        else if (ex == 31) v = man ? NAN : INFINITY;
        else v = ldexpf((float)(man | 1024), (int)ex - 25);
        uint32_t u;
        memcpy(&u, &v, 4);
        u |= sign;
        memcpy(&f[i], &u, 4);
      }
      r = pp_shard_set_tensor(s, nm.c_str(), PP_F32, f.data(), (uint64_t)n);
    } else {
      r = fail(s, PP_E_INVALID, "%s: unsupported dtype %s", nm.c_str(), en.dtype.c_str());
    }
  }
  munmap(mp, size);
  return r;
}

pp_status pp_shard_forward_tokens(pp_shard* s, uint32_t pos, const int32_t* tokens, uint32_t m,
                                  float* out_hidden, pp_verify_out* verify) {
  if (!s || !tokens) return fail(s, PP_E_INVALID, "null argument");
  if (!s->first) return fail(s, PP_E_INVALID, "invalid token input");
  pp_status r = check_step(s, pos, m);
  if (r) return r;
  for (uint32_t i = 0; i < m; ++i)  // src/qwen/model.rs:383-389
    if (tokens[i] < 0 || (uint32_t)tokens[i] >= (uint32_t)s->V)
      return fail(s, PP_E_INVALID, "invalid token input");
  CK(cudaSetDevice(s->dev));
  int slot;
  StepDesc& d = *next_desc(s, &slot);
  d.pos = (int32_t)pos;
  d.m = (int32_t)m;
  d.n_drafts = (int32_t)m - 1;
  d.flags = (verify && verify->logits) ? 1 : 0;
  for (uint32_t i = 0; i < m; ++i) d.tokens[i] = tokens[i];
  for (uint32_t i = 1; i < m; ++i) d.drafts[i - 1] = tokens[i];
  if ((r = upload_desc(s, slot, s->stream))) return r;
  return finish_host_step(s, m, out_hidden, verify);
}

static pp_status write_word(pp_shard* s, uint32_t* host_word, uint32_t value);

static pp_status prefill_check(pp_shard* s, uint32_t pos, uint32_t t) {
  if (s->hd != kFlashHd || (s->G != 1 && s->G != 2 && s->G != 4 && s->G != 8))
    return fail(s, PP_E_UNSUPPORTED, "the prompt prefill takes head size 128 and 1, 2, 4 or 8 query heads per KV head");
  if (t == 0 || t > (uint32_t)kPrefillMax) return fail(s, PP_E_INVALID, "t must be 1..2048 rows");
  if ((uint64_t)pos + t > s->d.capacity) return fail(s, PP_E_INVALID, "chunk exceeds KV capacity");
  if (pp_shard_missing(s, nullptr, 0))
    return fail(s, PP_E_MISSING, "parameters missing; see pp_shard_missing");
  return PP_OK;
}

// The prefill pass over the rows staged for it; synchronous.
static pp_status prefill_run(pp_shard* s, uint32_t pos, uint32_t t) {
  pp_status r;
  if ((r = enqueue_prefill(s, pos, (int)t))) {
    cudaStreamSynchronize(s->stream);
    return r;
  }
  uint32_t err = 0;
  CK(cudaMemcpyAsync(&err, s->pf.err, 4, cudaMemcpyDeviceToHost, s->stream));
  CK(cudaMemcpyAsync(s->h_res, s->d_res, sizeof(StepResult), cudaMemcpyDeviceToHost, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  if (err) return fail(s, PP_E_TIMEOUT, "a bounded wait of the prompt projection expired");
  return status_of(s, *s->h_res);
}

pp_status pp_shard_prefill(pp_shard* s, uint32_t pos, const int32_t* tokens, uint32_t t) {
  if (!s || !tokens) return fail(s, PP_E_INVALID, "null argument");
  if (!s->first) return fail(s, PP_E_INVALID, "token input on a shard that is not the first");
  pp_status r = prefill_check(s, pos, t);
  if (r) return r;
  for (uint32_t i = 0; i < t; ++i)  // src/qwen/model.rs:383-389
    if (tokens[i] < 0 || (uint32_t)tokens[i] >= (uint32_t)s->V)
      return fail(s, PP_E_INVALID, "invalid token input");
  CK(cudaSetDevice(s->dev));
  if ((r = prefill_alloc(s))) return r;
  CK(cudaMemcpyAsync(s->pf.tokens, tokens, (size_t)t * 4, cudaMemcpyHostToDevice, s->stream));
  return prefill_run(s, pos, t);
}

pp_status pp_shard_prefill_hidden(pp_shard* s, uint32_t pos, uint32_t t, const float* hidden) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  if (s->first) return fail(s, PP_E_INVALID, "hidden input on the first shard");
  pp_status r = prefill_check(s, pos, t);
  if (r) return r;
  CK(cudaSetDevice(s->dev));
  if ((r = prefill_alloc(s))) return r;
  if (hidden) {
    for (size_t i = 0; i < (size_t)t * s->H; ++i)  // src/qwen/model.rs:390-392
      if (!std::isfinite(hidden[i])) return fail(s, PP_E_INVALID, "invalid hidden input");
    CK(cudaMemcpyAsync(s->pf.x, hidden, (size_t)t * s->H * 4, cudaMemcpyHostToDevice, s->stream));
  }
  return prefill_run(s, pos, t);
}

pp_status pp_shard_prefill_read(pp_shard* s, uint32_t t, float* out) {
  if (!s || !out) return fail(s, PP_E_INVALID, "null argument");
  if (s->last) return fail(s, PP_E_INVALID, "the last shard leaves no output rows");
  if (!s->pf.x || t == 0 || t > (uint32_t)kPrefillMax) return fail(s, PP_E_INVALID, "no rows");
  CK(cudaSetDevice(s->dev));
  CK(cudaMemcpyAsync(out, s->pf.x, (size_t)t * s->H * 4, cudaMemcpyDeviceToHost, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  return PP_OK;
}

pp_status pp_shard_prefill_handoff(pp_shard* from, pp_shard* to, uint32_t t) {
  pp_shard* s = to;
  if (!from || !to) return fail(to, PP_E_INVALID, "null shard");
  if (from->last || to->first || from->H != to->H || from->d.layer_end != to->d.layer_begin)
    return fail(to, PP_E_INVALID, "shards are not adjacent stages");
  if (!from->pf.x || t == 0 || t > (uint32_t)kPrefillMax)
    return fail(to, PP_E_INVALID, "no prefill rows to hand off");
  CK(cudaSetDevice(to->dev));
  pp_status r = prefill_alloc(to);
  if (r) return r;
  CK(cudaStreamSynchronize(from->stream));
  const size_t bytes = (size_t)t * to->H * 4;
  if (from->dev == to->dev)
    CK(cudaMemcpyAsync(to->pf.x, from->pf.x, bytes, cudaMemcpyDeviceToDevice, to->stream));
  else
    CK(cudaMemcpyPeerAsync(to->pf.x, to->dev, from->pf.x, from->dev, bytes, to->stream));
  return PP_OK;
}

pp_status pp_shard_prefill_export(pp_shard* s, void* handle) {
  if (!s || !handle) return fail(s, PP_E_INVALID, "null argument");
  if (s->first) return fail(s, PP_E_INVALID, "the first stage takes tokens");
  CK(cudaSetDevice(s->dev));
  pp_status r = prefill_alloc(s);
  if (r) return r;
  CK(cudaStreamSynchronize(s->stream));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, s->pf.x));
  memcpy(handle, &h, sizeof h);
  return PP_OK;
}

pp_status pp_shard_prefill_open(pp_shard* s, const void* handle) {
  if (!s || !handle) return fail(s, PP_E_INVALID, "null argument");
  if (s->last) return fail(s, PP_E_INVALID, "the last stage has no next stage");
  if (s->pf_peer) return fail(s, PP_E_INVALID, "already open");
  CK(cudaSetDevice(s->dev));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void* p = nullptr;
  CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  s->pf_peer = (float*)p;
  return PP_OK;
}

pp_status pp_shard_prefill_send(pp_shard* s, uint32_t seq, uint32_t t, uint32_t* mail,
                                uint32_t info) {
  if (!s || !mail) return fail(s, PP_E_INVALID, "null argument");
  if (!s->pf_peer || !s->pf.x) return fail(s, PP_E_INVALID, "no prefill link: pp_shard_prefill_open first");
  if (t == 0 || t > (uint32_t)kPrefillMax) return fail(s, PP_E_INVALID, "t must be 1..2048 rows");
  CK(cudaSetDevice(s->dev));
  CK(cudaMemcpyAsync(s->pf_peer, s->pf.x, (size_t)t * s->H * 4, cudaMemcpyDeviceToDevice, s->stream));
  pp_status r;
  if ((r = write_word(s, mail + 1, info))) return r;
  return write_word(s, mail, seq + 1);
}

pp_status pp_shard_decode_greedy(pp_shard* s, uint32_t pos, int32_t token, uint32_t n,
                                 int32_t* out) {
  if (!s || !out) return fail(s, PP_E_INVALID, "null argument");
  if (!s->first || !s->last) return fail(s, PP_E_INVALID, "greedy decode needs the whole model");
  if (n == 0 || n > (uint32_t)kDecodeMax) return fail(s, PP_E_INVALID, "n must be 1..%d", kDecodeMax);
  if ((uint64_t)pos + n > s->d.capacity) return fail(s, PP_E_INVALID, "chunk exceeds KV capacity");
  if (token < 0 || token >= s->V) return fail(s, PP_E_INVALID, "invalid token input");
  if (pp_shard_missing(s, nullptr, 0))
    return fail(s, PP_E_MISSING, "parameters missing; see pp_shard_missing");
  CK(cudaSetDevice(s->dev));
  int slot;
  StepDesc& d = *next_desc(s, &slot);
  d.pos = (int32_t)pos;
  d.m = 1;
  d.n_drafts = 0;
  d.flags = 0;
  d.tokens[0] = token;
  pp_status r;
  if ((r = upload_desc(s, slot, s->stream))) return r;
  CK(cudaMemsetAsync(s->d_decode + kDecodeMax, 0, 4, s->stream));
  for (uint32_t i = 0; i < n; ++i) {
    if ((r = run_step(s, 0, s->stream))) return r;
    pp_decode_feed_kernel<<<1, 1, 0, s->stream>>>(s->d_desc, s->d_res, s->d_decode, (int32_t)i,
                                                i + 1 < n ? 1 : 0);
    CK(cudaGetLastError());
  }
  CK(cudaMemcpyAsync(s->h_decode, s->d_decode, (kDecodeMax + 1) * 4, cudaMemcpyDeviceToHost,
                     s->stream));
  CK(cudaStreamSynchronize(s->stream));
  for (uint32_t i = 0; i < n; ++i) out[i] = s->h_decode[i];
  StepResult st = {};
  st.status = s->h_decode[kDecodeMax];
  return status_of(s, st);
}

pp_status pp_shard_forward_hidden(pp_shard* s, uint32_t pos, uint32_t m, const float* hidden,
                                  const int32_t* drafts, uint32_t n_drafts, float* out_hidden,
                                  pp_verify_out* verify) {
  if (!s || !hidden) return fail(s, PP_E_INVALID, "null argument");
  if (s->first) return fail(s, PP_E_INVALID, "invalid hidden input");
  pp_status r = check_step(s, pos, m);
  if (r) return r;
  if (n_drafts > (uint32_t)kMaxRows || (n_drafts && !drafts))
    return fail(s, PP_E_INVALID, "invalid drafts");
  for (size_t i = 0; i < (size_t)m * s->H; ++i)  // src/qwen/model.rs:390-392
    if (!std::isfinite(hidden[i])) return fail(s, PP_E_INVALID, "invalid hidden input");
  CK(cudaSetDevice(s->dev));
  int slot;
  StepDesc& d = *next_desc(s, &slot);
  d.pos = (int32_t)pos;
  d.m = (int32_t)m;
  d.n_drafts = (int32_t)n_drafts;
  d.flags = (verify && verify->logits) ? 1 : 0;
  for (uint32_t i = 0; i < n_drafts; ++i) d.drafts[i] = drafts[i];
  memcpy(s->h_stage, hidden, (size_t)m * s->H * 4);
  if ((r = upload_desc(s, slot, s->stream))) return r;
  CK(cudaMemcpy2DAsync(s->x, (size_t)s->Hp * 4, s->h_stage, (size_t)s->H * 4, (size_t)s->H * 4, m,
                       cudaMemcpyHostToDevice, s->stream));
  return finish_host_step(s, m, out_hidden, verify);
}

pp_status pp_shard_set_step(pp_shard* s, uint32_t pos, uint32_t m, const int32_t* tokens,
                            const int32_t* drafts, uint32_t n_drafts, int32_t flags,
                            void* stream) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  pp_status r = check_step(s, pos, m);
  if (r) return r;
  if (n_drafts > (uint32_t)kMaxRows || (n_drafts && !drafts) || (s->first && !tokens))
    return fail(s, PP_E_INVALID, "invalid step");
  if (s->first)
    for (uint32_t i = 0; i < m; ++i)
      if (tokens[i] < 0 || (uint32_t)tokens[i] >= (uint32_t)s->V)
        return fail(s, PP_E_INVALID, "invalid token input");
  CK(cudaSetDevice(s->dev));
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  int slot;
  StepDesc& d = *next_desc(s, &slot);
  d.pos = (int32_t)pos;
  d.m = (int32_t)m;
  d.n_drafts = (int32_t)n_drafts;
  d.flags = flags;
  for (uint32_t i = 0; i < m && tokens; ++i) d.tokens[i] = tokens[i];
  for (uint32_t i = 0; i < n_drafts; ++i) d.drafts[i] = drafts[i];
  return upload_desc(s, slot, st);
}

pp_status pp_shard_step_device(pp_shard* s, uint32_t max_rows, void* stream) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  if (max_rows == 0 || max_rows > (uint32_t)kMaxRows) return fail(s, PP_E_UNSUPPORTED, "max_rows must be 1..16");
  if (max_rows > 8 && s->G > 4)
    return fail(s, PP_E_UNSUPPORTED, "16-row chunks need at most 4 query heads per KV head");
  CK(cudaSetDevice(s->dev));
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  return run_step(s, variant_of((int)max_rows), st);
}

pp_status pp_shard_buffers(pp_shard* s, void** hidden, void** header, void** result) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  if (hidden) *hidden = s->x;
  if (header) *header = s->d_desc;
  if (result) *result = s->d_res;
  return PP_OK;
}

pp_status pp_shard_read_result(pp_shard* s, uint32_t m, pp_verify_out* verify, void* stream) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  CK(cudaSetDevice(s->dev));
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  CK(cudaMemcpyAsync(s->h_res, s->d_res, sizeof(StepResult), cudaMemcpyDeviceToHost, st));
  if (s->last && verify && verify->logits)
    CK(cudaMemcpyAsync(verify->logits, s->logits, (size_t)m * s->V * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (verify) fill_verify(s, m, verify);
  return status_of(s, *s->h_res);
}

pp_status pp_shard_reset(pp_shard* s) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  CK(cudaSetDevice(s->dev));
  for (auto& Ld : s->L) {
    CK(cudaMemsetAsync(Ld.kc, 0, (size_t)s->nkv * s->d.capacity * kv_row_bytes(s->hd), s->stream));
    CK(cudaMemsetAsync(Ld.vc, 0, (size_t)s->nkv * s->d.capacity * kv_row_bytes(s->hd), s->stream));
  }
  CK(cudaStreamSynchronize(s->stream));
  return PP_OK;
}

pp_status pp_shard_fill_kv(pp_shard* s, uint64_t seed, uint32_t rows) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  if (rows > s->d.capacity) return fail(s, PP_E_INVALID, "rows exceed capacity");
  CK(cudaSetDevice(s->dev));
  for (int l = 0; l < s->nl; ++l) {
    const uint64_t key = mix64h(seed * 0x9E3779B97F4A7C15ull ^ (uint64_t)(l + 1));
    pp_fill_kv_kernel<<<1024, 256, 0, s->stream>>>(s->L[l].kc, s->L[l].vc, rows, s->KV, s->nkv, s->hd,
                                                s->d.capacity, key);
    CK(cudaGetLastError());
  }
  CK(cudaStreamSynchronize(s->stream));
  return PP_OK;
}

pp_status pp_shard_profile_kernels(pp_shard* s, uint32_t max_rows, uint32_t iters, float* ms,
                                   int32_t* kinds, uint32_t cap, uint32_t* count) {
  if (!s || !ms || !kinds || !count || iters == 0) return fail(s, PP_E_INVALID, "null argument");
  if (max_rows == 0 || max_rows > (uint32_t)kMaxRows) return fail(s, PP_E_UNSUPPORTED, "max_rows must be 1..16");
  if (max_rows > 8 && s->G > 4)
    return fail(s, PP_E_UNSUPPORTED, "16-row chunks need at most 4 query heads per KV head");
  if (pp_shard_missing(s, nullptr, 0)) return fail(s, PP_E_MISSING, "parameters missing");
  CK(cudaSetDevice(s->dev));
  // Capture the step with an event record after every kernel, then replay the graph: the
  // per-kernel times carry no host launch overhead (the events do serialise the kernels).
  std::vector<cudaEvent_t> ev;
  std::vector<int> kd;
  cudaEvent_t start;
  CK(cudaEventCreate(&start));
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ge = nullptr;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = cudaEventRecordWithFlags(start, s->stream, cudaEventRecordExternal);
  s->prof_events = &ev;
  s->prof_kinds = &kd;
  pp_status r = e == cudaSuccess ? enqueue_variant(s, variant_of((int)max_rows), s->stream)
                                 : fail(s, PP_E_CUDA, "profile: %s", cudaGetErrorString(e));
  s->prof_events = nullptr;
  s->prof_kinds = nullptr;
  e = cudaStreamEndCapture(s->stream, &g);
  if (r == PP_OK && e != cudaSuccess) r = fail(s, PP_E_CUDA, "profile capture: %s", cudaGetErrorString(e));
  if (r == PP_OK) {
    e = cudaGraphInstantiate(&ge, g, 0);
    if (e != cudaSuccess) r = fail(s, PP_E_CUDA, "profile instantiate: %s", cudaGetErrorString(e));
  }
  std::vector<double> acc(ev.size(), 0.0);
  for (uint32_t it = 0; r == PP_OK && it <= iters; ++it) {
    e = cudaGraphLaunch(ge, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) {
      r = fail(s, PP_E_CUDA, "profile: %s", cudaGetErrorString(e));
      break;
    }
    if (it == 0) continue;  // warm-up replay
    cudaEvent_t prev = start;
    for (size_t k = 0; k < ev.size(); ++k) {
      float t = 0.f;
      cudaEventElapsedTime(&t, prev, ev[k]);
      acc[k] += t;
      prev = ev[k];
    }
  }
  if (ge) cudaGraphExecDestroy(ge);
  if (g) cudaGraphDestroy(g);
  cudaEventDestroy(start);
  for (cudaEvent_t x : ev) cudaEventDestroy(x);
  if (r) return r;
  *count = (uint32_t)acc.size();
  for (size_t k = 0; k < acc.size() && k < cap; ++k) {
    ms[k] = (float)(acc[k] / iters);
    kinds[k] = kd[k];
  }
  return PP_OK;
}

void* pp_shard_stream(const pp_shard* s) { return s ? (void*)s->stream : nullptr; }

pp_status pp_shard_handoff(pp_shard* from, pp_shard* to, uint32_t m) {
  pp_shard* s = to;
  if (!from || !to) return fail(to, PP_E_INVALID, "null shard");
  if (from->last || to->first || from->H != to->H || from->d.layer_end != to->d.layer_begin)
    return fail(to, PP_E_INVALID, "shards are not adjacent stages");
  if (m == 0 || m > (uint32_t)kMaxRows) return fail(to, PP_E_INVALID, "bad row count");
  CK(cudaSetDevice(from->dev));
  CK(cudaEventRecord(from->handoff_ev, from->stream));
  CK(cudaSetDevice(to->dev));
  CK(cudaStreamWaitEvent(to->stream, from->handoff_ev, 0));
  const size_t bytes = (size_t)m * to->Hp * 4;
  if (from->dev == to->dev)
    CK(cudaMemcpyAsync(to->x, from->x, bytes, cudaMemcpyDeviceToDevice, to->stream));
  else
    CK(cudaMemcpyPeerAsync(to->x, to->dev, from->x, from->dev, bytes, to->stream));
  // `from` may not overwrite its output rows before they have been copied out.
  CK(cudaEventRecord(to->handoff_done_ev, to->stream));
  CK(cudaSetDevice(from->dev));
  CK(cudaStreamWaitEvent(from->stream, to->handoff_done_ev, 0));
  return PP_OK;
}

pp_status pp_shard_inbox_export(pp_shard* s, uint32_t slots, void* handle) {
  if (!s || !handle) return fail(s, PP_E_INVALID, "null argument");
  if (slots == 0 || slots > 4096) return fail(s, PP_E_INVALID, "slots must be 1..4096");
  if (s->first) return fail(s, PP_E_INVALID, "the first stage has no inbox");
  CK(cudaSetDevice(s->dev));
  if (s->inbox && s->inbox_slots != slots) return fail(s, PP_E_INVALID, "inbox already exported");
  if (!s->inbox) {
    // Its own allocation: an IPC handle names the start of one.
    CK(cudaMalloc(&s->inbox, slots * inbox_slot_bytes(s->Hp)));
    s->inbox_slots = slots;
    s->bytes += slots * inbox_slot_bytes(s->Hp);
  }
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, s->inbox));
  memcpy(handle, &h, sizeof h);
  return PP_OK;
}

pp_status pp_shard_outbox_open(pp_shard* s, const void* handle, uint32_t slots) {
  if (!s || !handle) return fail(s, PP_E_INVALID, "null argument");
  if (s->last) return fail(s, PP_E_INVALID, "the last stage sends results, not hidden rows");
  if (slots == 0 || slots > 4096) return fail(s, PP_E_INVALID, "slots must be 1..4096");
  if (s->outbox) return fail(s, PP_E_INVALID, "outbox already open");
  CK(cudaSetDevice(s->dev));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void* p = nullptr;
  CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  s->outbox = (uint8_t*)p;
  s->outbox_slots = slots;
  return PP_OK;
}

// The stream-ordered write of `value` into a word of registered host memory.
static pp_status write_word(pp_shard* s, uint32_t* host_word, uint32_t value) {
  StreamWriteValue32Fn fn = write_value_fn();
  if (!fn) return fail(s, PP_E_CUDA, "cuStreamWriteValue32 is not available");
  void* dp = nullptr;
  CK(cudaHostGetDevicePointer(&dp, host_word, 0));
  if (fn((CUstream)s->stream, (CUdeviceptr)dp, value, 0) != CUDA_SUCCESS)
    return fail(s, PP_E_CUDA, "cuStreamWriteValue32 failed");
  return PP_OK;
}

pp_status pp_shard_send(pp_shard* s, uint32_t seq, uint32_t m, uint32_t* mail, uint32_t info) {
  if (!s || !mail) return fail(s, PP_E_INVALID, "null argument");
  if (!s->outbox) return fail(s, PP_E_INVALID, "no outbox: pp_shard_outbox_open first");
  if (m > (uint32_t)kMaxRows) return fail(s, PP_E_INVALID, "bad row count");
  CK(cudaSetDevice(s->dev));
  uint8_t* slot = s->outbox + (size_t)(seq % s->outbox_slots) * inbox_slot_bytes(s->Hp);
  if (m) {
    // Header and hidden rows over NVLink on the copy engines, ordered after the step.
    CK(cudaMemcpyAsync(slot, s->d_desc, sizeof(StepDesc), cudaMemcpyDeviceToDevice, s->stream));
    CK(cudaMemcpyAsync(slot + 256, s->x, (size_t)m * s->Hp * 4, cudaMemcpyDeviceToDevice, s->stream));
  }
  pp_status r;
  if ((r = write_word(s, mail + 1, info))) return r;
  return write_word(s, mail, seq + 1);
}

pp_status pp_shard_recv(pp_shard* s, uint32_t seq, uint32_t m) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  if (!s->inbox) return fail(s, PP_E_INVALID, "no inbox: pp_shard_inbox_export first");
  if (m == 0 || m > (uint32_t)kMaxRows) return fail(s, PP_E_INVALID, "bad row count");
  CK(cudaSetDevice(s->dev));
  const uint8_t* slot = s->inbox + (size_t)(seq % s->inbox_slots) * inbox_slot_bytes(s->Hp);
  CK(cudaMemcpyAsync(s->d_desc, slot, sizeof(StepDesc), cudaMemcpyDeviceToDevice, s->stream));
  CK(cudaMemcpyAsync(s->x, slot + 256, (size_t)m * s->Hp * 4, cudaMemcpyDeviceToDevice, s->stream));
  return PP_OK;
}

pp_status pp_shard_send_result(pp_shard* s, void* host_result, uint32_t* mail, uint32_t value) {
  if (!s || !host_result || !mail) return fail(s, PP_E_INVALID, "null argument");
  if (!s->last) return fail(s, PP_E_INVALID, "only the last stage has results");
  CK(cudaSetDevice(s->dev));
  CK(cudaMemcpyAsync(host_result, s->d_res, sizeof(StepResult), cudaMemcpyDeviceToHost, s->stream));
  return write_word(s, mail, value);
}

pp_status pp_host_register(void* p, size_t bytes) {
  if (!p || !bytes) {
    pp::set_global_error("null argument");
    return PP_E_INVALID;
  }
  cudaError_t e = cudaHostRegister(p, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    pp::set_global_error(cudaGetErrorString(e));
    return PP_E_CUDA;
  }
  return PP_OK;
}

pp_status pp_host_unregister(void* p) {
  if (cudaHostUnregister(p) != cudaSuccess) {
    pp::set_global_error("cudaHostUnregister failed");
    return PP_E_CUDA;
  }
  return PP_OK;
}

pp_status pp_shard_result_enqueue(pp_shard* s, uint32_t slot) {
  if (!s || slot >= (uint32_t)kRing) return fail(s, PP_E_INVALID, "bad result slot");
  CK(cudaSetDevice(s->dev));
  CK(cudaMemcpyAsync(&s->h_slots[slot], s->d_res, sizeof(StepResult), cudaMemcpyDeviceToHost,
                     s->stream));
  CK(cudaEventRecord(s->slot_ev[slot], s->stream));
  return PP_OK;
}

pp_status pp_shard_result_wait(pp_shard* s, uint32_t slot, uint32_t m, pp_verify_out* verify) {
  if (!s || slot >= (uint32_t)kRing || m == 0 || m > (uint32_t)kMaxRows)
    return fail(s, PP_E_INVALID, "bad result slot");
  CK(cudaSetDevice(s->dev));
  CK(cudaEventSynchronize(s->slot_ev[slot]));
  const StepResult& r = s->h_slots[slot];
  if (verify) {
    for (uint32_t i = 0; i < m; ++i) {
      if (verify->argmax) verify->argmax[i] = r.argmax[i];
      if (verify->top1) verify->top1[i] = r.top1[i];
      if (verify->top2) verify->top2[i] = r.top2[i];
    }
    verify->n_accepted = r.n_accepted;
    verify->correction = r.correction;
    verify->nonfinite_rows = r.nonfinite_rows;
  }
  return status_of(s, r);
}

uint32_t pp_shard_capacity(const pp_shard* s) { return s->d.capacity; }
uint32_t pp_shard_chunk_size(const pp_shard* s) { return s->d.chunk; }
void pp_shard_range(const pp_shard* s, uint32_t* b, uint32_t* e) {
  if (b) *b = s->d.layer_begin;
  if (e) *e = s->d.layer_end;
}
uint32_t pp_shard_hidden_dim(const pp_shard* s) { return (uint32_t)s->H; }
uint32_t pp_shard_vocab_size(const pp_shard* s) { return (uint32_t)s->V; }
uint32_t pp_shard_model_layers(const pp_shard* s) { return s->d.cfg.layers; }
uint64_t pp_shard_device_bytes(const pp_shard* s) { return s->bytes; }
uint32_t pp_shard_last_launches(const pp_shard* s) { return s->variant_launches[s->last_variant]; }

pp_status pp_shard_set_graphs(pp_shard* s, int32_t enabled) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  s->use_graphs = enabled != 0;
  return PP_OK;
}
pp_status pp_shard_set_sm_limit(pp_shard* s, uint32_t ctas) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  const int n = ctas == 0 || (int)ctas > s->num_sms ? s->num_sms : (int)ctas;
  if (n < s->nkv) return fail(s, PP_E_INVALID, "an SM limit below n_kv_heads (%d)", s->nkv);
  s->max_grid = n;
  s->splits = s->attn_per_sm * n / s->nkv > 256 ? 256 : s->attn_per_sm * n / s->nkv;  // buffers were sized for the whole GPU
  drop_graphs(s);
  return PP_OK;
}
uint32_t pp_shard_sm_limit(const pp_shard* s) { return s ? (uint32_t)s->max_grid : 0u; }

pp_status pp_shard_set_decode_kernel(pp_shard* s, int32_t enabled) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  CK(cudaSetDevice(s->dev));
  if (enabled && !s->dec_on) {
    if (!(s->first && s->last))
      return fail(s, PP_E_UNSUPPORTED, "the decode kernel runs shards that hold every layer");
    // A gate/up pair of rows (two rows of the padded H) and a row of the padded Q and I must
    // fit one ring slot; the attention takes head size 128 and up to 4 query heads per KV head,
    // and the gate/up input sums the O shares of at most 8 KV heads.
    if (s->H % 8 || s->Q % 8 || s->I % 8 || 4 * dec_kpad(s->H) > kDecSlot ||
        2 * dec_kpad(s->Q) > kDecSlot || 2 * dec_kpad(s->I) > kDecSlot || s->hd != kDecHd ||
        (s->G != 1 && s->G != 2 && s->G != 4) || s->nkv > kDecMaxAdds)
      return fail(s, PP_E_UNSUPPORTED, "geometry outside the decode kernel's row and slot sizes");
    const int vec = decode_vec_floats(s->H, s->Q, s->I, s->hd, s->G);
    size_t budget = dyn_smem_limit(s, pp_decode_step_kernel<1>);
    for (size_t b : {dyn_smem_limit(s, pp_decode_step_kernel<2>), dyn_smem_limit(s, pp_decode_step_kernel<4>)})
      budget = b < budget ? b : budget;
    // The fixed part at the smallest grid an SM limit allows (n_kv CTAs).
    const size_t fixed =
        DecodeSmem(0, vec, decode_own_cap(s, s->nkv), decode_part_rows(s->H, s->Q, s->KV, s->I, s->nkv, s->nkv))
            .total();
    const int ns = budget > fixed ? (int)((budget - fixed) / kDecSlot) : 0;
    if (ns < 2) return fail(s, PP_E_UNSUPPORTED, "the decode kernel's ring does not fit");
    pp_status r = decode_alloc(s);
    if (r) return r;
    s->dec_budget = budget;
    s->dec_vec = vec;
    s->dec_stale = true;
  }
  s->dec_on = enabled != 0;
  if (s->exec[0]) {
    cudaGraphExecDestroy(s->exec[0]);
    s->exec[0] = nullptr;
  }
  return PP_OK;
}
int32_t pp_shard_decode_kernel(const pp_shard* s) { return s && s->dec_on ? 1 : 0; }

pp_status pp_shard_set_pdl(pp_shard* s, int32_t enabled) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  s->use_pdl = enabled != 0;
  drop_graphs(s);
  return PP_OK;
}

pp_status pp_shard_set_wait_test(pp_shard* s, uint32_t limit_us, int32_t unreachable) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  s->dec_wait_ns = limit_us ? (uint64_t)limit_us * 1000 : kDecBarrierNs;
  s->dec_unreachable = unreachable ? 1 : 0;
  drop_graphs(s);
  return PP_OK;
}

pp_status pp_shard_set_taps(pp_shard* s, const uint32_t* layers, uint32_t n) {
  if (!s || (n && !layers)) return fail(s, PP_E_INVALID, "null argument");
  std::vector<int> t(layers, layers + n);
  std::sort(t.begin(), t.end());
  t.erase(std::unique(t.begin(), t.end()), t.end());
  for (int l : t) {
    // src/node.rs:118-124: the model's last layer feeds the logits and cannot be tapped.
    if (l + 1 >= (int)s->d.cfg.layers)
      return fail(s, PP_E_INVALID, "tapped layer %d must be below the model's last layer (%u)", l,
                  s->d.cfg.layers - 1);
    if (l < (int)s->d.layer_begin || l >= (int)s->d.layer_end)
      return fail(s, PP_E_INVALID, "tapped layer %d is outside the shard's layers [%u, %u)", l,
                  s->d.layer_begin, s->d.layer_end);
  }
  CK(cudaSetDevice(s->dev));
  if ((int)t.size() > s->taps_cap) {
    pp_status r = dalloc(s, &s->d_taps, t.size() * (size_t)kMaxRows * s->H * 4);
    if (r) return r;
    CK(cudaStreamSynchronize(s->stream));
    s->taps_cap = (int)t.size();
  }
  s->taps = t;
  drop_graphs(s);
  return PP_OK;
}

uint32_t pp_shard_tap_layers(const pp_shard* s, uint32_t* layers, uint32_t cap) {
  if (!s) return 0;
  for (size_t i = 0; i < s->taps.size() && i < cap; ++i) layers[i] = (uint32_t)s->taps[i];
  return (uint32_t)s->taps.size();
}

pp_status pp_shard_read_taps(pp_shard* s, uint32_t m, float* f32, uint16_t* bf16) {
  if (!s) return fail(s, PP_E_INVALID, "null shard");
  if (m == 0 || m > (uint32_t)kMaxRows) return fail(s, PP_E_INVALID, "m must be 1..%d", kMaxRows);
  CK(cudaSetDevice(s->dev));
  const size_t row = (size_t)m * s->H;
  std::vector<float> tmp(f32 ? 0 : row);
  for (size_t i = 0; i < s->taps.size(); ++i) {
    float* dst = f32 ? f32 + i * row : tmp.data();
    CK(cudaMemcpyAsync(dst, s->d_taps + i * (size_t)kMaxRows * s->H, row * 4,
                       cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    if (bf16) {
      // LayerTap::from_f32 (src/transport.rs:160-168): round to nearest even, NaN kept quiet.
      for (size_t j = 0; j < row; ++j) {
        uint32_t u;
        memcpy(&u, &dst[j], 4);
        bf16[i * row + j] = (u & 0x7fffffffu) > 0x7f800000u
                                ? (uint16_t)((u >> 16) | 0x40)
                                : (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
      }
    }
  }
  return PP_OK;
}

}  // extern "C"
