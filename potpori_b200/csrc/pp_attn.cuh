// Causal GQA attention of the verify chunk against the shard's KV cache
// (src/qwen/model.rs:282-302 `paged_attention` + `causal_bias`; the scalar statement is
// src/qwen/tiny.rs:77-101): for the query row at absolute position p = pos + r,
//   out = softmax(q . k_j / sqrt(head_dim), j = 0..p) . v_j
// Keys 0..pos-1 were written by earlier steps, keys pos..pos+m-1 by this step's QKV epilogue;
// rows past pos+m-1 (a rejected speculative tail) are never read, which is the reference's
// rollback-by-overwrite.
//
// Split-KV decode layout: one CTA per (KV head, key range); all G*m query vectors that share
// the KV head (G = n_heads / n_kv_heads <= 8) are processed together so every K/V byte is
// read once per step. A second kernel merges the per-split partials.
#pragma once
#include "pp_common.cuh"

namespace pp {

struct AttnArgs {
  const float* q;          // [MT][q_dim], normed and rotated
  const uint8_t* kcache;   // [n_kv][capacity] rows, split BF16 (kv_offset layout)
  const uint8_t* vcache;
  float* part;             // [n_kv][splits][nq_max][4 + head_dim]: max, sum, -, -, out
  uint8_t* out_split;      // attention output rows, split BF16 layout (input of the O GEMV)
  int32_t n_heads, n_kv, head_dim, capacity, splits, q_dim, nq_max;
  float scale;  // sqrt(head_dim); scores are divided by it as in tiny.rs:90
  const StepDesc* desc;
  StepResult* res;
};

constexpr int kAttnStages = 2;  // K/V tiles in flight per CTA
constexpr int kAttnSplitsPerSm = 2;  // key splits per KV head: at most this many per SM of the budget

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4a(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Shared memory of one attention unit (bytes from a 128-aligned base):
//   K/V tiles [stages][K, V][32 rows][row]  | queries [8*NT rows][row] (cache row format)
//   scores S[8*NT][33] F32 | probabilities P[hi, lo][8*NT][40] BF16 (80-byte rows)
//   running max, sum, rescale [8*NT] F32, causal limit [8*NT] int | mbarriers [stages]
struct AttnSmem {
  int rowb, nq8, stages;
  __host__ __device__ AttnSmem(int hd, int nt, int st)
      : rowb(kv_row_bytes(hd)), nq8(8 * nt), stages(st) {}
  __host__ __device__ size_t q_off() const { return (size_t)stages * 2 * kAttnTile * rowb; }
  __host__ __device__ size_t s_off() const { return q_off() + (size_t)nq8 * rowb; }
  __host__ __device__ size_t p_off() const { return s_off() + (size_t)nq8 * 33 * 4; }
  __host__ __device__ size_t st_off() const { return p_off() + (size_t)2 * nq8 * 80; }
  __host__ __device__ size_t bar_off() const { return st_off() + (size_t)4 * nq8 * 4; }
  __host__ __device__ size_t total() const { return bar_off() + 8 * (size_t)stages; }
};
__host__ inline size_t attn_smem_bytes(int hd, int nt) {
  return AttnSmem(hd, nt, kAttnStages).total() + 128;
}

// OR of a predicate over the 256 consumer threads (named barrier 1).
__device__ __forceinline__ bool consumer_or(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n"
      " barrier.red.or.pred po, 1, 256, pi;\n selp.u32 %0, 1, 0, po;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void attn_init_barriers(const AttnSmem& L, uint8_t* sm) {
  uint64_t* bar = (uint64_t*)(sm + L.bar_off());
  for (int i = 0; i < L.stages; ++i) mbar_init(&bar[i], 1);
  fence_barrier_init();
}

// Key range of split s: 32-key tiles [t0, t1) of the keys visible to the chunk's last row,
// keys [t0 * 32, kend).
__device__ __forceinline__ void attn_split_range(const AttnArgs& a, int s, int& t0, int& t1,
                                                 int& kend) {
  const int c = a.desc->pos + a.desc->m;  // keys visible to the last row
  const int ntiles = (c + kAttnTile - 1) / kAttnTile;
  const int tps = (ntiles + a.splits - 1) / a.splits;
  t0 = s * tps;
  t1 = min(ntiles, t0 + tps);
  kend = min(c, t1 * kAttnTile);
}

// Bulk copy of the K and V rows of tile `tile` (rows j0 .. min(j0 + 32, kend)) of KV head h into
// ring buffer `bi`, completing on bar[bi].
__device__ __forceinline__ void attn_issue_tile(const AttnArgs& a, const AttnSmem& L, uint8_t* sm,
                                                int h, int tile, int kend, int bi) {
  const int rowb = L.rowb;
  uint64_t* bar = (uint64_t*)(sm + L.bar_off());
  const int j0 = tile * kAttnTile;
  const uint32_t bytes = (uint32_t)min(kAttnTile, kend - j0) * rowb;
  uint8_t* dst = sm + (size_t)bi * 2 * kAttnTile * rowb;
  mbar_arrive_expect_tx(&bar[bi], 2 * bytes);
  bulk_load(dst, a.kcache + ((size_t)h * a.capacity + j0) * rowb, bytes, &bar[bi]);
  bulk_load(dst + (size_t)kAttnTile * rowb, a.vcache + ((size_t)h * a.capacity + j0) * rowb, bytes,
            &bar[bi]);
}

// Before the step's QKV kernel has finished (thread 0, the CTA's first unit): the first ring
// buffers' worth of this split's tiles whose keys all precede pos — rows written by earlier
// steps, which the QKV kernel does not touch. Returns the number of tiles issued.
__device__ __forceinline__ int attn_prefetch(const AttnArgs& a, int h, int s, const AttnSmem& L,
                                             uint8_t* sm) {
  int t0, t1, kend;
  attn_split_range(a, s, t0, t1, kend);
  const int pos = a.desc->pos;
  int n = 0;
  for (int tile = t0; tile < t1 && n < L.stages && (tile + 1) * kAttnTile <= pos; ++tile, ++n)
    attn_issue_tile(a, L, sm, h, tile, kend, n);
  return n;
}

// One (KV head h, key split s) unit on the 8 consumer warps (threads 0..255), NT query tiles
// of 8 (NT = ceil(G*MT / 8)). Per 32-key tile, on the tensor cores (m16n8k16 BF16, F32
// accumulate), every F32 operand carried as hi + lo BF16 and the three products
// hi.hi + hi.lo + lo.hi (about 2^-16 relative, the reference's F32 arithmetic to within its
// rounding):
//  1. S^T = K . Q^T: the 32 keys are the M dimension (two m16 tiles), the queries N; a warp
//     takes one (key tile, query tile) unit; scaled by 1/sqrt(head_dim) and masked (split
//     range, causal limit pos + r) into S.
//  2. Online softmax per query (a warp per query, lane = key): running max, rescale factor,
//     running sum; P = exp(S - max) written as hi/lo BF16.
//  3. O^T += V^T . P^T: head dims are M (ldmatrix.trans of the V rows), queries N; a warp owns
//     16 dims x its query tiles, accumulators rescaled first.
// K/V tiles are contiguous 32-row blocks of the cache, fetched by thread 0 with one bulk copy
// each into a ring of L.stages buffers (mbarrier completion, bounded waits). `uses` counts the
// tiles this CTA has taken through the ring before (buffer and parity of the next one); it is
// advanced on return. `issued` tiles of the unit were requested already (attn_prefetch, thread
// 0 only). Writes the split's partial (max, sum, unnormalised output) and returns false when a
// wait expired (ST_TIMEOUT set, copies in flight drained).
template <int MT, int NT>
__device__ __forceinline__ bool attn_unit(const AttnArgs& a, int h, int s, const AttnSmem& L,
                                          uint8_t* sm, uint32_t& uses, int issued = 0) {
  const int hd = a.head_dim, hdk = kv_hdk(hd), mask = kv_swz_mask(hd);
  const int rowb = L.rowb, S = L.stages;
  constexpr int NQ8 = 8 * NT;
  uint8_t* kvs = sm;
  uint8_t* qsm = sm + L.q_off();
  float* S_s = (float*)(sm + L.s_off());
  uint8_t* P_s = sm + L.p_off();
  float* m_s = (float*)(sm + L.st_off());
  float* l_s = m_s + NQ8;
  float* al_s = l_s + NQ8;
  int* lim_s = (int*)(al_s + NQ8);
  uint64_t* bar = (uint64_t*)(sm + L.bar_off());

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = a.desc->pos, m = a.desc->m;
  const int G = a.n_heads / a.n_kv;
  const int nq = G * MT;
  int t0, t1, kend;  // this split covers keys [t0*32, kend)
  attn_split_range(a, s, t0, t1, kend);

  int next_issue = t0 + issued;  // thread 0: first tile not yet requested
  auto issue = [&](int tile) {
    const uint32_t k = uses + (uint32_t)(tile - t0);
    attn_issue_tile(a, L, sm, h, tile, kend, (int)(k % (uint32_t)S));
  };
  if (tid == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (; next_issue < t1 && next_issue < t0 + S; ++next_issue) issue(next_issue);
  }

  // Queries of this KV head (qi = g * MT + r: query head h*G + g, chunk row r) as hi/lo rows;
  // a thread converts 16 dims with its loads issued together.
  for (int e = tid; e < NQ8 * (hdk / 16); e += kAttnThreads) {
    const int qi = e / (hdk / 16), d0 = (e - qi * (hdk / 16)) * 16;
    const int g = qi / MT, r = qi - g * MT;
    const bool valid = qi < nq && r < m;
    const float* src = a.q + (size_t)r * a.q_dim + (h * G + g) * hd;
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      v[j] = (valid && d0 + 4 * j < hd) ? *(const float4*)(src + d0 + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
    uint8_t* row = qsm + (size_t)qi * rowb;
    // Two 16-byte units (dims d0 .. d0 + 7 and d0 + 8 .. d0 + 15) of hi and of lo parts, each
    // stored whole where kv_offset puts it.
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float x[8] = {v[2 * u].x, v[2 * u].y, v[2 * u].z, v[2 * u].w,
                          v[2 * u + 1].x, v[2 * u + 1].y, v[2 * u + 1].z, v[2 * u + 1].w};
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint16_t h0, l0, h1, l1;
        split_bf16(x[2 * p], h0, l0);
        split_bf16(x[2 * p + 1], h1, l1);
        hw[p] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lw[p] = (uint32_t)l0 | ((uint32_t)l1 << 16);
      }
      const int d = d0 + 8 * u;
      *(uint4*)(row + kv_offset(qi, d, 0, hd)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *(uint4*)(row + kv_offset(qi, d, 1, hd)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  for (int q = tid; q < NQ8; q += kAttnThreads) {
    const int r = q % MT;
    lim_s[q] = (q < nq && r < m) ? pos + r : -1;
    m_s[q] = -INFINITY;
    l_s[q] = 0.f;
  }
  consumer_sync();

  const float inv_scale = 1.0f / a.scale;
  const int mtd_n = hdk / 16;  // 16-dim tiles of the output
  const int g4 = lane >> 2, t4 = lane & 3, mat = lane >> 3, l7 = lane & 7;
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;

  bool ok = true;
  for (int tile = t0; tile < t1; ++tile) {
    const uint32_t k = uses + (uint32_t)(tile - t0);
    const int bi = (int)(k % (uint32_t)S);
    const int j0 = tile * kAttnTile, nrows = min(kAttnTile, kend - j0);
    const uint8_t* kt = kvs + (size_t)bi * 2 * kAttnTile * rowb;
    const uint8_t* vt = kt + (size_t)kAttnTile * rowb;
    // V rows past the split's keys are zeroed (P is 0 there, and 0 * stale bits must be 0).
    for (int e = nrows * rowb / 16 + tid; e < kAttnTile * rowb / 16; e += kAttnThreads)
      ((uint4*)vt)[e] = make_uint4(0u, 0u, 0u, 0u);
    const bool mine = mbar_wait(&bar[bi], (k / (uint32_t)S) & 1u);
    if (consumer_or(!mine)) {
      ok = false;
      break;
    }

    // ---- 1. S^T = K . Q^T
    for (int u = warp; u < 2 * NT; u += 8) {
      const int mt = u & 1, nt = u >> 1;
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
      const int arow = mt * 16 + l7 + (mat & 1) * 8;
      const uint8_t* krow = kt + (size_t)arow * rowb;
      const int brow = nt * 8 + l7;
      const uint8_t* qrow = qsm + (size_t)brow * rowb + (mat >> 1) * 2 * hdk;
      for (int ks = 0; ks < hdk / 16; ++ks) {
        uint32_t khi[4], klo[4], qf[4];
        const int ua = 2 * ks + (mat >> 1);
        ldmatrix_x4a(khi, krow + ((ua ^ (arow & mask)) << 4));
        ldmatrix_x4a(klo, krow + 2 * hdk + ((ua ^ (arow & mask)) << 4));
        const int ub = 2 * ks + (mat & 1);
        ldmatrix_x4a(qf, qrow + ((ub ^ (brow & mask)) << 4));
        mma_bf16_16816(acc0, khi, qf[0], qf[1]);
        mma_bf16_16816(acc1, khi, qf[2], qf[3]);
        mma_bf16_16816(acc0, klo, qf[0], qf[1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = mt * 16 + g4 + (e >> 1) * 8, q = nt * 8 + 2 * t4 + (e & 1);
        const int jg = j0 + key;
        const bool vis = jg < kend && jg <= lim_s[q];
        S_s[q * 33 + key] = vis ? (acc0[e] + acc1[e]) * inv_scale : -INFINITY;
      }
    }
    consumer_sync();

    // ---- 2. online softmax, lane = key; warp w takes queries w, w + 8, ... (NT of them), their
    // shuffle reductions interleaved
    {
      float sc[NT], mo[NT], mx[NT];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int q = warp + 8 * i;
        sc[i] = S_s[q * 33 + lane];
        mo[i] = m_s[q];
        mx[i] = sc[i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < NT; ++i) mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], o));
      float p[NT], ps[NT], alpha[NT];
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        mx[i] = fmaxf(mo[i], mx[i]);
        alpha[i] = (mo[i] == -INFINITY) ? 0.f : __expf(mo[i] - mx[i]);
        p[i] = (sc[i] == -INFINITY) ? 0.f : __expf(sc[i] - mx[i]);
        ps[i] = p[i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < NT; ++i) ps[i] += __shfl_xor_sync(0xffffffffu, ps[i], o);
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int q = warp + 8 * i;
        uint16_t ph, pl;
        split_bf16(p[i], ph, pl);
        *(uint16_t*)(P_s + (size_t)q * 80 + lane * 2) = ph;
        *(uint16_t*)(P_s + (size_t)(NQ8 + q) * 80 + lane * 2) = pl;
        if (lane == 0) {
          m_s[q] = mx[i];
          l_s[q] = l_s[q] * alpha[i] + ps[i];
          al_s[q] = alpha[i];
        }
      }
    }
    consumer_sync();

    // ---- 3. O^T += V^T . P^T
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int u = warp + 8 * i;
      if (u >= mtd_n * NT) break;
      const int mtd = u % mtd_n, nt = u / mtd_n;
      const float a0 = al_s[nt * 8 + 2 * t4], a1 = al_s[nt * 8 + 2 * t4 + 1];
      o[i][0] *= a0;
      o[i][1] *= a1;
      o[i][2] *= a0;
      o[i][3] *= a1;
      uint32_t phi[4], plo[4];
      const uint8_t* prow = P_s + (size_t)(nt * 8 + l7) * 80 + mat * 16;
      ldmatrix_x4a(phi, prow);
      ldmatrix_x4a(plo, prow + (size_t)NQ8 * 80);
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int vrow = ks * 16 + l7 + 8 * (mat >> 1);
        const int uv = 2 * mtd + (mat & 1);
        const uint8_t* va = vt + (size_t)vrow * rowb + ((uv ^ (vrow & mask)) << 4);
        uint32_t vhi[4], vlo[4];
        ldmatrix_x4_trans(vhi, va);
        ldmatrix_x4_trans(vlo, va + 2 * hdk);
        mma_bf16_16816(o[i], vhi, phi[2 * ks], phi[2 * ks + 1]);
        mma_bf16_16816(o[i], vhi, plo[2 * ks], plo[2 * ks + 1]);
        mma_bf16_16816(o[i], vlo, phi[2 * ks], phi[2 * ks + 1]);
      }
    }
    consumer_sync();  // the tile's buffer, S and P are free
    if (tid == 0 && next_issue < t1) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(next_issue++);
    }
  }

  if (!ok) {
    if (tid == 0) {
      atomicOr(&a.res->status, ST_TIMEOUT);
      // Let the copies still in flight land before the shared memory is reused or released.
      for (int tt = max(t0, next_issue - S); tt < next_issue; ++tt) {
        const uint32_t k = uses + (uint32_t)(tt - t0);
        mbar_wait(&bar[k % (uint32_t)S], (k / (uint32_t)S) & 1u);
      }
    }
    return false;
  }
  uses += (uint32_t)max(0, t1 - t0);

  // Partial of this split: running max, running sum, unnormalised output.
  float* pbase = a.part + ((size_t)h * a.splits + s) * a.nq_max * (hd + 4);
  for (int q = tid; q < nq; q += kAttnThreads) {
    pbase[(size_t)q * (hd + 4) + 0] = m_s[q];
    pbase[(size_t)q * (hd + 4) + 1] = l_s[q];
  }
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int u = warp + 8 * i;
    if (u >= mtd_n * NT) break;
    const int mtd = u % mtd_n, nt = u / mtd_n;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int dim = mtd * 16 + g4 + (e >> 1) * 8, q = nt * 8 + 2 * t4 + (e & 1);
      if (q < nq && dim < hd) pbase[(size_t)q * (hd + 4) + 4 + dim] = o[i][e];
    }
  }
  consumer_sync();  // m_s / l_s and the query rows are free for the next unit
  return true;
}

template <int MT, int NT>
__global__ void __launch_bounds__(kAttnThreads) pp_attn_split_kernel(const AttnArgs a) {
  extern __shared__ uint8_t attn_smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)attn_smem_raw + 127) & ~(uintptr_t)127);
  const AttnSmem L(a.head_dim, NT, kAttnStages);
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (bad_step(a.desc, a.capacity, MT)) return;
  int issued = 0;
  if (threadIdx.x == 0) {
    attn_init_barriers(L, sm);
    issued = attn_prefetch(a, blockIdx.x, blockIdx.y, L, sm);
  }
  pdl_wait();
  consumer_sync();  // barrier init visible to every thread
  uint32_t uses = 0;
  attn_unit<MT, NT>(a, blockIdx.x, blockIdx.y, L, sm, uses, issued);
}

// Merge of the splits of one (query head hq, chunk row r) by `nthr` threads (t = 0..nthr-1,
// nthr >= head_dim, synchronised on named barrier `bar_id`), one thread per dimension. Every
// split's (max, sum) pair and output value is fetched in one batch of independent loads (up
// to 64 splits per round trip); the merge weights are exp(max_s - max), formed by the first
// warp (lane k sums splits k, k + 32, ..., then a butterfly over the lanes; nthr >= 32).
// sm_m / sm_w: [splits] floats of shared memory, red_l: one float.
template <int MT>
__device__ __forceinline__ void combine_unit(const AttnArgs& a, int hq, int r, int t, int nthr,
                                             int bar_id, float* sm_m, float* sm_w, float* red_l) {
  const int G = a.n_heads / a.n_kv;
  const int h = hq / G, g = hq - h * G;
  const int qi = g * MT + r;
  const int hd = a.head_dim;
  const size_t stride = (size_t)a.nq_max * (hd + 4);
  const float* base = a.part + ((size_t)h * a.splits * a.nq_max + qi) * (hd + 4);
  const int S = a.splits;
  for (int s = t; s < S; s += nthr) {
    const float2 ml = __ldcg((const float2*)(base + s * stride));
    sm_m[s] = ml.x;
    sm_w[s] = ml.y;
  }
  // Output values of the first kPv splits, in flight while the weights are formed.
  constexpr int kPv = 64;
  const int dd = t;
  float pv[kPv];
#pragma unroll
  for (int q = 0; q < kPv; ++q)
    pv[q] = (q < S && dd < hd) ? __ldcg(base + q * stride + 4 + dd) : 0.f;
  named_sync(bar_id, nthr);
  if (t < 32) {  // the first warp: lane k takes splits k, k + 32, ...
    float mx = -INFINITY;
    for (int s = t; s < S; s += 32) mx = fmaxf(mx, sm_m[s]);
    mx = warp_max(mx);
    float l = 0.f;
    for (int s = t; s < S; s += 32) {
      const float f = (sm_m[s] == -INFINITY) ? 0.f : expf(sm_m[s] - mx);
      l += sm_w[s] * f;
      sm_w[s] = f;  // now the scale of split s
    }
    l = warp_sum(l);
    if (t == 0) *red_l = l;
  }
  named_sync(bar_id, nthr);
  if (dd < hd) {
    float o = 0.f;
#pragma unroll
    for (int q = 0; q < kPv; ++q)
      if (q < S) o += pv[q] * sm_w[q];
    for (int s = kPv; s < S; ++s) o += __ldcg(base + s * stride + 4 + dd) * sm_w[s];
    store_split<MT>(a.out_split, r, hq * hd + dd, o / *red_l);
  }
  named_sync(bar_id, nthr);  // sm_m / sm_w / red_l are free again
}

// Grid (n_heads, m), block max(32, head_dim) threads.
template <int MT>
__global__ void pp_attn_combine_kernel(const AttnArgs a) {
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (bad_step(a.desc, a.capacity, MT)) return;
  pdl_wait();
  if ((int)blockIdx.y >= a.desc->m) return;
  __shared__ float sm_m[256], sm_w[256];
  __shared__ float red_l;
  combine_unit<MT>(a, blockIdx.x, blockIdx.y, threadIdx.x, blockDim.x, 1, sm_m, sm_w, &red_l);
}

}  // namespace pp
