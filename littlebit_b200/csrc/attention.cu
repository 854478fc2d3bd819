// Decode / verify attention over a bf16 KV cache for sm_100a.
//
// Replaces fused_attention (patches/littlebit_cpu_optimized.cpp:1172-1301) and
// the causal loop of full_forward_batch (cpp:1963-2021), adding what the CPU
// path lacks: rotary embedding (HF Llama rotate_half form), a bf16 cache,
// and tree masks for tree verification (tree_utils.py:72-175 masks).
//
// Split over the key sequence in fixed 64-key chunks (flash-decoding): CTA
// (chunk c, kv head h) scores every query row of the GQA group against its
// chunk and writes an unnormalised partial (max, sum, Σ p·v); a combine kernel
// merges the chunks in chunk order.  Keys are ordered by their RANK in each
// query's visible sequence -- the cached prefix by slot, then the visible new
// tokens in index order -- and chunk membership, lane placement in the
// reductions and the p·v order all follow the rank.  A query's output is
// therefore the same bit pattern whether it is decoded alone, inside a causal
// verify batch, or as a node of a tree whose ancestors sit at scattered slots.
//
// New tokens' keys are rotated, rounded to bf16 and written to the cache by
// the CTA whose chunk holds their slot; the same CTA uses the rounded values,
// so no CTA ever reads a cache slot written in the same launch.

#include "common.cuh"

namespace lbx {

constexpr int ACH = 64;       // key slots per chunk
constexpr int ATHREADS = 128;
constexpr int AMAX_ROWS = 64; // query rows (tokens x GQA group) per CTA; more rows -> more CTAs

struct AttnParams {
  int n, heads, kvh, d, max_seq, prefix, rep, R, nchunk;
  const int32_t *prefix_dev;  // actual cached-slot count (prefix is then a bound)
  float scale, theta;
  const float *q; int64_t q_ld;
  const float *k_new; const float *v_new; int64_t kv_ld;
  const int32_t *pos;
  const uint64_t *tree;
  uint16_t *kc; uint16_t *vc;
  float *out;
  float *part_o;  // [kvh][nchunk][R][d]
  float2 *part_ml; // [kvh][nchunk][R]
};

LBX_DEV void rope_cs_a(int pos, int i, int d, float theta, float &c, float &s) {
  if (!(theta > 0.f)) {  // theta <= 0: no rotation (the reference CPU runtime applies none)
    c = 1.f;
    s = 0.f;
    return;
  }
  const double inv = pow((double)theta, -2.0 * (double)i / (double)d);
  double sd, cd;
  sincos((double)pos * inv, &sd, &cd);
  c = (float)cd;
  s = (float)sd;
}

__global__ void __launch_bounds__(ATHREADS) attn_chunk_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  const int d = p.d, half = d / 2;
  const int c = blockIdx.x, h = blockIdx.y;
  const int rlo = blockIdx.z * AMAX_ROWS;        // this CTA's query rows: rlo .. rlo+Rg-1
  const int Rg = min(AMAX_ROWS, p.R - rlo);
  const int tid = threadIdx.x;
  float *Ks = sm;                       // ACH x (d+1)   cached keys of ranks 64c..64c+63
  float *Vs = Ks + ACH * (d + 1);       // ACH x d
  float *Kn = Vs + ACH * d;             // n x (d+1)     the new tokens' keys (rotated, bf16-rounded)
  float *Vn = Kn + p.n * (d + 1);       // n x d
  float *Qs = Vn + p.n * d;             // Rg x d
  float *P = Qs + AMAX_ROWS * d;        // Rg x ACH
  uint8_t *sel = reinterpret_cast<uint8_t *>(P + AMAX_ROWS * ACH);  // n x 64: t-th visible new token of query i
  __shared__ int s_cnt[64];

  pdl_trigger();
  pdl_wait();
  const int prefix = p.prefix_dev ? __ldcg(p.prefix_dev) : p.prefix;
  const int total = prefix + p.n;
  const int64_t pbase = ((int64_t)h * p.nchunk + c) * p.R;
  if (c * ACH >= total) {  // chunk past the live sequence: an empty partial
    for (int r = tid; r < Rg; r += ATHREADS) p.part_ml[pbase + rlo + r] = make_float2(-INFINITY, 0.f);
    return;
  }
  const int r0 = c * ACH;                 // first rank of this chunk
  const bool has_new = r0 + ACH > prefix; // ranks >= prefix name new tokens

  // visible new tokens of each query in index order (tree: the set bits of its
  // mask, which for generate_tree_buffers trees is root-to-node depth order;
  // causal: 0..i), so rank prefix+t of query i is new token sel[i][t]
  if (has_new && tid < p.n) {
    const int i = tid;
    int cnt = 0;
    if (p.tree) {
      uint64_t m = p.tree[i];
      if (p.n < 64) m &= (1ull << p.n) - 1ull;
      while (m) {
        const int j = __ffsll((long long)m) - 1;
        sel[i * 64 + cnt++] = (uint8_t)j;
        m &= m - 1ull;
      }
    } else {
      for (int j = 0; j <= i; ++j) sel[i * 64 + cnt++] = (uint8_t)j;
    }
    s_cnt[i] = cnt;
  }

  // queries of this kv head's group, rotated
  for (int e = tid; e < Rg * half; e += ATHREADS) {
    const int r = e / half, j = e - r * half;
    const int gr = rlo + r;
    const int i = gr / p.rep, qh = h * p.rep + (gr - i * p.rep);
    const float *qr = p.q + (int64_t)i * p.q_ld + (int64_t)qh * d;
    float cs, sn;
    rope_cs_a(p.pos[i], j, d, p.theta, cs, sn);
    const float x1 = qr[j], x2 = qr[j + half];
    Qs[r * d + j] = x1 * cs - x2 * sn;
    Qs[r * d + j + half] = x2 * cs + x1 * sn;
  }
  // cached keys / values of ranks r0.. (rank == slot below the prefix)
  const int64_t cache_base = (int64_t)h * p.max_seq * d;
  for (int e = tid; e < ACH * half; e += ATHREADS) {
    const int jj = e / half, j = e - jj * half;
    const int slot = r0 + jj;
    float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
    if (slot < prefix) {
      const uint16_t *kr = p.kc + cache_base + (int64_t)slot * d;
      const uint16_t *vr = p.vc + cache_base + (int64_t)slot * d;
      k1 = bf16_to_f32(kr[j]); k2 = bf16_to_f32(kr[j + half]);
      v1 = bf16_to_f32(vr[j]); v2 = bf16_to_f32(vr[j + half]);
    }
    Ks[jj * (d + 1) + j] = k1; Ks[jj * (d + 1) + j + half] = k2;
    Vs[jj * d + j] = v1; Vs[jj * d + j + half] = v2;
  }
  // the new tokens: rotate, round to bf16; the CTA whose slot range holds
  // cache slot prefix+j writes it (no CTA reads a slot written in this launch)
  if (has_new) {
    for (int e = tid; e < p.n * half; e += ATHREADS) {
      const int i = e / half, j = e - i * half;
      const float *kr = p.k_new + (int64_t)i * p.kv_ld + (int64_t)h * d;
      const float *vr = p.v_new + (int64_t)i * p.kv_ld + (int64_t)h * d;
      float cs, sn;
      rope_cs_a(p.pos[i], j, d, p.theta, cs, sn);
      const uint16_t b1 = f32_to_bf16(kr[j] * cs - kr[j + half] * sn);
      const uint16_t b2 = f32_to_bf16(kr[j + half] * cs + kr[j] * sn);
      const uint16_t c1 = f32_to_bf16(vr[j]), c2 = f32_to_bf16(vr[j + half]);
      const int slot = prefix + i;
      if (slot >= r0 && slot < r0 + ACH) {
        uint16_t *kw = p.kc + cache_base + (int64_t)slot * d;
        uint16_t *vw = p.vc + cache_base + (int64_t)slot * d;
        kw[j] = b1; kw[j + half] = b2; vw[j] = c1; vw[j + half] = c2;
      }
      Kn[i * (d + 1) + j] = bf16_to_f32(b1); Kn[i * (d + 1) + j + half] = bf16_to_f32(b2);
      Vn[i * d + j] = bf16_to_f32(c1); Vn[i * d + j + half] = bf16_to_f32(c2);
    }
  }
  __syncthreads();

  // scores by rank: every quantity below depends only on the key's rank in
  // the query's visible sequence, so a tree node computes exactly what the
  // same token computes when its path is decoded as a plain causal sequence
  for (int e = tid; e < Rg * ACH; e += ATHREADS) {
    const int r = e / ACH, jj = e - r * ACH;
    const int i = (rlo + r) / p.rep;
    const int rank = r0 + jj;
    const float *kr = nullptr;
    if (rank < prefix) {
      kr = Ks + jj * (d + 1);
    } else {
      const int t = rank - prefix;
      if (t < s_cnt[i]) kr = Kn + sel[i * 64 + t] * (d + 1);
    }
    float sc = -INFINITY;
    if (kr) {
      const float *qr = Qs + r * d;
      float a = 0.f;
      for (int t = 0; t < d; ++t) a = fmaf(qr[t], kr[t], a);
      sc = a * p.scale;
    }
    P[r * ACH + jj] = sc;
  }
  __syncthreads();

  // chunk-local softmax numerators
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < Rg; r += ATHREADS / 32) {
    const float s0 = P[r * ACH + lane], s1 = P[r * ACH + lane + 32];
    const float m = warp_max(fmaxf(s0, s1));
    float e0 = 0.f, e1 = 0.f;
    if (m != -INFINITY) {
      e0 = s0 == -INFINITY ? 0.f : expf(s0 - m);
      e1 = s1 == -INFINITY ? 0.f : expf(s1 - m);
    }
    P[r * ACH + lane] = e0;
    P[r * ACH + lane + 32] = e1;
    const float l = warp_sum(e0 + e1);
    if (lane == 0) p.part_ml[pbase + rlo + r] = make_float2(m, l);
  }
  __syncthreads();

  // Σ p·v in rank order (invisible ranks carry p = 0 and v = 0)
  for (int e = tid; e < Rg * d; e += ATHREADS) {
    const int r = e / d, t = e - r * d;
    const int i = (rlo + r) / p.rep;
    const float *pr = P + r * ACH;
    float a = 0.f;
    for (int jj = 0; jj < ACH; ++jj) {
      const int rank = r0 + jj;
      float v = 0.f;
      if (rank < prefix) {
        v = Vs[jj * d + t];
      } else {
        const int tt = rank - prefix;
        if (tt < s_cnt[i]) v = Vn[sel[i * 64 + tt] * d + t];
      }
      a = fmaf(pr[jj], v, a);
    }
    p.part_o[(pbase + rlo + r) * d + t] = a;
  }
}

__global__ void attn_combine_kernel(const __grid_constant__ AttnParams p) {
  const int r = blockIdx.x, h = blockIdx.y;
  const int d = p.d;
  pdl_trigger();
  pdl_wait();
  float M = -INFINITY;
  for (int c = 0; c < p.nchunk; ++c) M = fmaxf(M, __ldcg(p.part_ml + ((int64_t)h * p.nchunk + c) * p.R + r).x);
  const int i = r / p.rep, qh = h * p.rep + (r - i * p.rep);
  for (int t = threadIdx.x; t < d; t += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int c = 0; c < p.nchunk; ++c) {
      const int64_t b = ((int64_t)h * p.nchunk + c) * p.R + r;
      const float2 ml = __ldcg(p.part_ml + b);
      if (ml.x == -INFINITY) continue;
      const float w = expf(ml.x - M);
      L = fmaf(w, ml.y, L);
      O = fmaf(w, __ldcg(p.part_o + b * d + t), O);
    }
    p.out[(int64_t)i * p.heads * d + (int64_t)qh * d + t] = L > 0.f ? O / L : 0.f;
  }
}

static void attn_fill(const lbx_attn_args *a, AttnParams &p) {
  p.n = a->n;
  p.heads = a->heads;
  p.kvh = a->kv_heads;
  p.d = a->head_dim;
  p.max_seq = a->max_seq;
  p.prefix = a->prefix_len;
  p.rep = a->heads / a->kv_heads;
  p.R = a->n * p.rep;
  p.nchunk = (a->prefix_len + a->n + ACH - 1) / ACH;
  p.scale = a->scale;
  p.theta = a->theta;
  p.q = a->q;
  p.q_ld = a->q_ld ? a->q_ld : (int64_t)a->heads * a->head_dim;
  p.k_new = a->k_new;
  p.v_new = a->v_new;
  p.kv_ld = a->kv_ld ? a->kv_ld : (int64_t)a->kv_heads * a->head_dim;
  p.pos = a->pos;
  p.tree = a->tree_mask;
  p.kc = a->k_cache;
  p.vc = a->v_cache;
  p.out = a->out;
  p.prefix_dev = a->prefix_dev;
}

}  // namespace lbx

extern "C" size_t lbx_attn_workspace_size(const lbx_attn_args *a) {
  if (!a || a->n < 1 || a->kv_heads < 1 || a->heads < a->kv_heads) return 0;
  const int rep = a->heads / a->kv_heads;
  const int64_t R = (int64_t)a->n * rep;
  const int64_t nchunk = (a->prefix_len + a->n + lbx::ACH - 1) / lbx::ACH;
  const size_t o = (size_t)a->kv_heads * nchunk * R * a->head_dim * 4;
  const size_t ml = (size_t)a->kv_heads * nchunk * R * 8;
  return ((o + 255) & ~(size_t)255) + ml;
}

extern "C" int lbx_attn_decode(const lbx_attn_args *a, void *ws, size_t ws_bytes,
                               cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(a, "args is NULL");
  LBX_CHECK_ARG(a->n >= 1 && a->n <= 64, "n must be in [1,64]");
  LBX_CHECK_ARG(a->kv_heads >= 1 && a->heads >= a->kv_heads && a->heads % a->kv_heads == 0,
                "heads must be a multiple of kv_heads");
  LBX_CHECK_ARG(a->head_dim > 0 && a->head_dim <= 128 && a->head_dim % 2 == 0,
                "head_dim must be even and <= 128");
  LBX_CHECK_ARG(a->prefix_len >= 0 && a->prefix_len + a->n <= a->max_seq,
                "prefix_len + n exceeds max_seq");
  LBX_CHECK_ARG(a->q && a->k_new && a->v_new && a->pos && a->k_cache && a->v_cache && a->out,
                "NULL pointer");
  const size_t need = lbx_attn_workspace_size(a);
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  AttnParams p = {};
  attn_fill(a, p);
  const size_t o = (size_t)p.kvh * p.nchunk * p.R * p.d * 4;
  p.part_o = reinterpret_cast<float *>(ws);
  p.part_ml = reinterpret_cast<float2 *>(reinterpret_cast<uint8_t *>(ws) + ((o + 255) & ~(size_t)255));
  const size_t smem = ((size_t)ACH * (p.d + 1) + (size_t)ACH * p.d + (size_t)p.n * (p.d + 1) +
                       (size_t)p.n * p.d + (size_t)AMAX_ROWS * p.d + (size_t)AMAX_ROWS * ACH) * 4 +
                      (size_t)p.n * 64;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = allow_max_smem(attn_chunk_kernel);
    if (e != cudaSuccess) return cuda_status(e, "attn smem attribute");
    attr_done = true;
  }
  const bool pdl = a->use_pdl != 0;
  const int ngroups = (p.R + AMAX_ROWS - 1) / AMAX_ROWS;
  cudaError_t e = launch(attn_chunk_kernel, dim3(p.nchunk, p.kvh, ngroups), dim3(ATHREADS), smem, stream, pdl, p);
  if (e != cudaSuccess) return cuda_status(e, "attn chunk launch");
  e = launch(attn_combine_kernel, dim3(p.R, p.kvh), dim3(128), 0, stream, pdl, p);
  return cuda_status(e, "attn combine launch");
}
