// Decode / verify attention over a bf16 KV cache for sm_100a.
//
// Replaces fused_attention (patches/littlebit_cpu_optimized.cpp:1172-1301) and
// the causal loop of full_forward_batch (cpp:1963-2021), adding what the CPU
// path lacks: rotary embedding (HF Llama rotate_half form), a bf16 cache,
// and tree masks for tree verification (tree_utils.py:72-175 masks).
//
// Split over the key sequence in fixed 64-slot chunks (flash-decoding): CTA
// (chunk c, kv head h) scores every query row of the GQA group against its
// chunk and writes an unnormalised partial (max, sum, Σ p·v); a combine kernel
// merges the chunks in chunk order.  Chunk boundaries depend only on slot
// indices, and masked keys contribute exact zeros, so a query's output is the
// same bit pattern whether it is decoded alone or inside a verify batch.
//
// New tokens' keys are rotated, rounded to bf16 and written to the cache by
// the CTA whose chunk holds their slot; the same CTA uses the rounded values,
// so no CTA ever reads a cache slot written in the same launch.

#include "common.cuh"

namespace lbx {

constexpr int ACH = 64;       // key slots per chunk
constexpr int ATHREADS = 128;
constexpr int AMAX_ROWS = 64; // query rows (tokens x GQA group) per launch

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
  const double inv = pow((double)theta, -2.0 * (double)i / (double)d);
  double sd, cd;
  sincos((double)pos * inv, &sd, &cd);
  c = (float)cd;
  s = (float)sd;
}

LBX_DEV bool visible(const AttnParams &p, int prefix, int i, int slot) {
  if (slot < prefix) return true;
  const int j = slot - prefix;
  if (j >= p.n) return false;
  if (p.tree) return (p.tree[i] >> j) & 1ull;
  return j <= i;
}

__global__ void __launch_bounds__(ATHREADS) attn_chunk_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  const int d = p.d, half = d / 2;
  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x;
  float *Ks = sm;                       // ACH x (d+1)
  float *Vs = Ks + ACH * (d + 1);       // ACH x d
  float *Qs = Vs + ACH * d;             // R x d
  float *P = Qs + p.R * d;              // R x ACH

  pdl_trigger();
  pdl_wait();
  const int prefix = p.prefix_dev ? __ldcg(p.prefix_dev) : p.prefix;
  const int total = prefix + p.n;
  const int64_t pbase = ((int64_t)h * p.nchunk + c) * p.R;
  if (c * ACH >= total) {  // chunk past the live sequence: an empty partial
    for (int r = tid; r < p.R; r += ATHREADS) p.part_ml[pbase + r] = make_float2(-INFINITY, 0.f);
    return;
  }

  // queries of this kv head's group, rotated
  for (int e = tid; e < p.R * half; e += ATHREADS) {
    const int r = e / half, j = e - r * half;
    const int i = r / p.rep, qh = h * p.rep + (r - i * p.rep);
    const float *qr = p.q + (int64_t)i * p.q_ld + (int64_t)qh * d;
    float cs, sn;
    rope_cs_a(p.pos[i], j, d, p.theta, cs, sn);
    const float x1 = qr[j], x2 = qr[j + half];
    Qs[r * d + j] = x1 * cs - x2 * sn;
    Qs[r * d + j + half] = x2 * cs + x1 * sn;
  }
  // keys / values of this chunk
  const int64_t cache_base = (int64_t)h * p.max_seq * d;
  for (int e = tid; e < ACH * half; e += ATHREADS) {
    const int jj = e / half, j = e - jj * half;
    const int slot = c * ACH + jj;
    float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
    if (slot < prefix) {
      const uint16_t *kr = p.kc + cache_base + (int64_t)slot * d;
      const uint16_t *vr = p.vc + cache_base + (int64_t)slot * d;
      k1 = bf16_to_f32(kr[j]); k2 = bf16_to_f32(kr[j + half]);
      v1 = bf16_to_f32(vr[j]); v2 = bf16_to_f32(vr[j + half]);
    } else if (slot < total) {
      const int i = slot - prefix;
      const float *kr = p.k_new + (int64_t)i * p.kv_ld + (int64_t)h * d;
      const float *vr = p.v_new + (int64_t)i * p.kv_ld + (int64_t)h * d;
      float cs, sn;
      rope_cs_a(p.pos[i], j, d, p.theta, cs, sn);
      const uint16_t b1 = f32_to_bf16(kr[j] * cs - kr[j + half] * sn);
      const uint16_t b2 = f32_to_bf16(kr[j + half] * cs + kr[j] * sn);
      const uint16_t c1 = f32_to_bf16(vr[j]), c2 = f32_to_bf16(vr[j + half]);
      uint16_t *kw = p.kc + cache_base + (int64_t)slot * d;
      uint16_t *vw = p.vc + cache_base + (int64_t)slot * d;
      kw[j] = b1; kw[j + half] = b2; vw[j] = c1; vw[j + half] = c2;
      k1 = bf16_to_f32(b1); k2 = bf16_to_f32(b2); v1 = bf16_to_f32(c1); v2 = bf16_to_f32(c2);
    }
    Ks[jj * (d + 1) + j] = k1; Ks[jj * (d + 1) + j + half] = k2;
    Vs[jj * d + j] = v1; Vs[jj * d + j + half] = v2;
  }
  __syncthreads();

  // scores
  for (int e = tid; e < p.R * ACH; e += ATHREADS) {
    const int r = e / ACH, jj = e - r * ACH;
    const int i = r / p.rep;
    const int slot = c * ACH + jj;
    float sc = -INFINITY;
    if (visible(p, prefix, i, slot)) {
      const float *qr = Qs + r * d;
      const float *kr = Ks + jj * (d + 1);
      float a = 0.f;
      for (int t = 0; t < d; ++t) a = fmaf(qr[t], kr[t], a);
      sc = a * p.scale;
    }
    P[r * ACH + jj] = sc;
  }
  __syncthreads();

  // chunk-local softmax numerators
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < p.R; r += ATHREADS / 32) {
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
    if (lane == 0) p.part_ml[pbase + r] = make_float2(m, l);
  }
  __syncthreads();

  // Σ p·v
  for (int e = tid; e < p.R * d; e += ATHREADS) {
    const int r = e / d, t = e - r * d;
    const float *pr = P + r * ACH;
    float a = 0.f;
#pragma unroll 8
    for (int jj = 0; jj < ACH; ++jj) a = fmaf(pr[jj], Vs[jj * d + t], a);
    p.part_o[(pbase + r) * d + t] = a;
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
  LBX_CHECK_ARG(a->n * (a->heads / a->kv_heads) <= AMAX_ROWS,
                "n * heads/kv_heads must be <= %d", AMAX_ROWS);
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
  const size_t smem = ((size_t)ACH * (p.d + 1) + (size_t)ACH * p.d + (size_t)p.R * p.d +
                       (size_t)p.R * ACH) * 4;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = allow_max_smem(attn_chunk_kernel);
    if (e != cudaSuccess) return cuda_status(e, "attn smem attribute");
    attr_done = true;
  }
  const bool pdl = a->use_pdl != 0;
  cudaError_t e = launch(attn_chunk_kernel, dim3(p.nchunk, p.kvh), dim3(ATHREADS), smem, stream, pdl, p);
  if (e != cudaSuccess) return cuda_status(e, "attn chunk launch");
  e = launch(attn_combine_kernel, dim3(p.R, p.kvh), dim3(128), 0, stream, pdl, p);
  return cuda_status(e, "attn combine launch");
}
