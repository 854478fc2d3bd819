// Whole decoder step: embedding -> L x (RMSNorm+q/k/v, attention, o + residual,
// RMSNorm+gate/up, SiLU·mul+down + residual) -> final RMSNorm [-> lm_head+argmax].
//
// Native replacement of full_forward (patches/littlebit_cpu_optimized.cpp:
// 1522-1840), full_forward_batch (cpp:1846-2079) and generate_token
// (cpp:2256-2317).  Layer order and residual structure follow cpp:1627-1835;
// the projections take their inputs as the reference's fused groups do
// (q/k/v share one normalised input, cpp:1700-1722; gate/up share one,
// cpp:1777-1798).  Differences from the CPU path, by design: rotary
// embedding is applied (the CPU path has none), the KV cache is bf16, the
// activations are not int8-quantised, and n tokens are processed together
// (one packed-weight read per step instead of one per token).
//
// Every kernel is launched on the caller's stream with programmatic dependent
// launch when m->use_pdl, so the sequence captures into one CUDA graph.

#include "common.cuh"

namespace lbx {

constexpr int FWD_MAX_TOKENS = 64;  // tokens per step (attention and tree-mask width)

struct FwdLayout {
  size_t x, q, kk, vv, att, gate, up, pos, lin, attn, lm, total;
  size_t lin_bytes, attn_bytes, lm_bytes;
};

static size_t al(size_t v) { return (v + 255) & ~(size_t)255; }

static FwdLayout fwd_layout(const lbx_model *m, int n) {
  FwdLayout L = {};
  const size_t H = m->hidden, I = m->intermediate, Q = (size_t)m->heads * m->head_dim,
               KV = (size_t)m->kv_heads * m->head_dim;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al(bytes); return o; };
  // the linear scratch comes first: its bookkeeping words (kept at zero between
  // calls) must sit at the same offset whatever n a call uses
  size_t lin = 0;
  for (int l = 0; l < m->n_layers; ++l) {
    const lbx_proj *pr = m->layers[l].proj;
    lin = std::max(lin, lbx_linear_workspace_size(pr + 0, 3, n));
    lin = std::max(lin, lbx_linear_workspace_size(pr + 3, 1, n));
    lin = std::max(lin, lbx_linear_workspace_size(pr + 4, 2, n));
    lin = std::max(lin, lbx_linear_workspace_size(pr + 6, 1, n));
  }
  L.lin_bytes = lin;
  L.lin = take(lin);
  L.x = take((size_t)n * H * 4);
  L.q = take((size_t)n * Q * 4);
  L.kk = take((size_t)n * KV * 4);
  L.vv = take((size_t)n * KV * 4);
  L.att = take((size_t)n * Q * 4);
  L.gate = take((size_t)n * I * 4);
  L.up = take((size_t)n * I * 4);
  L.pos = take((size_t)n * 4);
  lbx_attn_args aa = {};
  aa.n = n;
  aa.heads = m->heads;
  aa.kv_heads = m->kv_heads;
  aa.head_dim = m->head_dim;
  aa.prefix_len = m->max_seq - n;
  L.attn_bytes = lbx_attn_workspace_size(&aa);
  L.attn = take(L.attn_bytes);
  L.lm_bytes = lbx_lmhead_workspace_size(n, m->vocab);
  L.lm = take(L.lm_bytes);
  L.total = off;
  return L;
}

__global__ void iota_kernel(int32_t *pos, int start, const int32_t *start_dev, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] = (start_dev ? *start_dev : start) + i;
}

// every (layer, kv head, k|v) row block: stage all source rows, then write
__global__ void kv_move_kernel(uint16_t *const *kc, uint16_t *const *vc, int kvh, int max_seq, int d,
                               const int32_t *src, const int32_t *dst, int n) {
  extern __shared__ uint16_t rows[];  // n x d
  const int layer = blockIdx.x / (2 * kvh);
  const int rem = blockIdx.x - layer * 2 * kvh;
  const int h = rem >> 1;
  uint16_t *base = ((rem & 1) ? vc[layer] : kc[layer]) + (int64_t)h * max_seq * d;
  for (int e = threadIdx.x; e < n * d; e += blockDim.x) {
    const int i = e / d, t = e - i * d;
    rows[e] = base[(int64_t)src[i] * d + t];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n * d; e += blockDim.x) {
    const int i = e / d, t = e - i * d;
    base[(int64_t)dst[i] * d + t] = rows[e];
  }
}

}  // namespace lbx

extern "C" size_t lbx_forward_workspace_size(const lbx_model *m, int32_t n_tokens) {
  if (!m || !m->layers || n_tokens < 1) return 0;
  return lbx::fwd_layout(m, n_tokens < lbx::FWD_MAX_TOKENS ? n_tokens : lbx::FWD_MAX_TOKENS).total;
}

extern "C" int lbx_kv_move(uint16_t *const *k_caches, uint16_t *const *v_caches, int32_t n_layers,
                           int32_t kv_heads, int32_t max_seq, int32_t head_dim, const int32_t *src,
                           const int32_t *dst, int32_t n, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(n >= 0 && n <= 64, "n must be in [0,64]");
  if (n == 0) return LBX_OK;
  LBX_CHECK_ARG(k_caches && v_caches && src && dst, "NULL pointer");
  LBX_CHECK_ARG(n_layers > 0 && kv_heads > 0 && head_dim > 0 && max_seq > 0, "bad shape");
  const size_t smem = (size_t)n * head_dim * 2;
  LBX_CHECK_SUP(smem <= 48 * 1024, "too many rows to move at once");
  kv_move_kernel<<<n_layers * 2 * kv_heads, 256, smem, stream>>>(k_caches, v_caches, kv_heads, max_seq,
                                                                  head_dim, src, dst, n);
  return cuda_status(cudaGetLastError(), "kv_move launch");
}

namespace lbx {
// one step of n <= FWD_MAX_TOKENS tokens (checked by the caller)
static int forward_chunk(const lbx_model *m, const int64_t *tokens, int32_t n, int32_t start,
                         const int32_t *start_dev, const int32_t *pos, const uint64_t *tree_mask,
                         float *hidden_out, float *logits, int64_t *argmax_out, void *ws,
                         size_t ws_bytes, cudaStream_t stream) {
  const FwdLayout L = fwd_layout(m, n);
  LBX_CHECK_ARG(ws && ws_bytes >= L.total, "workspace too small (%zu < %zu)", ws_bytes, L.total);
  uint8_t *w = reinterpret_cast<uint8_t *>(ws);
  float *x = reinterpret_cast<float *>(w + L.x);
  float *q = reinterpret_cast<float *>(w + L.q);
  float *kk = reinterpret_cast<float *>(w + L.kk);
  float *vv = reinterpret_cast<float *>(w + L.vv);
  float *att = reinterpret_cast<float *>(w + L.att);
  float *gate = reinterpret_cast<float *>(w + L.gate);
  float *up = reinterpret_cast<float *>(w + L.up);
  int32_t *posb = reinterpret_cast<int32_t *>(w + L.pos);
  void *lin = w + L.lin;
  void *attn_ws = w + L.attn;
  void *lm_ws = w + L.lm;
  const int pdl = m->use_pdl;

  int rc = lbx_embed(m->embed, tokens, n, m->hidden, m->vocab, x, stream);
  if (rc) return rc;
  if (!pos) {
    iota_kernel<<<(n + 127) / 128, 128, 0, stream>>>(posb, start, start_dev, n);
    rc = cuda_status(cudaGetLastError(), "iota launch");
    if (rc) return rc;
    pos = posb;
  }
  for (int l = 0; l < m->n_layers; ++l) {
    const lbx_layer &ly = m->layers[l];
    // q, k, v from RMSNorm(x)
    lbx_linear_args a = {};
    a.n_proj = 3;
    a.n_tokens = n;
    a.x_dtype = LBX_F32;
    a.y_dtype = LBX_F32;
    a.prologue = LBX_PRO_RMSNORM;
    a.epilogue = LBX_EPI_STORE;
    a.eps = m->rms_eps;
    a.use_pdl = pdl;
    a.x = x;
    a.norm_w = ly.ln1;
    a.y[0] = q;
    a.y[1] = kk;
    a.y[2] = vv;
    rc = lbx_linear_verify(ly.proj + 0, &a, lin, L.lin_bytes, stream);
    if (rc) return rc;
    // attention with RoPE and KV write
    lbx_attn_args aa = {};
    aa.n = n;
    aa.heads = m->heads;
    aa.kv_heads = m->kv_heads;
    aa.head_dim = m->head_dim;
    aa.max_seq = m->max_seq;
    aa.prefix_len = start;
    aa.prefix_dev = start_dev;
    aa.scale = m->attn_scale;
    aa.theta = m->rope_theta;
    aa.use_pdl = pdl;
    aa.q = q;
    aa.k_new = kk;
    aa.v_new = vv;
    aa.pos = pos;
    aa.tree_mask = tree_mask;
    aa.k_cache = ly.k_cache;
    aa.v_cache = ly.v_cache;
    aa.out = att;
    rc = lbx_attn_decode(&aa, attn_ws, L.attn_bytes, stream);
    if (rc) return rc;
    // x += o(att)
    lbx_linear_args o = {};
    o.n_proj = 1;
    o.n_tokens = n;
    o.x_dtype = LBX_F32;
    o.y_dtype = LBX_F32;
    o.prologue = LBX_PRO_NONE;
    o.epilogue = LBX_EPI_ADD;
    o.use_pdl = pdl;
    o.x = att;
    o.y[0] = x;
    rc = lbx_linear_verify(ly.proj + 3, &o, lin, L.lin_bytes, stream);
    if (rc) return rc;
    // gate, up from RMSNorm(x)
    lbx_linear_args gu = a;
    gu.n_proj = 2;
    gu.norm_w = ly.ln2;
    gu.y[0] = gate;
    gu.y[1] = up;
    gu.y[2] = nullptr;
    rc = lbx_linear_verify(ly.proj + 4, &gu, lin, L.lin_bytes, stream);
    if (rc) return rc;
    // x += down(silu(gate) * up)
    lbx_linear_args dn = o;
    dn.prologue = LBX_PRO_SILU_MUL;
    dn.x = gate;
    dn.x2 = up;
    rc = lbx_linear_verify(ly.proj + 6, &dn, lin, L.lin_bytes, stream);
    if (rc) return rc;
  }
  if (hidden_out) {
    rc = lbx_rmsnorm(x, m->final_norm, n, m->hidden, m->rms_eps, hidden_out, stream);
    if (rc) return rc;
  }
  if (logits || argmax_out) {
    rc = lbx_lmhead_argmax(x, m->final_norm, m->rms_eps, n, m->hidden, m->lm_head, m->vocab,
                           logits, argmax_out, lm_ws, L.lm_bytes, pdl, stream);
    if (rc) return rc;
  }
  return LBX_OK;
}
}  // namespace lbx

extern "C" int lbx_forward(const lbx_model *m, const int64_t *tokens, int32_t n, int32_t start,
                           const int32_t *start_dev, const int32_t *pos, const uint64_t *tree_mask,
                           float *hidden_out, float *logits, int64_t *argmax_out, void *ws,
                           size_t ws_bytes, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(m && m->layers, "model is NULL");
  LBX_CHECK_ARG(n >= 1 && tokens, "need n >= 1 tokens");
  LBX_CHECK_ARG(start >= 0 && start + n <= m->max_seq, "start + n exceeds max_seq");
  LBX_CHECK_ARG(m->heads % m->kv_heads == 0, "heads must be a multiple of kv_heads");
  LBX_CHECK_ARG(m->embed && m->final_norm, "embed/final_norm required");
  LBX_CHECK_ARG(!(logits || argmax_out) || m->lm_head, "lm_head required for logits/argmax");
  LBX_CHECK_ARG(n <= FWD_MAX_TOKENS || (!tree_mask && !start_dev),
                "more than %d tokens only as a causal run at a host-given start", FWD_MAX_TOKENS);
  const size_t need = fwd_layout(m, n < FWD_MAX_TOKENS ? n : FWD_MAX_TOKENS).total;
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  // a long causal run is a sequence of steps of FWD_MAX_TOKENS tokens
  for (int a = 0; a < n; a += FWD_MAX_TOKENS) {
    const int c = n - a < FWD_MAX_TOKENS ? n - a : FWD_MAX_TOKENS;
    const int rc = forward_chunk(m, tokens + a, c, start + a, start_dev, pos ? pos + a : nullptr, tree_mask,
                                 hidden_out ? hidden_out + (int64_t)a * m->hidden : nullptr,
                                 logits ? logits + (int64_t)a * m->vocab : nullptr,
                                 argmax_out ? argmax_out + a : nullptr, ws, ws_bytes, stream);
    if (rc) return rc;
  }
  return LBX_OK;
}
