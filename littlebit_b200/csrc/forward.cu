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
constexpr int FWD_MAX_SEQ = 64;     // independent sequences per multi-sequence step

struct FwdLayout {
  size_t tk, sw, x, q, kk, vv, att, gate, up, pos, rope, lin, attn, lm, total;
  size_t lin_bytes, attn_bytes, lm_bytes;
};

static size_t al(size_t v) { return (v + 255) & ~(size_t)255; }

// n tokens of each of S sequences (S = 1: one sequence)
static FwdLayout fwd_layout(const lbx_model *m, int n, int S = 1) {
  FwdLayout L = {};
  const size_t H = m->hidden, I = m->intermediate, Q = (size_t)m->heads * m->head_dim,
               KV = (size_t)m->kv_heads * m->head_dim;
  const int T = n * S;  // rows of every activation buffer
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al(bytes); return o; };
  // the attention tickets and the linear scratch come first: their bookkeeping
  // words (kept at zero between calls) must sit at the same offset whatever n
  // a call uses
  L.tk = take(attn_ticket_bytes(m->kv_heads, FWD_MAX_SEQ));
  L.sw = take(16);
  size_t lin = 0;
  for (int l = 0; l < m->n_layers; ++l) {
    const lbx_proj *pr = m->layers[l].proj;
    lin = std::max(lin, lbx_linear_workspace_size(pr + 0, 3, T));
    lin = std::max(lin, lbx_linear_workspace_size(pr + 3, 1, T));
    lin = std::max(lin, lbx_linear_workspace_size(pr + 4, 2, T));
    lin = std::max(lin, lbx_linear_workspace_size(pr + 6, 1, T));
  }
  L.lin_bytes = lin;
  L.lin = take(lin);
  L.x = take((size_t)T * H * 4);
  L.q = take((size_t)T * Q * 4);
  L.kk = take((size_t)T * KV * 4);
  L.vv = take((size_t)T * KV * 4);
  L.att = take((size_t)T * Q * 4);
  L.gate = take((size_t)T * I * 4);
  L.up = take((size_t)T * I * 4);
  L.pos = take((size_t)T * 4);
  L.rope = take((size_t)T * m->head_dim * 4);
  lbx_attn_args aa = {};
  aa.n = n;
  aa.n_seq = S;
  aa.heads = m->heads;
  aa.kv_heads = m->kv_heads;
  aa.head_dim = m->head_dim;
  aa.prefix_len = m->max_seq - n;
  L.attn_bytes = attn_partial_bytes(&aa, nullptr);
  L.attn = take(L.attn_bytes);
  L.lm_bytes = lbx_lmhead_workspace_size(T, m->vocab);
  L.lm = take(L.lm_bytes);
  L.total = off;
  return L;
}

__global__ void iota_kernel(int32_t *pos, int start, const int32_t *start_dev, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] = (start_dev ? *start_dev : start) + i;
}

// positions of S sequences of n tokens: row s*n + i at start_seq[s] + i
__global__ void iota_seq_kernel(int32_t *pos, const int32_t *start_seq, int n, int S) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e < n * S) pos[e] = start_seq[e / n] + e % n;
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
// one step of n <= FWD_MAX_TOKENS tokens (checked by the caller); with S > 1,
// n tokens of each of S independent sequences (start_seq: their first slots,
// seq_stride: elements between their caches), rows ordered by sequence
static int forward_chunk(const lbx_model *m, const int64_t *tokens, int32_t n, int32_t start,
                         const int32_t *start_dev, const int32_t *pos, const uint64_t *tree_mask,
                         float *hidden_out, float *logits, int64_t *argmax_out, void *ws,
                         size_t ws_bytes, cudaStream_t stream, int S = 1,
                         const int32_t *start_seq = nullptr, int64_t seq_stride = 0) {
  const FwdLayout L = fwd_layout(m, n, S);
  const int T = n * S;
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
  void *attn_part = w + L.attn;
  unsigned *attn_tk = reinterpret_cast<unsigned *>(w + L.tk);
  float *rope = reinterpret_cast<float *>(w + L.rope);
  void *lm_ws = w + L.lm;
  const int pdl = m->use_pdl;

  int rc = lbx_embed(m->embed, tokens, T, m->hidden, m->vocab, x, stream);
  if (rc) return rc;
  if (!pos) {
    if (S > 1)
      iota_seq_kernel<<<(T + 127) / 128, 128, 0, stream>>>(posb, start_seq, n, S);
    else
      iota_kernel<<<(n + 127) / 128, 128, 0, stream>>>(posb, start, start_dev, n);
    rc = cuda_status(cudaGetLastError(), "iota launch");
    if (rc) return rc;
    pos = posb;
  }
  // RoPE (cos, sin) of this step's positions, once for all layers
  rc = lbx_rope_table(pos, T, m->head_dim, m->rope_theta, rope, stream);
  if (rc) return rc;
  for (int l = 0; l < m->n_layers; ++l) {
    const lbx_layer &ly = m->layers[l];
    // q, k, v from RMSNorm(x)
    lbx_linear_args a = {};
    a.exec = m->exec_mode == LBX_EXEC_KERNELS ? LBX_EXEC_KERNELS : LBX_EXEC_AUTO;
    a.n_proj = 3;
    a.n_tokens = T;
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
    aa.rope_cs = rope;
    aa.k_cache = ly.k_cache;
    aa.v_cache = ly.v_cache;
    aa.out = att;
    if (S > 1) {
      aa.n_seq = S;
      aa.prefix_seq = start_seq;
      aa.cache_seq_stride = seq_stride;
      aa.prefix_dev = nullptr;
    }
    rc = attn_launch(&aa, attn_part, attn_tk, stream);
    if (rc) return rc;
    // x += o(att)
    lbx_linear_args o = {};
    o.exec = a.exec;
    o.n_proj = 1;
    o.n_tokens = T;
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
    gu.y[0] = gate;  // silu(gate), computed once per element (the down prologue multiplies)
    gu.y[1] = up;
    gu.y[2] = nullptr;
    gu.epilogue = LBX_EPI_SILU0;
    rc = lbx_linear_verify(ly.proj + 4, &gu, lin, L.lin_bytes, stream);
    if (rc) return rc;
    // x += down(silu(gate) * up)
    lbx_linear_args dn = o;
    dn.prologue = LBX_PRO_MUL;
    dn.x = gate;
    dn.x2 = up;
    rc = lbx_linear_verify(ly.proj + 6, &dn, lin, L.lin_bytes, stream);
    if (rc) return rc;
  }
  if (hidden_out) {
    rc = lbx_rmsnorm(x, m->final_norm, T, m->hidden, m->rms_eps, hidden_out, stream);
    if (rc) return rc;
  }
  if (logits || argmax_out) {
    rc = lbx_lmhead_argmax(x, m->final_norm, m->rms_eps, T, m->hidden, m->lm_head, m->vocab,
                           logits, argmax_out, lm_ws, L.lm_bytes, pdl, stream);
    if (rc) return rc;
  }
  return LBX_OK;
}
}  // namespace lbx

namespace lbx {
// the whole step as one persistent program (n <= LBX_MAX_TOKENS)
static int forward_program(const lbx_model *m, const int64_t *tokens, int32_t n, int32_t start,
                           const int32_t *start_dev, const int32_t *pos, const uint64_t *tree_mask,
                           float *hidden_out, float *logits, int64_t *argmax_out, void *ws,
                           size_t ws_bytes, cudaStream_t stream) {
  LBX_CHECK_SUP(n <= LBX_MAX_TOKENS, "a program step takes at most %d tokens", LBX_MAX_TOKENS);
  const FwdLayout L = fwd_layout(m, n);
  LBX_CHECK_ARG(ws && ws_bytes >= L.total, "workspace too small (%zu < %zu)", ws_bytes, L.total);
  uint8_t *w = reinterpret_cast<uint8_t *>(ws);
  const int nchunk = (start + n + 63) / 64;
  const int flags = (tree_mask ? 1 : 0) | (pos ? 2 : 0) | (hidden_out ? 4 : 0) | (logits ? 8 : 0) |
                    (argmax_out ? 16 : 0) | (m->use_pdl ? 32 : 0);
  uint64_t key = 0xF0A3Dull;
  key = mix(key, (uintptr_t)m);
  key = mix(key, (uintptr_t)m->layers);
  key = mix(key, (uint64_t)n);
  key = mix(key, (uint64_t)nchunk);
  key = mix(key, (uint64_t)flags);
  key = mix(key, (uintptr_t)ws);
  key = mix(key, (uintptr_t)m->embed);
  key = mix(key, (uintptr_t)m->lm_head);
  key = mix(key, (uintptr_t)m->final_norm);
  for (int l = 0; l < m->n_layers; ++l) {
    const lbx_layer &ly = m->layers[l];
    key = mix(key, (uintptr_t)ly.ln1);
    key = mix(key, (uintptr_t)ly.ln2);
    key = mix(key, (uintptr_t)ly.k_cache);
    key = mix(key, (uintptr_t)ly.v_cache);
    for (int p = 0; p < 7; ++p)
      for (int b = 0; b < ly.proj[p].n_branches; ++b) {
        key = mix(key, (uintptr_t)ly.proj[p].br[b].v_sign);
        key = mix(key, (uintptr_t)ly.proj[p].br[b].u_sign);
        key = mix(key, (uintptr_t)ly.proj[p].br[b].mid);
      }
  }
  float *x = reinterpret_cast<float *>(w + L.x);
  float *q = reinterpret_cast<float *>(w + L.q);
  float *kk = reinterpret_cast<float *>(w + L.kk);
  float *vv = reinterpret_cast<float *>(w + L.vv);
  float *att = reinterpret_cast<float *>(w + L.att);
  float *gate = reinterpret_cast<float *>(w + L.gate);
  float *up = reinterpret_cast<float *>(w + L.up);
  int32_t *posb = reinterpret_cast<int32_t *>(w + L.pos);
  int32_t *sw = reinterpret_cast<int32_t *>(w + L.sw);
  float *rope = reinterpret_cast<float *>(w + L.rope);
  void *lin = w + L.lin;
  void *attn_part = w + L.attn;
  unsigned *attn_tk = reinterpret_cast<unsigned *>(w + L.tk);
  void *lm_ws = w + L.lm;

  std::lock_guard<std::mutex> lk(g_prog_mu);
  Program *P = nullptr;
  auto it = g_progs.find(key);
  if (it != g_progs.end()) {
    P = it->second;
  } else {
    size_t budget = 0;
    int nsm = 0;
    int rc = program_budget(budget, nsm);
    if (rc) return rc;
    ProgBuilder B;
    Phase st = {};
    st.kind = PH_START;
    st.units = n;
    st.io = IO_TOKENS;
    st.st.table = m->embed;
    st.st.hidden = m->hidden;
    st.st.vocab = m->vocab;
    st.st.n = n;
    st.st.d = m->head_dim;
    st.st.theta = m->rope_theta;
    st.st.x = x;
    st.st.pos = posb;
    st.st.start_word = sw;
    st.st.rope = reinterpret_cast<float2 *>(rope);
    B.push(st, 0, 0);
    for (int l = 0; l < m->n_layers; ++l) {
      const lbx_layer &ly = m->layers[l];
      lbx_linear_args a = {};
      a.n_proj = 3;
      a.n_tokens = n;
      a.x_dtype = a.y_dtype = LBX_F32;
      a.prologue = LBX_PRO_RMSNORM;
      a.epilogue = LBX_EPI_STORE;
      a.eps = m->rms_eps;
      a.x = x;
      a.norm_w = ly.ln1;
      a.y[0] = q;
      a.y[1] = kk;
      a.y[2] = vv;
      rc = build_linear(B, ly.proj + 0, a, lin, budget);
      if (rc) return rc;
      lbx_attn_args aa = {};
      aa.n = n;
      aa.heads = m->heads;
      aa.kv_heads = m->kv_heads;
      aa.head_dim = m->head_dim;
      aa.max_seq = m->max_seq;
      aa.prefix_len = start;
      aa.prefix_dev = sw;
      aa.scale = m->attn_scale;
      aa.theta = m->rope_theta;
      aa.q = q;
      aa.k_new = kk;
      aa.v_new = vv;
      aa.pos = posb;
      aa.tree_mask = tree_mask;
      aa.k_cache = ly.k_cache;
      aa.v_cache = ly.v_cache;
      aa.out = att;
      aa.rope_cs = rope;
      Phase ap = {};
      size_t asmem = 0;
      rc = attn_prep(&aa, attn_part, attn_tk, ap.a, asmem);
      if (rc) return rc;
      ap.kind = PH_ATTN;
      ap.units = ap.a.nchunk * ap.a.kvh * ap.a.ngroups;
      ap.io = tree_mask ? IO_TREE : IO_NONE;
      ap.a.tree = nullptr;  // the kernel argument, attached at run time
      B.push(ap, 0, asmem);
      lbx_linear_args o = {};
      o.n_proj = 1;
      o.n_tokens = n;
      o.x_dtype = o.y_dtype = LBX_F32;
      o.prologue = LBX_PRO_NONE;
      o.epilogue = LBX_EPI_ADD;
      o.x = att;
      o.y[0] = x;
      rc = build_linear(B, ly.proj + 3, o, lin, budget);
      if (rc) return rc;
      lbx_linear_args gu = a;
      gu.n_proj = 2;
      gu.norm_w = ly.ln2;
      gu.y[0] = gate;  // silu(gate)
      gu.y[1] = up;
      gu.y[2] = nullptr;
      gu.epilogue = LBX_EPI_SILU0;
      rc = build_linear(B, ly.proj + 4, gu, lin, budget);
      if (rc) return rc;
      lbx_linear_args dn = o;
      dn.prologue = LBX_PRO_MUL;
      dn.x = gate;
      dn.x2 = up;
      rc = build_linear(B, ly.proj + 6, dn, lin, budget);
      if (rc) return rc;
    }
    if (hidden_out) {
      Phase nm = {};
      nm.kind = PH_NORM;
      nm.units = n;
      nm.io = IO_HIDDEN;
      nm.nm.x = x;
      nm.nm.w = m->final_norm;
      nm.nm.hidden = m->hidden;
      nm.nm.eps = m->rms_eps;
      B.push(nm, 0, 0);
    }
    if (logits || argmax_out) {
      LBX_CHECK_SUP(m->hidden % 256 == 0, "hidden must be a multiple of 256");
      // one pass width for the whole program (rows past a pass's tokens are
      // zero and every token's sum is computed the same way at any width)
      const int NT = n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8;
      LBX_CHECK_SUP((size_t)NT * m->hidden * 4 <= 128 * 1024, "hidden too wide for a program lm_head pass");
      B.lmnt = NT;
      const int per = NT;
      for (int t0 = 0; t0 < n; t0 += per) {
        const int nt = std::min(per, n - t0);
        Phase lp = {};
        lp.kind = PH_LM;
        lp.units = nsm;
        lp.ncb = NT;
        lp.io = IO_LOGITS;
        lp.io_off = (int64_t)t0 * m->vocab;
        lp.l.x = x + (int64_t)t0 * m->hidden;
        lp.l.norm_w = m->final_norm;
        lp.l.eps = m->rms_eps;
        lp.l.n = nt;
        lp.l.hidden = m->hidden;
        lp.l.vocab = m->vocab;
        lp.l.nblocks = nsm;
        lp.l.w = m->lm_head;
        lp.l.best = reinterpret_cast<unsigned long long *>(lm_ws);
        B.push(lp, 0, (size_t)NT * m->hidden * 4);
        if (argmax_out) {
          Phase am = {};
          am.kind = PH_ARGMAX;
          am.units = 1;
          am.io = IO_ARGMAX;
          am.io_off = t0;
          am.am.best = reinterpret_cast<const unsigned long long *>(lm_ws);
          am.am.nblocks = nsm;
          am.am.n = nt;
          B.push(am, 0, 0);
        }
      }
    }
    LBX_CHECK_SUP(((B.smax + 255) & ~(size_t)255) + B.wmax <= budget,
                  "the step program needs %zu bytes of shared memory (max %zu)",
                  ((B.smax + 255) & ~(size_t)255) + B.wmax, budget);
    rc = finish_program(key, B, stream, P);
    if (rc) return rc;
  }
  ProgIo io = {};
  io.tokens = tokens;
  io.start = start;
  io.start_dev = start_dev;
  io.pos = pos;
  io.tree = tree_mask;
  io.hidden = hidden_out;
  io.logits = logits;
  io.argmax = argmax_out;
  return launch_program(P, gridbar_of(lin), io, stream);
}
}  // namespace lbx

extern "C" size_t lbx_forward_multi_workspace_size(const lbx_model *m, int32_t n_seq, int32_t n_tokens) {
  if (!m || !m->layers || n_seq < 1 || n_seq > lbx::FWD_MAX_SEQ || n_tokens < 1 ||
      n_tokens > lbx::FWD_MAX_TOKENS)
    return 0;
  return lbx::fwd_layout(m, n_tokens, n_seq).total;
}

extern "C" int lbx_forward_multi(const lbx_model *m, const int64_t *tokens, int32_t n_seq, int32_t n,
                                 int32_t max_start, const int32_t *start_seq, int64_t cache_seq_stride,
                                 const int32_t *pos, const uint64_t *tree_mask, float *hidden_out,
                                 float *logits, int64_t *argmax_out, void *ws, size_t ws_bytes,
                                 cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(m && m->layers, "model is NULL");
  LBX_CHECK_ARG(n_seq >= 1 && n_seq <= FWD_MAX_SEQ, "n_seq must be in [1,%d]", FWD_MAX_SEQ);
  LBX_CHECK_ARG(n >= 1 && n <= FWD_MAX_TOKENS && tokens, "n must be in [1,%d]", FWD_MAX_TOKENS);
  LBX_CHECK_ARG(start_seq, "start_seq is NULL");
  LBX_CHECK_ARG(max_start >= 0 && max_start + n <= m->max_seq, "max_start + n exceeds max_seq");
  LBX_CHECK_ARG(cache_seq_stride >= (int64_t)m->kv_heads * m->max_seq * m->head_dim,
                "cache_seq_stride is smaller than one sequence's cache");
  LBX_CHECK_ARG(m->heads % m->kv_heads == 0, "heads must be a multiple of kv_heads");
  LBX_CHECK_ARG(m->embed && m->final_norm, "embed/final_norm required");
  LBX_CHECK_ARG(!(logits || argmax_out) || m->lm_head, "lm_head required for logits/argmax");
  LBX_CHECK_SUP(m->exec_mode != LBX_EXEC_PROGRAM, "multi-sequence steps run on the kernel path");
  const size_t need = fwd_layout(m, n, n_seq).total;
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  return forward_chunk(m, tokens, n, max_start, nullptr, pos, tree_mask, hidden_out, logits, argmax_out, ws,
                       ws_bytes, stream, n_seq, start_seq, cache_seq_stride);
}

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
  LBX_CHECK_ARG(m->exec_mode >= LBX_EXEC_AUTO && m->exec_mode <= LBX_EXEC_PROGRAM, "bad exec_mode");
  if (m->exec_mode == LBX_EXEC_PROGRAM) {
    // programs of up to LBX_MAX_TOKENS tokens; a longer causal run is a sequence of them
    LBX_CHECK_SUP(n <= LBX_MAX_TOKENS || (!tree_mask && !start_dev),
                  "a program step with a tree mask or a device start takes at most %d tokens", LBX_MAX_TOKENS);
    for (int a = 0; a < n; a += LBX_MAX_TOKENS) {
      const int c = n - a < LBX_MAX_TOKENS ? n - a : LBX_MAX_TOKENS;
      const int rc = forward_program(m, tokens + a, c, start + a, start_dev, pos ? pos + a : nullptr, tree_mask,
                                     hidden_out ? hidden_out + (int64_t)a * m->hidden : nullptr,
                                     logits ? logits + (int64_t)a * m->vocab : nullptr,
                                     argmax_out ? argmax_out + a : nullptr, ws, ws_bytes, stream);
      if (rc) return rc;
    }
    return LBX_OK;
  }
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
