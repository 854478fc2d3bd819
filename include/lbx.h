/*
 * lbx.h — C ABI of the B200 (sm_100a) LittleBit kernels.
 *
 * Every pointer is a caller-owned DEVICE buffer unless the comment says "host".
 * Every call is stream-ordered on the given cudaStream_t, performs no host
 * synchronisation and no device allocation, and returns an int status:
 *   LBX_OK (0), LBX_EINVAL (1, bad argument/shape), LBX_EUNSUPPORTED (2),
 *   LBX_ECUDA (3, a CUDA launch error; text in lbx_last_error).
 * No C++ exception crosses this boundary.  The reference's native op library
 * (patches/littlebit_cpu_optimized.cpp, TORCH_LIBRARY at :2321-2377) raised
 * TORCH_CHECK errors instead; the Python layer turns a non-zero status into a
 * RuntimeError carrying lbx_last_error(), so callers see the same exception type.
 *
 * Bit-packing contract (quantization/utils/binary_packer.py:4-50): a {-1,+1}
 * matrix [R, C] is stored as int32 words [R, ceil(C/32)], bit j of word w is
 * column 32*w + j (LSB first), bit 1 <=> -1, pad columns are +1 (bit 0).
 */
#ifndef LBX_H
#define LBX_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LBX_OK 0
#define LBX_EINVAL 1
#define LBX_EUNSUPPORTED 2
#define LBX_ECUDA 3

/* element types for activations */
#define LBX_F32 0
#define LBX_BF16 1

/* largest token batch one linear launch handles; larger batches are split
 * by the host into independent launches (tokens never interact in a linear). */
#define LBX_MAX_TOKENS 16
/* largest number of projections sharing one input in a single launch */
#define LBX_MAX_PROJ 3

/* One LittleBit branch: y_b = u1 ⊙ U_sign·(mid ⊙ V_sign·(v2 ⊙ x)).
 * Reference: quantization/modules/littlebit.py:114-121 (_compute_forward),
 * runtime keys convert_hf_to_runtime.py:47-57 (u_sign_rt, v_sign_rt, u1, v2,
 * mid = v1*u2). */
typedef struct lbx_branch {
  const int32_t *v_sign; /* [rank, ceil(in/32)]; NULL => reuse branch 0's V-stage */
  const float *v2;       /* [in]   (NULL when v_sign is NULL)                     */
  const float *mid;      /* [rank] v1*u2                                          */
  const int32_t *u_sign; /* [out, ceil(rank/32)]                                  */
  const float *u1;       /* [out]                                                 */
  int32_t rank;
} lbx_branch;

/* One LittleBitLinear (littlebit.py:95-112): main branch, optional residual
 * branch (littlebit.py:104-107, or the shared-factor residual of
 * littlespec_ref/littlebit_itq_spec.py:298-309 when br[1].v_sign == NULL),
 * optional bias. */
typedef struct lbx_proj {
  int32_t in_features;
  int32_t out_features;
  int32_t n_branches; /* 1 or 2 */
  int32_t _pad;
  lbx_branch br[2];
  const float *bias; /* [out] or NULL */
} lbx_proj;

/* Input transform applied while the kernel stages x (fused, no extra pass). */
#define LBX_PRO_NONE 0
#define LBX_PRO_RMSNORM 1 /* x <- x * rsqrt(mean(x^2)+eps) * norm_w              */
#define LBX_PRO_SILU_MUL 2 /* x <- silu(x) * x2   (cpp:1117-1170 silu_mul)        */
#define LBX_PRO_MUL 3      /* x <- x * x2 (x already silu'd by LBX_EPI_SILU0)     */

/* Output mode. */
#define LBX_EPI_STORE 0 /* y  = linear(x)                                        */
#define LBX_EPI_ADD 1   /* y += linear(x)   (residual stream update, fp32 only)  */
#define LBX_EPI_SILU0 2 /* y[0] = silu(linear_0(x)), other projections store:
                         * a gate/up call whose gate feeds an LBX_PRO_MUL down
                         * projection computes silu once per element instead of
                         * in every CTA of the down projection (with fp32 y the
                         * down projection's bits are those of LBX_PRO_SILU_MUL) */

typedef struct lbx_linear_args {
  int32_t n_proj;      /* 1..LBX_MAX_PROJ projections sharing the input x      */
  int32_t n_tokens;    /* k tokens (rows of x)                                 */
  int32_t x_dtype;     /* LBX_F32 / LBX_BF16                                   */
  int32_t y_dtype;     /* LBX_F32 / LBX_BF16                                   */
  int32_t prologue;    /* LBX_PRO_*                                            */
  int32_t epilogue;    /* LBX_EPI_*                                            */
  float eps;           /* RMSNorm epsilon                                      */
  int32_t use_pdl;     /* launch with programmatic dependent launch            */
  const void *x;       /* [k, in] row-major                                    */
  const void *x2;      /* [k, in] second input of LBX_PRO_SILU_MUL             */
  const float *norm_w; /* [in] RMSNorm weight of LBX_PRO_RMSNORM               */
  void *y[LBX_MAX_PROJ];   /* per projection [k, out] row-major                */
  int64_t y_ld[LBX_MAX_PROJ]; /* row stride (elements) of each y; 0 => out    */
  int32_t exec;        /* LBX_EXEC_AUTO: one cluster launch when the call fits
                        * it, else the two stage grids; LBX_EXEC_KERNELS: the
                        * two stage grids; LBX_EXEC_CLUSTER: the cluster launch
                        * or LBX_EUNSUPPORTED; LBX_EXEC_KERNELS_ONE_CTA_V,
                        * LBX_EXEC_TC, LBX_EXEC_NO_TC (see below).  All give
                        * the same bits.                                      */
  int32_t _pad;
} lbx_linear_args;

/* Bytes of device scratch one lbx_linear / lbx_linear_verify call needs on
 * any executor (the two stage grids need less; LBX_EXEC_CLUSTER needs this).
 * The workspace must be zero-filled once when it is allocated: its header
 * holds a few bookkeeping words (the cluster executor's tickets) that every
 * call expects at zero and leaves at zero when it completes.  Calls sharing a
 * workspace must be ordered on one stream. */
size_t lbx_linear_workspace_size(const lbx_proj *projs /* host */, int32_t n_proj,
                                 int32_t n_tokens);

/* Batch-1 LittleBitLinear.  Replaces littlebit_cpu_ops::littlebit_linear
 * (patches/littlebit_cpu_optimized.cpp:598-701) and the inline projection
 * lb_linear_i2_inline (cpp:1320-1369); fp32-accurate, no int8 activation loss. */
int lbx_linear(const lbx_proj *projs /* host */, const lbx_linear_args *a /* host */,
               void *ws, size_t ws_bytes, cudaStream_t stream);

/* Batch-k verify LittleBitLinear: one packed-weight read for all k tokens.
 * Each token's result is bit-identical to lbx_linear on that token alone.
 * Replaces the serial per-token projection loop of full_forward_batch
 * (cpp:1942-1946).  Same arguments as lbx_linear with a->n_tokens = k. */
int lbx_linear_verify(const lbx_proj *projs, const lbx_linear_args *a, void *ws,
                      size_t ws_bytes, cudaStream_t stream);

/* lbx_linear_verify for callers that cannot allocate device memory.  No
 * counterpart in the reference (its CPU op allocated its own scratch): this
 * entry point is for code that must not call cudaMalloc or hand the library a
 * buffer — e.g. a host application whose own allocator owns every device
 * allocation and cannot lend one, or a service that sets up all device
 * memory at start-up and may not allocate while serving.  The scratch is a fixed module-level device array of
 * lbx_linear_noalloc_max_bytes() bytes (1 MiB) that every GPU loading the
 * library holds until exit; calls needing more scratch than that are rejected
 * with LBX_EUNSUPPORTED.  No cudaMalloc, cudaFree or allocating library
 * routine is called.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress), so make that first call before any stream
 * capture.  All calls share the array and it keeps the previous call's
 * contents: each call clears the words that must start at zero, and calls
 * whose work overlaps on the GPU (different streams, or different host
 * threads on one device) race on it — order them on one stream. */
int lbx_linear_noalloc(const lbx_proj *projs, const lbx_linear_args *a, cudaStream_t stream);
size_t lbx_linear_noalloc_max_bytes(void);

/* ---- bit packing (quantization/utils/binary_packer.py) ------------------ */
/* binary_packer (binary_packer.py:4-50): int8 ±1 [rows, cols] -> int32 words.
 * Entries other than -1/+1 set *bad_count (device int, may be NULL). */
int lbx_pack_signs(const int8_t *signs, int64_t rows, int64_t cols, int32_t *packed,
                   int32_t *bad_count, cudaStream_t stream);
/* binary_unpacker (binary_packer.py:53-97): int32 words -> int8 ±1. */
int lbx_unpack_signs(const int32_t *packed, int64_t rows, int64_t cols, int8_t *signs,
                     cudaStream_t stream);
/* pack_weights (littlebit.py:307-320): sign(w) with 0 -> +1 (functions/binary.py:7-10),
 * then binary_packer, straight from a float/bf16 latent factor. */
int lbx_pack_signs_from_float(const void *w, int32_t w_dtype, int64_t rows, int64_t cols,
                              int32_t *packed, cudaStream_t stream);

/* ---- decoder pieces ------------------------------------------------------ */
/* embedding_lookup (cpp:973-996): out[i,:] = float(table[ids[i],:]); bf16 table. */
int lbx_embed(const uint16_t *table_bf16, const int64_t *ids, int32_t n, int32_t hidden,
              int32_t vocab, float *out, cudaStream_t stream);
/* rms_norm (cpp:998-1052), n rows. out may alias x. */
int lbx_rmsnorm(const float *x, const float *w, int32_t n, int32_t hidden, float eps,
                float *out, cudaStream_t stream);
/* silu_mul (cpp:1117-1170): out = g*sigmoid(g)*u, exact expf. */
int lbx_silu_mul(const float *g, const float *u, int64_t n, float *out, cudaStream_t stream);
/* HF Llama rotary embedding (rotate_half convention), in place on
 * x [n, heads, head_dim] at positions pos[n]. Missing in the reference CPU
 * path (it applies none); the GPU/HF path applies it. */
int lbx_rope(float *x, const int32_t *pos, int32_t n, int32_t heads, int32_t head_dim,
             float theta, cudaStream_t stream);

/* Decode attention over a bf16 KV cache with fused RoPE and KV write.
 * Replaces fused_attention (cpp:1172-1301) and the causal loop of
 * full_forward_batch (cpp:1963-2021).  q/k_new/v_new are the raw projection
 * outputs [n, heads*d] / [n, kv_heads*d] fp32 (row strides q_ld / kv_ld).
 * New token i is rotated with position pos[i] and written to cache slot
 * prefix_len + i.  Query i sees cache slots [0, prefix_len) plus the new slots
 * prefix_len + j with bit j of tree_mask[i] set (its tree ancestors and
 * itself) or, when tree_mask == NULL, j <= i (causal).  GQA: query head h
 * reads kv head h / (heads / kv_heads) (cpp:1238).  Caches are
 * [kv_heads, max_seq, head_dim] bf16; head_dim a multiple of 4, <= 128; n <= 64.
 * A query's keys are the cached prefix, then its visible new tokens in index
 * order (a tree's ancestors precede their descendants, as in
 * generate_tree_buffers); the arithmetic follows that order, so a tree node's
 * output is bit-identical to decoding its path as a causal sequence.
 * theta <= 0 applies no rotation (the reference CPU runtime applies none). */
typedef struct lbx_attn_args {
  int32_t n;
  int32_t heads, kv_heads, head_dim, max_seq;
  int32_t prefix_len;         /* cached slots; with prefix_dev: an upper bound */
  float scale, theta;
  int32_t use_pdl;
  const int32_t *prefix_dev;  /* device copy of the cached-slot count, or NULL:
                                 lets one CUDA graph replay at any position */
  const float *q; int64_t q_ld;
  const float *k_new; const float *v_new; int64_t kv_ld;
  const int32_t *pos;        /* [n] rotary positions */
  const uint64_t *tree_mask; /* [n] or NULL          */
  uint16_t *k_cache; uint16_t *v_cache;
  float *out;                /* [n, heads*d]         */
  const float *rope_cs;      /* [n][head_dim/2] (cos, sin) pairs from
                                lbx_rope_table for pos[], or NULL: computed
                                in the kernel (same values)               */
  /* Independent sequences in one launch (0 or 1: one sequence, as above).
   * With n_seq = S > 1, n is the token count of EACH sequence and the rows
   * of q, k_new, v_new, pos, tree_mask, rope_cs and out hold S*n tokens,
   * sequence by sequence; sequence s's caches start cache_seq_stride
   * elements after sequence s-1's (k_cache / v_cache are sequence 0's), and
   * its cached-slot count is prefix_seq[s] (device; prefix_len bounds them
   * all).  Each sequence's outputs are bit-identical to a launch of its
   * own.  S <= LBX_ATTN_MAX_SEQ. */
  int32_t n_seq;
  int32_t _pad;
  int64_t cache_seq_stride;
  const int32_t *prefix_seq;
} lbx_attn_args;
#define LBX_ATTN_MAX_SEQ 256
/* Workspace: zero-filled once at allocation (it holds self-resetting tickets). */
size_t lbx_attn_workspace_size(const lbx_attn_args *a);
int lbx_attn_decode(const lbx_attn_args *a, void *ws, size_t ws_bytes, cudaStream_t stream);
/* (cos, sin) of pos[i] * theta^(-2j/head_dim), j < head_dim/2, evaluated in
 * double and rounded to float: out [n][head_dim/2][2].  theta <= 0 gives (1, 0). */
int lbx_rope_table(const int32_t *pos, int32_t n, int32_t head_dim, float theta, float *out,
                   cudaStream_t stream);

/* Fused final RMSNorm + lm_head (bf16 [vocab, hidden]) + argmax.
 * Replaces dense_gemv_f32 (cpp:1054-1115) + the argmax of generate_token
 * (cpp:2306-2314).  x [n, hidden] fp32 is the pre-norm hidden state when
 * norm_w != NULL.  logits [n, vocab] fp32 may be NULL; argmax_out [n] int64
 * takes the lowest index among equal maxima (torch.argmax order). */
size_t lbx_lmhead_workspace_size(int32_t n, int32_t vocab);
int lbx_lmhead_argmax(const float *x, const float *norm_w, float eps, int32_t n,
                      int32_t hidden, const uint16_t *w_bf16, int32_t vocab, float *logits,
                      int64_t *argmax_out, void *ws, size_t ws_bytes, int32_t use_pdl,
                      cudaStream_t stream);

/* Greedy chain acceptance (speculative_decoding.py:315-330, 356-363):
 * draft[k], target_argmax[k+1] -> out[0] = accepted count a, out[1] = the
 * token appended after them (target_argmax[a]). */
int lbx_accept_greedy_chain(const int64_t *draft, const int64_t *target_argmax, int32_t k,
                            int64_t *out, cudaStream_t stream);
/* Greedy tree acceptance (tree_utils.py:182-214 on the gather of
 * speculative_decoding.py:541-554): cand [L, D+1] token ids (-1 pad),
 * node_argmax [T] argmax of each tree node's logits, retrieve [L, D+1] node
 * indices (-1 pad) -> out[0] = best leaf row, out[1] = accept length,
 * out[2] = bonus token, out[3..3+D) = accepted node indices. */
int lbx_accept_greedy_tree(const int64_t *cand, const int64_t *node_argmax,
                           const int64_t *retrieve, int32_t L, int32_t D1, int64_t *out,
                           cudaStream_t stream);

/* Chain of single-projection LittleBit layers as one persistent program:
 * acts[i+1] = layer_i(acts[i]) for i < n_layers, n_tokens rows each, all
 * activations of one dtype (LBX_F32 / LBX_BF16).  Same numerics as calling
 * lbx_linear layer by layer.  The workspace (zero-filled once) is shared by
 * the layers; the program is built on the first call with these pointers,
 * outside stream capture. */
size_t lbx_linear_chain_workspace_size(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens);
int lbx_linear_chain(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens, int32_t dtype,
                     void *const *acts, void *ws, size_t ws_bytes, cudaStream_t stream);

/* ---- fused layer chain --------------------------------------------------
 * No reference counterpart (the reference runs one layer per op call): a chain
 * of single-projection layers, acts[i+1] = layer_i(acts[i]) as in
 * lbx_linear_chain, as n_layers + 1 launches instead of two per layer.  Launch
 * i runs layer i's U-stage and, from the outputs it has just formed, layer
 * i+1's V-stage partial sums (one thread-block cluster of 6 CTAs per 256
 * output rows; the first launch forms layer 0's partials from acts[0]).
 * Every output is bit-identical to calling lbx_linear layer by layer.
 * Requirements: in/out features multiples of 256 (in <= 8192), no prologue,
 * store epilogue, 1-2 branches of at most 30 quantisation groups (128 ranks)
 * together, 1..8 tokens, one activation dtype (LBX_F32 / LBX_BF16).  A call
 * of 2..8 tokens runs as two chains of ceil(k/2) and floor(k/2) tokens at
 * once, the second on a helper stream the library keeps per device, forked
 * from `stream` and joined back to it with events (so the call may be
 * captured in a CUDA graph); calls on one device then come from one host
 * thread at a time.
 * lbx_chain_prepare writes, once, a copy of the chain's sign words laid out
 * so that each CTA's share of a layer is contiguous (blob of
 * lbx_chain_prepare_size bytes, 16-byte aligned); the layers' scale vectors
 * are read from the descriptors.  The workspace (any contents) holds the
 * partial sums between launches; calls sharing it must be ordered.
 * Outside stream capture the library keeps, per device, instantiated CUDA
 * graphs of the last 16 distinct calls (keyed by the layer descriptors'
 * fields, the buffer pointers and sizes, the token count and the dtype).  A
 * call equal to one of them replays its graph, one host launch instead of
 * n_layers + 1; the first such call captures the launches on a private stream
 * (the caller's stream never enters capture mode).  Graphs read the buffers
 * through their pointers, so new contents need no new graph.  Inside the
 * caller's stream capture the call makes its launches directly. */
size_t lbx_chain_prepare_size(const lbx_proj *projs, int32_t n_layers);
int lbx_chain_prepare(const lbx_proj *projs, int32_t n_layers, void *blob, size_t blob_bytes,
                      cudaStream_t stream);
size_t lbx_chain_fused_workspace_size(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens);
int lbx_chain_fused(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens, int32_t dtype,
                    void *const *acts, const void *blob, size_t blob_bytes, void *ws, size_t ws_bytes,
                    cudaStream_t stream);

/* ---- row-sharded LittleBitLinear over NVLink ----------------------------
 * No reference counterpart (the reference decodes on one CPU host): the
 * tensor-parallel split of one wide layer, with its all-gather fused into the
 * U-stage.  `proj` holds this rank's rows of U and u1 (out_features = its
 * share) and the full V, h, l.  Every result (token t, column y_col0 + i) is
 * stored into every rank's exchange buffer xbuf_peers[j] as one 8-byte word
 * (call number << 32 | fp32 bits) at word t * ld + y_col0 + i of the half
 * given by the call number's parity (halves half_words apart).  The buffers
 * must be addressable from this GPU (symmetric memory or IPC mappings, this
 * rank's own included), zero-filled before the first call.  state (device,
 * two zeroed uint32: completed calls, ticket) is this rank's call counter;
 * lbx_allgather_unpack advances it.  One projection, fp32, store epilogue,
 * n_tokens <= LBX_MAX_TOKENS; workspace as for lbx_linear.  Every rank makes
 * the same sequence of calls. */
int lbx_linear_allgather(const lbx_proj *proj, const lbx_linear_args *a, int32_t n_peer,
                         uint64_t *const *xbuf_peers /* host array */, int64_t half_words,
                         int32_t y_col0, int64_t ld, const uint32_t *state, void *ws,
                         size_t ws_bytes, cudaStream_t stream);

/* This rank's exchange buffer -> y [n_tokens, n] fp32 (row stride y_ld):
 * waits for every word of the current call (bounded: after 1 s it records
 * device error 0x601, writes NaN for what is missing and returns), then
 * advances state.  Launch it on the stream of the lbx_linear_allgather call,
 * before that stream's next lbx_linear_allgather: a rank overwrites a buffer
 * half only after every rank has unpacked it. */
int lbx_allgather_unpack(const uint64_t *xbuf, int64_t half_words, int32_t n_tokens, int32_t n,
                         int64_t ld, float *y, int64_t y_ld, uint32_t *state, int32_t use_pdl,
                         cudaStream_t stream);

/* ---- whole decoder step (cpp:1522-1840 full_forward, 1846-2079
 *      full_forward_batch, 2256-2317 generate_token) ----------------------- */
typedef struct lbx_layer {
  const float *ln1; /* input_layernorm  [hidden] */
  const float *ln2; /* post_attention_layernorm [hidden] */
  lbx_proj proj[7]; /* q, k, v, o, gate, up, down (cpp:1307-1317 order) */
  uint16_t *k_cache; uint16_t *v_cache; /* [kv_heads, max_seq, head_dim] bf16 */
} lbx_layer;

typedef struct lbx_model {
  int32_t n_layers, hidden, intermediate, heads, kv_heads, head_dim, vocab, max_seq;
  float rms_eps, rope_theta, attn_scale;
  int32_t use_pdl;
  const uint16_t *embed;   /* [vocab, hidden] bf16 */
  const float *final_norm; /* [hidden] */
  const uint16_t *lm_head; /* [vocab, hidden] bf16, may be NULL for hidden-only */
  const lbx_layer *layers; /* host array [n_layers] */
  int32_t exec_mode;       /* LBX_EXEC_*: how lbx_forward runs a step */
  int32_t _pad2;
} lbx_model;

/* lbx_forward execution: the kernel path launches one grid per op (chained
 * with programmatic dependent launch); a persistent program runs the whole
 * step (n <= LBX_MAX_TOKENS) as one cooperative launch with grid barriers
 * between phases.  Both compute the same bits.  AUTO selects the kernel path,
 * the faster of the two on B200 at present.  A program is built and uploaded
 * on the first call of each (model, n, cached length / 64, outputs,
 * workspace) combination, which must happen outside stream capture; later
 * calls may be captured. */
#define LBX_EXEC_AUTO 0
#define LBX_EXEC_KERNELS 1
#define LBX_EXEC_PROGRAM 2
#define LBX_EXEC_CLUSTER 3 /* lbx_linear_args.exec only */
/* lbx_linear_args.exec only: the two stage grids with every V unit's staging
 * passes in one CTA (inputs wider than 4096 columns otherwise run a cluster of
 * one CTA per pass on small grids).  Same bits; for validation. */
#define LBX_EXEC_KERNELS_ONE_CTA_V 4
/* lbx_linear_args.exec only: the tensor-core executor (tcgen05 kind::i8,
 * up to 64 tokens per launch) for any token count.  AUTO and KERNELS select
 * it for calls of 32 tokens or more, and of 16 or more when the call is large
 * (sum over projections of (in + out features) x ranks >= 2.5e7), provided the
 * workspace holds a batch; lbx_linear_workspace_size counts it for exactly
 * those calls.  Same bits. */
#define LBX_EXEC_TC 5
/* lbx_linear_args.exec only: the two stage grids at every token count (never
 * the tensor-core executor).  Same bits; for validation. */
#define LBX_EXEC_NO_TC 6

/* Workspace of lbx_forward: zero-filled once at allocation, like lbx_linear's. */
size_t lbx_forward_workspace_size(const lbx_model *m /* host */, int32_t n_tokens);
/* n tokens at cache slots start..start+n-1 (rotary positions pos[] or, when
 * pos == NULL, the slots).  With start_dev != NULL the slot offset is read
 * from device memory and `start` is only an upper bound (for CUDA graphs that
 * replay at varying positions; pos must then be given).  tree_mask as in
 * lbx_attn_args (NULL = causal).  hidden_out [n, hidden] receives the
 * final-RMSNorm output (may be NULL); logits [n, vocab] / argmax [n] as in
 * lbx_lmhead_argmax (may be NULL).  n <= 64 with tree_mask or start_dev; a
 * longer causal run at a host-given start proceeds in steps of 64 tokens
 * (the workspace is sized for min(n, 64)). */
int lbx_forward(const lbx_model *m, const int64_t *tokens, int32_t n, int32_t start,
                const int32_t *start_dev, const int32_t *pos, const uint64_t *tree_mask,
                float *hidden_out, float *logits, int64_t *argmax_out, void *ws,
                size_t ws_bytes, cudaStream_t stream);

/* Multi-sequence step (no reference counterpart: the reference decodes one
 * sequence per process): n tokens of each of n_seq independent sequences in
 * one step, so that every packed-weight read serves n_seq * n tokens (the
 * linear calls batch LBX_MAX_TOKENS of them per launch).  Rows of tokens,
 * pos, tree_mask and of the outputs are ordered sequence by sequence.
 * Sequence s's KV caches start cache_seq_stride elements after sequence
 * s-1's (the model's layer caches are sequence 0's; each is
 * [kv_heads, max_seq, head_dim] bf16) and its first new slot is
 * start_seq[s] (device int32; max_start bounds them all).  pos == NULL:
 * rotary positions start_seq[s] + i.  tree_mask: each row's mask over its
 * own sequence's n tokens, or NULL (causal).  Every sequence's outputs are
 * bit-identical to an lbx_forward call for it alone.  Kernel path only;
 * n_seq <= 64, n <= 64. */
size_t lbx_forward_multi_workspace_size(const lbx_model *m, int32_t n_seq, int32_t n_tokens);
int lbx_forward_multi(const lbx_model *m, const int64_t *tokens, int32_t n_seq, int32_t n, int32_t max_start,
                      const int32_t *start_seq, int64_t cache_seq_stride, const int32_t *pos,
                      const uint64_t *tree_mask, float *hidden_out, float *logits, int64_t *argmax_out,
                      void *ws, size_t ws_bytes, cudaStream_t stream);

/* Move KV rows inside the caches of every layer: for i < n, slot dst[i] <- slot
 * src[i] (all sources are read before any destination is written), used to
 * compact an accepted tree path into consecutive slots after tree
 * verification.  k_caches / v_caches: DEVICE arrays of n_layers cache pointers
 * ([kv_heads, max_seq, head_dim] bf16 each); n <= 64. */
int lbx_kv_move(uint16_t *const *k_caches, uint16_t *const *v_caches, int32_t n_layers,
                int32_t kv_heads, int32_t max_seq, int32_t head_dim, const int32_t *src,
                const int32_t *dst, int32_t n, cudaStream_t stream);

/* ---- diagnostics --------------------------------------------------------- */
/* Launch floor of a linear call, for benchmarks (no reference counterpart):
 * the call's two stage grids with the same launch shapes, shared memory and
 * PDL chaining as lbx_linear_verify (the one-CTA V-stage form), each CTA doing
 * no arithmetic.  mode 0: each CTA waits for the preceding grid and makes one
 * dependent load and store; mode 1: it also streams its unit's weights into
 * shared memory and waits for them.  Writes one word per CTA of the call's
 * scratch and of each y; the results are meaningless.  Arguments and
 * workspace as for lbx_linear_verify. */
int lbx_linear_floor(const lbx_proj *projs, const lbx_linear_args *a, int32_t mode, void *ws,
                     size_t ws_bytes, cudaStream_t stream);

/* Copies the last host-side error text of the calling thread. */
int lbx_last_error(char *buf, size_t n);
/* Device error word written by bounded waits that ran out (0 = none). */
int lbx_device_error(int32_t *out_host, cudaStream_t stream);
int lbx_clear_device_error(cudaStream_t stream);
/* Library version / build arch string (host). */
const char *lbx_version(void);

#ifdef __cplusplus
}
#endif
#endif /* LBX_H */
