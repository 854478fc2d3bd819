// Small decoder kernels: embedding gather, RMSNorm, SiLU·mul, RoPE and the
// on-device greedy acceptance of speculative decoding.

#include "common.cuh"

namespace lbx {

// cos/sin of pos * theta^(-2i/d), evaluated in double precision (HF Llama's
// LlamaRotaryEmbedding computes the same angle in fp32).
LBX_DEV void rope_cs(int pos, int i, int d, float theta, float &c, float &s) {
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

__global__ void embed_kernel(const uint16_t *__restrict__ table, const int64_t *__restrict__ ids,
                             int hidden, int vocab, float *__restrict__ out) {
  const int i = blockIdx.x;
  const int64_t id = ids[i];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) atomicCAS(&g_lbx_device_error, 0, 0x301);
  for (int h = threadIdx.x; h < hidden; h += blockDim.x)
    out[(int64_t)i * hidden + h] = ok ? bf16_to_f32(table[id * hidden + h]) : 0.f;
}

__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w, int hidden,
                               float eps, float *out) {
  const int i = blockIdx.x;
  const float *xr = x + (int64_t)i * hidden;
  float ss = 0.f;
  for (int h = threadIdx.x; h < hidden; h += blockDim.x) ss += xr[h] * xr[h];
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rs = 1.0f / sqrtf(red[0] / (float)hidden + eps);
  for (int h = threadIdx.x; h < hidden; h += blockDim.x)
    out[(int64_t)i * hidden + h] = xr[h] * rs * w[h];
}

__global__ void silu_mul_kernel(const float *__restrict__ g, const float *__restrict__ u, int64_t n,
                                float *__restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float x = g[i];
    out[i] = (x / (1.0f + expf(-x))) * u[i];
  }
}

__global__ void rope_kernel(float *x, const int32_t *__restrict__ pos, int heads, int d,
                            float theta) {
  const int i = blockIdx.x;
  const int half = d / 2;
  const int p = pos[i];
  for (int e = threadIdx.x; e < heads * half; e += blockDim.x) {
    const int h = e / half, j = e - h * half;
    float c, s;
    rope_cs(p, j, d, theta, c, s);
    float *row = x + ((int64_t)i * heads + h) * d;
    const float x1 = row[j], x2 = row[j + half];
    row[j] = x1 * c - x2 * s;
    row[j + half] = x2 * c + x1 * s;
  }
}

__global__ void accept_chain_kernel(const int64_t *draft, const int64_t *tgt, int k, int64_t *out) {
  if (threadIdx.x != 0) return;
  int a = 0;
  while (a < k && draft[a] == tgt[a]) ++a;
  out[0] = a;
  out[1] = tgt[a];
}

// evaluate_posterior_greedy (tree_utils.py:182-214) over paths gathered with
// retrieve_indices: candidate row l accepts the longest prefix where
// cand[l][i+1] == argmax(logits of node retrieve[l][i]).
__global__ void accept_tree_kernel(const int64_t *cand, const int64_t *node_argmax,
                                   const int64_t *retrieve, int L, int D1, int64_t *out) {
  if (threadIdx.x != 0) return;
  int best = 0, best_len = 0;
  for (int l = 0; l < L; ++l) {
    int len = 0;
    for (int i = 0; i + 1 < D1; ++i) {
      const int64_t node = retrieve[l * D1 + i];
      const int64_t am = node >= 0 ? node_argmax[node] : 0;  // padded rows: zero logits
      if (cand[l * D1 + i + 1] != am) break;
      ++len;
    }
    if (len > best_len) {  // first maximum, as torch.argmax
      best_len = len;
      best = l;
    }
  }
  out[0] = best;
  out[1] = best_len;
  const int64_t bnode = retrieve[best * D1 + best_len];
  out[2] = bnode >= 0 ? node_argmax[bnode] : 0;
  for (int i = 0; i + 1 < D1; ++i) out[3 + i] = i < best_len ? retrieve[best * D1 + i + 1] : -1;
}

}  // namespace lbx

extern "C" int lbx_embed(const uint16_t *table, const int64_t *ids, int32_t n, int32_t hidden,
                         int32_t vocab, float *out, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(n >= 0 && hidden > 0 && vocab > 0, "bad shape");
  if (n == 0) return LBX_OK;
  LBX_CHECK_ARG(table && ids && out, "NULL pointer");
  embed_kernel<<<n, 256, 0, stream>>>(table, ids, hidden, vocab, out);
  return cuda_status(cudaGetLastError(), "embed launch");
}

extern "C" int lbx_rmsnorm(const float *x, const float *w, int32_t n, int32_t hidden, float eps,
                           float *out, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(n >= 0 && hidden > 0, "bad shape");
  if (n == 0) return LBX_OK;
  LBX_CHECK_ARG(x && w && out, "NULL pointer");
  rmsnorm_kernel<<<n, 256, 0, stream>>>(x, w, hidden, eps, out);
  return cuda_status(cudaGetLastError(), "rmsnorm launch");
}

extern "C" int lbx_silu_mul(const float *g, const float *u, int64_t n, float *out,
                            cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(n >= 0, "bad shape");
  if (n == 0) return LBX_OK;
  LBX_CHECK_ARG(g && u && out, "NULL pointer");
  silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(g, u, n, out);
  return cuda_status(cudaGetLastError(), "silu_mul launch");
}

extern "C" int lbx_rope(float *x, const int32_t *pos, int32_t n, int32_t heads, int32_t head_dim,
                        float theta, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(n >= 0 && heads > 0 && head_dim > 0 && head_dim % 2 == 0, "bad shape");
  if (n == 0) return LBX_OK;
  LBX_CHECK_ARG(x && pos, "NULL pointer");
  rope_kernel<<<n, 256, 0, stream>>>(x, pos, heads, head_dim, theta);
  return cuda_status(cudaGetLastError(), "rope launch");
}

extern "C" int lbx_accept_greedy_chain(const int64_t *draft, const int64_t *target_argmax, int32_t k,
                                       int64_t *out, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(k >= 0, "k must be >= 0");
  LBX_CHECK_ARG((draft || k == 0) && target_argmax && out, "NULL pointer");
  accept_chain_kernel<<<1, 32, 0, stream>>>(draft, target_argmax, k, out);
  return cuda_status(cudaGetLastError(), "accept_chain launch");
}

extern "C" int lbx_accept_greedy_tree(const int64_t *cand, const int64_t *node_argmax,
                                      const int64_t *retrieve, int32_t L, int32_t D1, int64_t *out,
                                      cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(L >= 1 && D1 >= 1, "bad shape");
  LBX_CHECK_ARG(cand && node_argmax && retrieve && out, "NULL pointer");
  accept_tree_kernel<<<1, 32, 0, stream>>>(cand, node_argmax, retrieve, L, D1, out);
  return cuda_status(cudaGetLastError(), "accept_tree launch");
}
