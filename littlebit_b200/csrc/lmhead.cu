// Final RMSNorm + lm_head GEMV (bf16 weights, fp32 accumulation) + argmax.
//
// Replaces dense_gemv_f32 (patches/littlebit_cpu_optimized.cpp:1054-1115) and
// the serial argmax of generate_token (cpp:2306-2314).  The 32000x4096 bf16
// matrix (262 MB) is the largest single read of a draft step, so the kernel
// is a pure HBM stream: every warp owns whole vocabulary rows, each lane
// issues all 16-byte loads of its row slice before reducing, and up to 8
// tokens share one pass over the weights (the normalised hidden states sit
// in shared memory).  Argmax keeps the lowest index among equal maxima
// (torch.argmax order) through an order-preserving 64-bit key; per-CTA
// winners are merged by a second kernel in CTA order.

#include "common.cuh"

namespace lbx {

constexpr int LM_WARPS = 16;
constexpr int LM_TOK = 8;    // tokens per pass

struct LmParams {
  const float *x;
  const float *norm_w;
  float eps;
  int n, hidden, vocab, nblocks;
  const uint16_t *w;
  float *logits;
  unsigned long long *best;  // [nblocks][LM_TOK]
};

LBX_DEV unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - (uint32_t)idx);
}

// one unit of the vocabulary stream (units interleave rows warp by warp);
// S holds the NT normalised hidden states
template <int NT>
LBX_DEV void lmhead_unit(const LmParams &p, int unit, int nunits, float *xs) {
  __shared__ float s_rs[LM_TOK];
  __shared__ unsigned long long s_best[LM_WARPS][LM_TOK];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = p.hidden;

  // normalised hidden states (RMSNorm recomputed per unit: n*hidden L2 reads)
  for (int t = warp; t < NT; t += LM_WARPS) {
    float ss = 0.f;
    if (p.norm_w && t < p.n)
      for (int h = lane; h < H; h += 32) {
        const float v = __ldcg(p.x + (int64_t)t * H + h);
        ss += v * v;
      }
    ss = warp_sum(ss);
    if (lane == 0) s_rs[t] = p.norm_w ? 1.0f / sqrtf(ss / (float)H + p.eps) : 1.0f;
  }
  __syncthreads();
  for (int e = tid; e < NT * H; e += LM_WARPS * 32) {
    const int t = e / H, h = e - t * H;
    float v = t < p.n ? __ldcg(p.x + (int64_t)t * H + h) * s_rs[t] : 0.f;
    if (p.norm_w) v *= p.norm_w[h];
    xs[e] = v;
  }
  __syncthreads();

  unsigned long long best[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) best[t] = 0ull;

  const int nvec = H / 256;  // 16-byte vectors per lane per row
  const int gw = unit * LM_WARPS + warp;
  const int tw = nunits * LM_WARPS;
  for (int row = gw; row < p.vocab; row += tw) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(p.w + (int64_t)row * H);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    uint4 buf[8];
    for (int v0 = 0; v0 < nvec; v0 += 8) {
      const int nb = min(8, nvec - v0);
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (b < nb) buf[b] = __ldcs(wr + (v0 + b) * 32 + lane);
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (b >= nb) break;
        const int h0 = ((v0 + b) * 32 + lane) * 8;
        const uint32_t ww[4] = {buf[b].x, buf[b].y, buf[b].z, buf[b].w};
        float wf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          wf[2 * e] = __uint_as_float(ww[e] << 16);
          wf[2 * e + 1] = __uint_as_float(ww[e] & 0xFFFF0000u);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4 xa = *reinterpret_cast<const float4 *>(xs + t * H + h0);
          const float4 xb = *reinterpret_cast<const float4 *>(xs + t * H + h0 + 4);
          float a = acc[t];
          a = fmaf(wf[0], xa.x, a); a = fmaf(wf[1], xa.y, a);
          a = fmaf(wf[2], xa.z, a); a = fmaf(wf[3], xa.w, a);
          a = fmaf(wf[4], xb.x, a); a = fmaf(wf[5], xb.y, a);
          a = fmaf(wf[6], xb.z, a); a = fmaf(wf[7], xb.w, a);
          acc[t] = a;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float v = warp_sum(acc[t]);
      if (t < p.n) {
        if (p.logits && lane == 0) p.logits[(int64_t)t * p.vocab + row] = v;
        const unsigned long long k = argmax_key(v, row);
        best[t] = k > best[t] ? k : best[t];
      }
    }
  }
  if (lane == 0)
#pragma unroll
    for (int t = 0; t < NT; ++t) s_best[warp][t] = best[t];
  __syncthreads();
  if (tid < NT && p.best) {
    unsigned long long b = 0ull;
    for (int w = 0; w < LM_WARPS; ++w) b = s_best[w][tid] > b ? s_best[w][tid] : b;
    p.best[(int64_t)unit * LM_TOK + tid] = b;
  }
  __syncthreads();
}

template <int NT>
__global__ void __launch_bounds__(LM_WARPS * 32) lmhead_kernel(const __grid_constant__ LmParams p) {
  extern __shared__ __align__(16) float xs[];  // NT x hidden
  pdl_trigger();
  pdl_wait();
  lmhead_unit<NT>(p, blockIdx.x, gridDim.x, xs);
}

// per-unit winners -> token ids (lowest index among equal maxima)
LBX_DEV void argmax_unit(const unsigned long long *best, int nblocks, int n, int64_t *out) {
  const int t = threadIdx.x;
  if (t < n) {
    unsigned long long b = 0ull;
    for (int i = 0; i < nblocks; ++i) {
      const unsigned long long v = __ldcg(best + (int64_t)i * LM_TOK + t);
      b = v > b ? v : b;
    }
    out[t] = (int64_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
  }
}

__global__ void argmax_final_kernel(const unsigned long long *best, int nblocks, int n,
                                    int64_t *out) {
  pdl_trigger();
  pdl_wait();
  argmax_unit(best, nblocks, n, out);
}

static int lm_blocks() { return device_sm_count(); }

}  // namespace lbx

extern "C" size_t lbx_lmhead_workspace_size(int32_t n, int32_t vocab) {
  (void)n;
  (void)vocab;
  return (size_t)lbx::lm_blocks() * lbx::LM_TOK * 8;
}

extern "C" int lbx_lmhead_argmax(const float *x, const float *norm_w, float eps, int32_t n,
                                 int32_t hidden, const uint16_t *w_bf16, int32_t vocab,
                                 float *logits, int64_t *argmax_out, void *ws, size_t ws_bytes,
                                 int32_t use_pdl, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(n >= 1 && vocab >= 1, "bad shape");
  LBX_CHECK_SUP(hidden > 0 && hidden % 256 == 0 && hidden * 4 <= 200 * 1024,
                "hidden must be a multiple of 256 and <= 51200");
  LBX_CHECK_ARG(x && w_bf16, "NULL pointer");
  LBX_CHECK_ARG(aligned16(w_bf16), "lm_head weight must be 16-byte aligned");
  LBX_CHECK_ARG(logits || argmax_out, "nothing to compute");
  const size_t need = lbx_lmhead_workspace_size(n, vocab);
  LBX_CHECK_ARG(!argmax_out || (ws && ws_bytes >= need), "workspace too small");
  static DevCache<int> attr;
  int attr_done = 0;
  const int arc = attr.get(attr_done, [](int &out) {
    for (auto k : {lmhead_kernel<1>, lmhead_kernel<2>, lmhead_kernel<4>, lmhead_kernel<6>, lmhead_kernel<8>}) {
      cudaError_t e = allow_max_smem(k);
      if (e != cudaSuccess) return cuda_status(e, "lmhead smem attribute");
    }
    out = 1;
    return (int)LBX_OK;
  });
  if (arc) return arc;
  const bool pdl = use_pdl != 0;
  const int nb = lm_blocks();
  // tokens per pass: the normalised hidden states of a pass live in shared
  // memory (8, 6, 4, 2 or 1 of them; 6 at hidden 8192).  Each token's logits
  // are the same fmaf chains whatever the pass holds.
  int per = LM_TOK;
  while (per > 1 && (size_t)per * hidden * 4 > 200 * 1024) per = per == 8 ? 6 : per == 6 ? 4 : per >> 1;
  for (int t0 = 0; t0 < n; t0 += per) {
    const int nt = std::min(per, n - t0);
    LmParams p = {};
    p.x = x + (int64_t)t0 * hidden;
    p.norm_w = norm_w;
    p.eps = eps;
    p.n = nt;
    p.hidden = hidden;
    p.vocab = vocab;
    p.nblocks = nb;
    p.w = w_bf16;
    p.logits = logits ? logits + (int64_t)t0 * vocab : nullptr;
    p.best = reinterpret_cast<unsigned long long *>(ws);
    const int NT = nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : nt <= 6 && per == 6 ? 6 : 8;  // rows >= nt staged as 0
    auto kern = NT == 1 ? lmhead_kernel<1> : NT == 2 ? lmhead_kernel<2> : NT == 4 ? lmhead_kernel<4>
                : NT == 6 ? lmhead_kernel<6> : lmhead_kernel<8>;
    const size_t smem = (size_t)NT * hidden * 4;
    cudaError_t e = launch(kern, dim3(nb), dim3(LM_WARPS * 32), smem, stream, pdl, p);
    if (e != cudaSuccess) return cuda_status(e, "lmhead launch");
    if (argmax_out) {
      e = launch(argmax_final_kernel, dim3(1), dim3(32), 0, stream, pdl,
                 (const unsigned long long *)p.best, nb, nt, argmax_out + t0);
      if (e != cudaSuccess) return cuda_status(e, "argmax launch");
    }
  }
  return LBX_OK;
}
