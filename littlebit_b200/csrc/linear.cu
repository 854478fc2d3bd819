// LittleBitLinear on packed sign words for sm_100a.
//
// y = u1 ⊙ U_sign·(mid ⊙ V_sign·(v2 ⊙ x))  (+ residual branch) (+ bias)
// Reference: quantization/modules/littlebit.py:95-121 (fp32 semantics) and
// patches/littlebit_cpu_optimized.cpp:598-701 (packed-word CPU kernel).
//
// One call = two kernels chained with programmatic dependent launch:
//   V-stage  t = V_sign·a,  a = v2 ⊙ prologue(x);  z_b = mid_b ⊙ t  -> scratch
//   U-stage  y = Σ_b u1_b ⊙ U_b·z_b
// Both stages are "sign matrix × activation" contractions done on the int8
// tensor cores:
//   * activations are quantised to 16-bit integers (two int8 digits) with a
//     per-token scale (per 1024-column chunk in the V-stage, per vector in the
//     U-stage), so Σ_j s_j·q_j is computed EXACTLY in int32;
//   * a sign word is expanded in registers with one prmt per 4 signs into
//     int8 0/−1 (= −bit), giving Σ_j (−b_j)·digit_j from mma.m16n8k32.s8;
//   * Σ_j s_j q_j = Σ_j q_j + 2·(256·D_hi + D_lo).
// Integer accumulation makes every token's result independent of how many
// tokens share the launch (verify batch == batch 1, bit for bit).
//
// Weights are prefetched with cp.async.bulk into shared memory BEFORE
// griddepcontrol.wait, so their HBM latency overlaps the preceding kernel.

#include <algorithm>

#include "common.cuh"

namespace lbx {

constexpr int CH_WORDS = 32;  // words per V-stage chunk (1024 columns)
constexpr int VWARPS = 4;     // warps per V-stage CTA (split the chunks)
constexpr int UWARPS_MAX = 8; // warps per U-stage CTA (one 16-row tile each)

// activation buffer: act[W][slot][col] uint32, word stride 8*ncols+8
__host__ __device__ inline int act_ws(int ncols) { return 8 * ncols + 8; }
// padded row pitch (words) for per-row weight copies: conflict-free banks
__host__ __device__ inline int row_pitch(int words) {
  return words + 4 + 4 * ((words / 4) & 1);
}

struct VSeg {
  const int32_t *v_sign; // [rank, Wv]
  const float *v2;       // [K]
  const float *mid0;     // [rank]
  const float *mid1;     // [rank] shared-V residual, or nullptr
  float *z0;             // [k, rank]
  float *z1;             // [k, rank] or nullptr
  int rank;
  int tile0;             // first CTA index of this segment
};

struct VParams {
  VSeg seg[2 * LBX_MAX_PROJ];
  int nseg;
  int K, Wv, pitch, nch;
  int k, ncols;
  int xdt, prologue;
  float eps;
  const void *x;
  const void *x2;
  const float *norm_w;
};

struct USeg {
  const int32_t *u_sign[2];
  const float *u1[2];
  const float *z[2];
  int rank[2];
  int words[2];   // ceil(rank/32)
  int pitch[2];   // smem row pitch (words)
  int perrow[2];  // 1: per-row copies (words % 4 == 0), 0: whole tile
  int nbr;
  int out;
  const float *bias;
  void *y;
  int64_t y_ld;
  int cta0;       // first CTA of this projection
};

struct UParams {
  USeg seg[LBX_MAX_PROJ];
  int nseg;
  int k, ncols, ydt, epi, uwarps;
  int act_words[2];   // max over projections of 4*ceil(words/4)
  int wtile_words;    // per-warp weight region (words)
};

// ---------------------------------------------------------------------------
// shared contraction: one warp, rows g and g+8 of a 16-row sign tile
// ---------------------------------------------------------------------------
// Consumes `ngroups` groups of 4 words.  Thread (g,q) reads word 4G+q of its two
// rows; its 8 prmt expansions feed 4 MMA k-steps.  The activation layout puts,
// for word w, slot s=(h*4+j), column c, the 4 digits of reduction positions
// 32w+16h+j+{0,4,8,12} into one uint32, matching the A-fragment bytes.
template <int NCB>
LBX_DEV void sign_mma(int (&acc)[NCB][4], const uint32_t *rowg, const uint32_t *rowg8,
                      const uint32_t *act, int ws, int ncols, int ngroups, int lane) {
  const int q = lane & 3;
  const int n8 = lane >> 2;
#pragma unroll 2
  for (int G = 0; G < ngroups; ++G) {
    const int w = 4 * G + q;
    const uint32_t wa = rowg[w];
    const uint32_t wb = rowg8[w];
    const uint32_t *aw = act + w * ws;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int sh = 16 * (r >> 1) + 2 * (r & 1);
      const uint32_t a0 = negbits4(wa >> sh);
      const uint32_t a2 = negbits4(wa >> (sh + 1));
      const uint32_t a1 = negbits4(wb >> sh);
      const uint32_t a3 = negbits4(wb >> (sh + 1));
      const int slot = 4 * (r >> 1) + 2 * (r & 1);
#pragma unroll
      for (int cb = 0; cb < NCB; ++cb) {
        const int col = cb * 8 + n8;
        uint32_t b0 = 0, b1 = 0;
        if (col < ncols) {
          b0 = aw[slot * ncols + col];
          b1 = aw[(slot + 1) * ncols + col];
        }
        mma_s8(acc[cb], a0, a1, a2, a3, b0, b1);
      }
    }
  }
}

LBX_DEV uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) |
         ((uint32_t)(d & 255) << 24);
}

// ---------------------------------------------------------------------------
// V-stage
// ---------------------------------------------------------------------------
LBX_DEV float v_input(const VParams &p, const float *v2, int tok, int pos, float *xsq) {
  const int64_t i = (int64_t)tok * p.K + pos;
  float x = load_act(p.x, p.xdt, i);
  float a;
  if (p.prologue == LBX_PRO_RMSNORM) {
    if (xsq) *xsq += x * x;
    a = x * __ldg(p.norm_w + pos);
  } else if (p.prologue == LBX_PRO_SILU_MUL) {
    const float u = load_act(p.x2, p.xdt, i);
    a = (x / (1.0f + expf(-x))) * u;
  } else {
    a = x;
  }
  return a * __ldg(v2 + pos);
}

template <int NCB>
__global__ void __launch_bounds__(VWARPS * 32) vstage_kernel(const __grid_constant__ VParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;

  // locate segment / tile
  int s = 0;
  while (s + 1 < p.nseg && (int)blockIdx.x >= p.seg[s + 1].tile0) ++s;
  const VSeg &sg = p.seg[s];
  const int row0 = ((int)blockIdx.x - sg.tile0) * 16;
  const int rows = min(16, sg.rank - row0);

  const int ws = act_ws(p.ncols);
  uint32_t *wbuf = reinterpret_cast<uint32_t *>(smem_raw);           // 16 x pitch
  uint32_t *actb = wbuf + 16 * p.pitch;                               // VWARPS x 32 x ws
  float *red = reinterpret_cast<float *>(actb + VWARPS * CH_WORDS * ws); // VWARPS x 16 x k
  float *ssq = red + VWARPS * 16 * p.k;                               // VWARPS x k
  uint64_t *bar = reinterpret_cast<uint64_t *>(ssq + VWARPS * LBX_MAX_TOKENS + 2);
  bar = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(bar) + 7) & ~uintptr_t(7));

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // weight prefetch (independent of the preceding kernel)
  if (warp == 0) {
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)rows * p.Wv * 4u);
    __syncwarp();
    if (lane < rows)
      bulk_g2s(wbuf + lane * p.pitch, sg.v_sign + (int64_t)(row0 + lane) * p.Wv,
               (uint32_t)p.Wv * 4u, bar);
  }
  pdl_trigger();
  pdl_wait();

  uint32_t *act = actb + warp * CH_WORDS * ws;
  float tacc[NCB][2];
#pragma unroll
  for (int cb = 0; cb < NCB; ++cb) tacc[cb][0] = tacc[cb][1] = 0.f;
  float xsq_tok = 0.f;  // lane-partial sum of squares for token `lane` (RMSNorm)
  bool have_w = false;
  bool ok = true;

  __shared__ float s_inv[VWARPS][LBX_MAX_TOKENS];
  __shared__ int s_sq[VWARPS][LBX_MAX_TOKENS];

  for (int c = warp; c < p.nch; c += VWARPS) {
    const int base = c * CH_WORDS * 32;
    const int cwords = min(CH_WORDS, p.Wv - c * CH_WORDS);
    // ---- stage this chunk: per token absmax, then digits
    for (int t = 0; t < p.k; ++t) {
      float amax = 0.f, sq = 0.f;
      for (int i = lane; i < cwords * 32; i += 32) {
        const float a = v_input(p, sg.v2, t, base + i, &sq);
        amax = fmaxf(amax, fabsf(a));
      }
      amax = warp_max(amax);
      if (p.prologue == LBX_PRO_RMSNORM) {
        sq = warp_sum(sq);
        if (lane == t) xsq_tok += sq;
      }
      const float sc = amax > 0.f ? QMAX / amax : 0.f;
      int sqi = 0;
      for (int it = 0; it < CH_WORDS / 4; ++it) {
        const int W = it * 4 + (lane >> 3);
        const int slot = lane & 7;
        const int hh = slot >> 2, jj = slot & 3;
        int hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int qv = 0;
          if (W < cwords) {
            const float a = v_input(p, sg.v2, t, base + 32 * W + 16 * hh + jj + 4 * e, nullptr);
            qv = __float2int_rn(a * sc);
          }
          sqi += qv;
          split_digits(qv, hi[e], lo[e]);
        }
        act[W * ws + slot * p.ncols + 2 * t] = pack4(hi[0], hi[1], hi[2], hi[3]);
        act[W * ws + slot * p.ncols + 2 * t + 1] = pack4(lo[0], lo[1], lo[2], lo[3]);
      }
      sqi = warp_sum_i(sqi);
      if (lane == 0) {
        s_inv[warp][t] = amax / QMAX;
        s_sq[warp][t] = sqi;
      }
    }
    __syncwarp();
    if (!have_w) {
      ok = mbar_wait_bounded(bar, 0, 0x101);
      have_w = true;
    }
    if (!ok) break;
    int acc[NCB][4];
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) acc[cb][0] = acc[cb][1] = acc[cb][2] = acc[cb][3] = 0;
    sign_mma<NCB>(acc, wbuf + g * p.pitch + c * CH_WORDS, wbuf + (g + 8) * p.pitch + c * CH_WORDS,
                  act, ws, p.ncols, cwords / 4, lane);
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) {
      const int t = cb * 4 + q;
      if (t < p.k) {
        const int sq = s_sq[warp][t];
        const float inv = s_inv[warp][t];
        tacc[cb][0] += __int2float_rn(sq + 2 * (256 * acc[cb][0] + acc[cb][1])) * inv;
        tacc[cb][1] += __int2float_rn(sq + 2 * (256 * acc[cb][2] + acc[cb][3])) * inv;
      }
    }
    __syncwarp();
  }
  // if this warp had no chunk it never waited; make sure the copy landed
  // before the CTA exits (shared memory must not be released under a copy).
  if (!have_w) ok = mbar_wait_bounded(bar, 0, 0x102);

  // ---- cross-warp reduction in fixed warp order
#pragma unroll
  for (int cb = 0; cb < NCB; ++cb) {
    const int t = cb * 4 + q;
    if (t < p.k) {
      red[(warp * 16 + g) * p.k + t] = tacc[cb][0];
      red[(warp * 16 + g + 8) * p.k + t] = tacc[cb][1];
    }
  }
  if (p.prologue == LBX_PRO_RMSNORM && lane < p.k) ssq[warp * LBX_MAX_TOKENS + lane] = xsq_tok;
  __syncthreads();
  if (!ok) return;
  for (int i = tid; i < rows * p.k; i += blockDim.x) {
    const int rr = i / p.k, t = i % p.k;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < VWARPS; ++w) v += red[(w * 16 + rr) * p.k + t];
    if (p.prologue == LBX_PRO_RMSNORM) {
      float s2 = 0.f;
#pragma unroll
      for (int w = 0; w < VWARPS; ++w) s2 += ssq[w * LBX_MAX_TOKENS + t];
      v *= rsqrtf(s2 / (float)p.K + p.eps);
    }
    const int r = row0 + rr;
    sg.z0[(int64_t)t * sg.rank + r] = __ldg(sg.mid0 + r) * v;
    if (sg.z1) sg.z1[(int64_t)t * sg.rank + r] = __ldg(sg.mid1 + r) * v;
  }
}

// ---------------------------------------------------------------------------
// U-stage
// ---------------------------------------------------------------------------
template <int NCB>
__global__ void __launch_bounds__(UWARPS_MAX * 32) ustage_kernel(const __grid_constant__ UParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int nthreads = blockDim.x;

  int s = 0;
  while (s + 1 < p.nseg && (int)blockIdx.x >= p.seg[s + 1].cta0) ++s;
  const USeg &sg = p.seg[s];
  const int n0 = ((int)blockIdx.x - sg.cta0) * (16 * p.uwarps) + 16 * warp;
  const bool active = n0 < sg.out;

  const int ws = act_ws(p.ncols);
  uint32_t *act0 = reinterpret_cast<uint32_t *>(smem_raw);
  uint32_t *act1 = act0 + p.act_words[0] * ws;
  uint32_t *wt = act1 + p.act_words[1] * ws;                 // uwarps x wtile_words
  uint64_t *bars = reinterpret_cast<uint64_t *>(wt + p.uwarps * p.wtile_words);
  __shared__ float s_inv[2][LBX_MAX_TOKENS];
  __shared__ int s_sq[2][LBX_MAX_TOKENS];

  uint32_t *mywt0 = wt + warp * p.wtile_words;
  uint32_t *mywt1 = mywt0 + 16 * sg.pitch[0] + 4;

  if (lane == 0) {
    mbar_init(bars + warp, 1);
    fence_mbar_init();
  }
  if (tid < 2 * LBX_MAX_TOKENS) (&s_sq[0][0])[tid] = 0;
  __syncthreads();
  if (active) {
    uint32_t bytes = 0;
    for (int b = 0; b < sg.nbr; ++b) bytes += 16u * sg.words[b] * 4u;
    if (lane == 0) mbar_arrive_expect_tx(bars + warp, bytes);
    __syncwarp();
    for (int b = 0; b < sg.nbr; ++b) {
      uint32_t *dst = b == 0 ? mywt0 : mywt1;
      const int32_t *src = sg.u_sign[b] + (int64_t)n0 * sg.words[b];
      if (sg.perrow[b]) {
        if (lane < 16)
          bulk_g2s(dst + lane * sg.pitch[b], src + (int64_t)lane * sg.words[b],
                   (uint32_t)sg.words[b] * 4u, bars + warp);
      } else if (lane == 0) {
        bulk_g2s(dst, src, 16u * sg.words[b] * 4u, bars + warp);
      }
    }
  }
  pdl_trigger();
  pdl_wait();

  // ---- stage z_b as 16-bit digits with one scale per token
  for (int b = 0; b < sg.nbr; ++b) {
    const float *z = sg.z[b];
    const int r = sg.rank[b];
    for (int t = warp; t < p.k; t += p.uwarps) {
      float m = 0.f;
      for (int i = lane; i < r; i += 32) m = fmaxf(m, fabsf(z[(int64_t)t * r + i]));
      m = warp_max(m);
      if (lane == 0) s_inv[b][t] = m / QMAX;
    }
  }
  __syncthreads();
  for (int b = 0; b < sg.nbr; ++b) {
    const float *z = sg.z[b];
    const int r = sg.rank[b];
    const int nw = 4 * ((sg.words[b] + 3) / 4);
    uint32_t *act = b == 0 ? act0 : act1;
    const int items = nw * 8 * p.k;
    for (int i = tid; i < items; i += nthreads) {
      const int t = i / (nw * 8);
      const int rem = i - t * nw * 8;
      const int W = rem >> 3, slot = rem & 7;
      const int hh = slot >> 2, jj = slot & 3;
      const float inv = s_inv[b][t];
      const float sc = inv > 0.f ? 1.0f / inv : 0.f;
      int hi[4], lo[4], sq = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int pos = 32 * W + 16 * hh + jj + 4 * e;
        int qv = 0;
        if (pos < r) qv = __float2int_rn(z[(int64_t)t * r + pos] * sc);
        sq += qv;
        split_digits(qv, hi[e], lo[e]);
      }
      act[W * ws + slot * p.ncols + 2 * t] = pack4(hi[0], hi[1], hi[2], hi[3]);
      act[W * ws + slot * p.ncols + 2 * t + 1] = pack4(lo[0], lo[1], lo[2], lo[3]);
      atomicAdd(&s_sq[b][t], sq);
    }
  }
  __syncthreads();

  bool ok = true;
  if (active) ok = mbar_wait_bounded(bars + warp, 0, 0x201);
  if (!active || !ok) return;

  int acc0[NCB][4], acc1[NCB][4];
#pragma unroll
  for (int cb = 0; cb < NCB; ++cb)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc0[cb][e] = acc1[cb][e] = 0;
  sign_mma<NCB>(acc0, mywt0 + g * sg.pitch[0], mywt0 + (g + 8) * sg.pitch[0], act0, ws, p.ncols,
                (sg.words[0] + 3) / 4, lane);
  if (sg.nbr > 1)
    sign_mma<NCB>(acc1, mywt1 + g * sg.pitch[1], mywt1 + (g + 8) * sg.pitch[1], act1, ws,
                  p.ncols, (sg.words[1] + 3) / 4, lane);

#pragma unroll
  for (int cb = 0; cb < NCB; ++cb) {
    const int t = cb * 4 + q;
    if (t >= p.k) continue;
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      const int n = n0 + g + 8 * hrow;
      float v = __ldg(sg.u1[0] + n) *
                (__int2float_rn(s_sq[0][t] + 2 * (256 * acc0[cb][2 * hrow] + acc0[cb][2 * hrow + 1])) *
                 s_inv[0][t]);
      if (sg.nbr > 1)
        v += __ldg(sg.u1[1] + n) *
             (__int2float_rn(s_sq[1][t] + 2 * (256 * acc1[cb][2 * hrow] + acc1[cb][2 * hrow + 1])) *
              s_inv[1][t]);
      if (sg.bias) v += __ldg(sg.bias + n);
      const int64_t off = (int64_t)t * sg.y_ld + n;
      if (p.ydt == LBX_F32) {
        float *y = reinterpret_cast<float *>(sg.y) + off;
        if (p.epi == LBX_EPI_ADD) v += *y;
        *y = v;
      } else {
        reinterpret_cast<uint16_t *>(sg.y)[off] = f32_to_bf16(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static size_t z_bytes(const lbx_proj *projs, int n_proj, int k) {
  size_t tot = 0;
  for (int i = 0; i < n_proj; ++i)
    for (int b = 0; b < projs[i].n_branches; ++b)
      tot += (((size_t)projs[i].br[b].rank * k * 4) + 255) & ~(size_t)255;
  return tot;
}

static int validate(const lbx_proj *projs, int n_proj) {
  LBX_CHECK_ARG(projs && n_proj >= 1 && n_proj <= LBX_MAX_PROJ, "n_proj must be in [1,%d]",
                LBX_MAX_PROJ);
  const int K = projs[0].in_features;
  for (int i = 0; i < n_proj; ++i) {
    const lbx_proj &pr = projs[i];
    LBX_CHECK_ARG(pr.in_features == K, "projections sharing an input need equal in_features");
    LBX_CHECK_SUP(K > 0 && K % 128 == 0, "in_features must be a positive multiple of 128 (got %d)",
                  K);
    LBX_CHECK_SUP(pr.out_features > 0 && pr.out_features % 16 == 0,
                  "out_features must be a positive multiple of 16 (got %d)", pr.out_features);
    LBX_CHECK_ARG(pr.n_branches == 1 || pr.n_branches == 2, "n_branches must be 1 or 2");
    for (int b = 0; b < pr.n_branches; ++b) {
      const lbx_branch &br = pr.br[b];
      LBX_CHECK_ARG(br.rank > 0, "rank must be positive");
      LBX_CHECK_ARG(br.mid && br.u_sign && br.u1, "branch %d: mid/u_sign/u1 required", b);
      LBX_CHECK_ARG(aligned16(br.u_sign), "u_sign must be 16-byte aligned");
      if (br.v_sign) {
        LBX_CHECK_ARG(br.v2, "branch %d: v2 required with v_sign", b);
        LBX_CHECK_ARG(aligned16(br.v_sign), "v_sign must be 16-byte aligned");
      } else {
        LBX_CHECK_ARG(b == 1 && pr.br[0].v_sign && br.rank == pr.br[0].rank,
                      "a shared-V branch must be the residual with the main branch's rank");
      }
    }
  }
  return LBX_OK;
}

static size_t vstage_smem(int Wv, int ncols, int k) {
  const int pitch = row_pitch(Wv);
  size_t b = (size_t)16 * pitch * 4 + (size_t)VWARPS * CH_WORDS * act_ws(ncols) * 4 +
             (size_t)VWARPS * 16 * k * 4 + (size_t)VWARPS * LBX_MAX_TOKENS * 4 + 8 + 16;
  return b;
}

static int run_batch(const lbx_proj *projs, const lbx_linear_args *a, int tok0, int k, void *ws,
                     cudaStream_t stream) {
  const int n_proj = a->n_proj;
  const int K = projs[0].in_features;
  const int ncols = 2 * k;
  const int ncb = (ncols + 7) / 8;
  const int esz_x = a->x_dtype == LBX_F32 ? 4 : 2;
  const int esz_y = a->y_dtype == LBX_F32 ? 4 : 2;

  // z scratch layout
  float *zp[LBX_MAX_PROJ][2] = {};
  {
    uint8_t *w = reinterpret_cast<uint8_t *>(ws);
    for (int i = 0; i < n_proj; ++i)
      for (int b = 0; b < projs[i].n_branches; ++b) {
        zp[i][b] = reinterpret_cast<float *>(w);
        w += (((size_t)projs[i].br[b].rank * k * 4) + 255) & ~(size_t)255;
      }
  }

  // ---------------- V-stage
  VParams vp = {};
  vp.K = K;
  vp.Wv = K / 32;
  vp.pitch = row_pitch(vp.Wv);
  vp.nch = (vp.Wv + CH_WORDS - 1) / CH_WORDS;
  vp.k = k;
  vp.ncols = ncols;
  vp.xdt = a->x_dtype;
  vp.prologue = a->prologue;
  vp.eps = a->eps;
  vp.x = reinterpret_cast<const uint8_t *>(a->x) + (size_t)tok0 * K * esz_x;
  vp.x2 = a->x2 ? reinterpret_cast<const uint8_t *>(a->x2) + (size_t)tok0 * K * esz_x : nullptr;
  vp.norm_w = a->norm_w;
  int tiles = 0;
  for (int i = 0; i < n_proj; ++i) {
    const lbx_proj &pr = projs[i];
    for (int b = 0; b < pr.n_branches; ++b) {
      if (!pr.br[b].v_sign) continue;
      VSeg &sg = vp.seg[vp.nseg++];
      sg.v_sign = pr.br[b].v_sign;
      sg.v2 = pr.br[b].v2;
      sg.mid0 = pr.br[b].mid;
      sg.z0 = zp[i][b];
      sg.rank = pr.br[b].rank;
      if (b == 0 && pr.n_branches == 2 && !pr.br[1].v_sign) {
        sg.mid1 = pr.br[1].mid;
        sg.z1 = zp[i][1];
      }
      sg.tile0 = tiles;
      tiles += (sg.rank + 15) / 16;
    }
  }
  const size_t vsmem = vstage_smem(vp.Wv, ncols, k);
  LBX_CHECK_SUP(vsmem <= 227 * 1024, "V-stage needs %zu bytes of shared memory", vsmem);

  // ---------------- U-stage
  UParams up = {};
  up.k = k;
  up.ncols = ncols;
  up.ydt = a->y_dtype;
  up.epi = a->epilogue;
  int maxw[2] = {0, 0}, maxtile = 0;
  for (int i = 0; i < n_proj; ++i) {
    const lbx_proj &pr = projs[i];
    USeg &sg = up.seg[i];
    sg.nbr = pr.n_branches;
    sg.out = pr.out_features;
    sg.bias = pr.bias;
    sg.y = reinterpret_cast<uint8_t *>(a->y[i]) +
           (size_t)tok0 * (a->y_ld[i] ? a->y_ld[i] : pr.out_features) * esz_y;
    sg.y_ld = a->y_ld[i] ? a->y_ld[i] : pr.out_features;
    int tw = 0;
    for (int b = 0; b < pr.n_branches; ++b) {
      sg.u_sign[b] = pr.br[b].u_sign;
      sg.u1[b] = pr.br[b].u1;
      sg.z[b] = zp[i][b];
      sg.rank[b] = pr.br[b].rank;
      sg.words[b] = (pr.br[b].rank + 31) / 32;
      sg.perrow[b] = (sg.words[b] % 4) == 0;
      sg.pitch[b] = sg.perrow[b] ? row_pitch(sg.words[b]) : sg.words[b];
      maxw[b] = std::max(maxw[b], 4 * ((sg.words[b] + 3) / 4));
      tw += 16 * sg.pitch[b] + 4;
    }
    maxtile = std::max(maxtile, tw);
  }
  up.act_words[0] = maxw[0];
  up.act_words[1] = maxw[1];
  up.wtile_words = (maxtile + 3) & ~3;
  int uw = UWARPS_MAX;
  size_t usmem = 0;
  for (; uw >= 1; uw >>= 1) {
    usmem = (size_t)(maxw[0] + maxw[1]) * act_ws(ncols) * 4 + (size_t)uw * up.wtile_words * 4 +
            (size_t)uw * 8 + 16;
    if (usmem <= 227 * 1024) break;
  }
  LBX_CHECK_SUP(uw >= 1, "U-stage needs too much shared memory (rank too large for k=%d)", k);
  up.uwarps = uw;
  int ctas = 0;
  for (int i = 0; i < n_proj; ++i) {
    up.seg[i].cta0 = ctas;
    ctas += (projs[i].out_features + 16 * uw - 1) / (16 * uw);
  }
  up.nseg = n_proj;

  const bool pdl = a->use_pdl != 0;
  cudaError_t e;
  auto vk = ncb == 1 ? vstage_kernel<1> : ncb == 2 ? vstage_kernel<2> : vstage_kernel<4>;
  auto uk = ncb == 1 ? ustage_kernel<1> : ncb == 2 ? ustage_kernel<2> : ustage_kernel<4>;
  e = cudaFuncSetAttribute(vk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vsmem);
  if (e != cudaSuccess) return cuda_status(e, "vstage smem attribute");
  e = cudaFuncSetAttribute(uk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)usmem);
  if (e != cudaSuccess) return cuda_status(e, "ustage smem attribute");
  e = launch(vk, dim3(tiles), dim3(VWARPS * 32), vsmem, stream, pdl, vp);
  if (e != cudaSuccess) return cuda_status(e, "vstage launch");
  e = launch(uk, dim3(ctas), dim3(uw * 32), usmem, stream, pdl, up);
  if (e != cudaSuccess) return cuda_status(e, "ustage launch");
  return LBX_OK;
}

}  // namespace lbx

extern "C" size_t lbx_linear_workspace_size(const lbx_proj *projs, int32_t n_proj,
                                            int32_t n_tokens) {
  if (!projs || n_proj < 1 || n_proj > LBX_MAX_PROJ || n_tokens < 1) return 0;
  const int k = n_tokens < LBX_MAX_TOKENS ? n_tokens : LBX_MAX_TOKENS;
  return lbx::z_bytes(projs, n_proj, k);
}

extern "C" int lbx_linear_verify(const lbx_proj *projs, const lbx_linear_args *a, void *ws,
                                 size_t ws_bytes, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(a, "args is NULL");
  int rc = validate(projs, a->n_proj);
  if (rc) return rc;
  LBX_CHECK_ARG(a->n_tokens >= 1, "n_tokens must be >= 1");
  LBX_CHECK_ARG(a->x, "x is NULL");
  LBX_CHECK_ARG(a->x_dtype == LBX_F32 || a->x_dtype == LBX_BF16, "bad x_dtype");
  LBX_CHECK_ARG(a->y_dtype == LBX_F32 || a->y_dtype == LBX_BF16, "bad y_dtype");
  LBX_CHECK_ARG(a->prologue >= LBX_PRO_NONE && a->prologue <= LBX_PRO_SILU_MUL, "bad prologue");
  LBX_CHECK_ARG(a->prologue != LBX_PRO_RMSNORM || a->norm_w, "RMSNorm prologue needs norm_w");
  LBX_CHECK_ARG(a->prologue != LBX_PRO_SILU_MUL || a->x2, "SiLU-mul prologue needs x2");
  LBX_CHECK_ARG(a->epilogue == LBX_EPI_STORE || (a->epilogue == LBX_EPI_ADD && a->y_dtype == LBX_F32),
                "bad epilogue (ADD needs fp32 y)");
  for (int i = 0; i < a->n_proj; ++i) LBX_CHECK_ARG(a->y[i], "y[%d] is NULL", i);
  const size_t need = lbx_linear_workspace_size(projs, a->n_proj, a->n_tokens);
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  for (int t0 = 0; t0 < a->n_tokens; t0 += LBX_MAX_TOKENS) {
    const int k = std::min(LBX_MAX_TOKENS, a->n_tokens - t0);
    rc = run_batch(projs, a, t0, k, ws, stream);
    if (rc) return rc;
  }
  return LBX_OK;
}

extern "C" int lbx_linear(const lbx_proj *projs, const lbx_linear_args *a, void *ws,
                          size_t ws_bytes, cudaStream_t stream) {
  return lbx_linear_verify(projs, a, ws, ws_bytes, stream);
}
