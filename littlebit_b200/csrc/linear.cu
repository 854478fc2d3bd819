// LittleBitLinear on packed sign words for sm_100a.
//
// y = u1 ⊙ U_sign·(mid ⊙ V_sign·(v2 ⊙ x))  (+ residual branch) (+ bias)
// Reference: quantization/modules/littlebit.py:95-121 (fp32 semantics) and
// patches/littlebit_cpu_optimized.cpp:598-701 (packed-word CPU kernel).
//
// One call = two stages, each a grid of independent units; standalone they are
// two kernels chained with programmatic dependent launch (PDL), and a
// persistent program (program.cu) runs the same unit bodies as phases:
//   V-stage  CTA = 16 rank rows x all of K, warp = 256-column blocks:
//            z_b = mid_b ⊙ (V_sign · a) [⊙ rsqrt(mean x^2 + eps) for a fused
//            RMSNorm],  a = v2 ⊙ prologue(x);  blocks summed in fixed order
//            (K > 4096 on a small grid: a cluster per unit, one CTA per
//            4096-column pass, vsplit_kernel; same sums, same order)
//   U-stage  CTA = ut 16-row output tiles, its 16 warps split tiles x ranks:
//            y = Σ_b u1_b ⊙ U_b · z_b (+ bias)
// Both contractions run on the int8 tensor cores:
//   * activations are quantised to 16-bit integers (two int8 digits); the
//     V-stage uses one scale per token per 256 columns, the U-stage a power
//     of two per token per 128-rank group, so every Σ_j s_j·q_j inside a
//     scale block is EXACT (U groups are then combined by exact integer shifts);
//   * a sign word is expanded in registers by one prmt per 4 signs into int8
//     0/−1 (= −bit), and mma.m16n8k32.s8 gives D = Σ_j (−b_j)·digit_j;
//   * Σ_j s_j q_j = Σ_j q_j + 2·(256·D_hi + D_lo).
// Block results are combined in a fixed order, so a token's output does not
// depend on how many tokens share the launch (verify batch == batch 1, bit for
// bit) and repeated calls are deterministic.
//
// All weights of a unit (sign words and scale vectors) are requested with
// cp.async.bulk into a shared-memory weight region before the unit's inputs
// exist (before griddepcontrol.wait, or before the preceding grid barrier), so
// their HBM latency overlaps the preceding work.

#include <algorithm>

#include "common.cuh"

namespace lbx {

constexpr int PASS_WORDS = 128; // V-stage staging pass: 4096 columns (512 threads x 8)
constexpr int BLK_WORDS = 8;    // V-stage scale block: 256 columns (one warp)
constexpr int VWARPS = 16;
constexpr int VTHREADS = VWARPS * 32;
constexpr int TBATCH = 2;       // tokens whose x loads are issued together in staging
constexpr int VCAP_MAX = 4096;  // leading v2/norm_w columns prefetched into shared memory (the rest
                                // come from L2 with the x loads: keeps wide inputs at 2 CTAs per SM)
constexpr int UWARPS = 16;      // warp (tile, split): ut row tiles x (16/ut) rank splits
constexpr int UTHREADS = UWARPS * 32;
constexpr int UT_MAX = 8;
constexpr int UGRP = 128;       // U-stage quantisation group: 128 ranks (4 sign words) of one branch
constexpr int ZGMAX = 64;       // quantisation groups per branch (rank <= 8192)
constexpr int LBX_MAX_PEERS = 8;

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
  const float *mid1;     // [rank] (shared-V residual) or nullptr
  float *z0;             // [k][rank]
  float *z1;             // [k][rank] or nullptr
  int *tmax;             // [tile][2][k] per-unit max |z0|, |z1| per token (float bits)
  int rank;
  int unit0;             // first unit (vt 16-row tiles) of this segment
};

struct VParams {
  VSeg seg[2 * LBX_MAX_PROJ];
  int nseg;
  int K, Wv, vpitch;
  int vt;                // 16-row tiles per unit (1 or 2)
  int vcap;              // columns of v2 / norm_w staged in shared memory
  int k, ncols;
  int xdt, prologue;
  float eps;
  const void *x;
  const void *x2;
  const float *norm_w;
  int s_bytes;           // shared-memory scratch region of a standalone launch (weights follow)
  int split;             // pass-split launch: one staging pass per CTA, a cluster per unit
};

struct USeg {
  const int32_t *u_sign[2];
  const float *u1[2];
  const float *z[2];     // [k][rank] from the V-stage
  const int *tmax[2];    // per-unit maxima [tile][2][k] of the V segment that produced z[b] (float bits)
  int tsel[2];           // which of the two per-unit maxima belongs to z[b]
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
  int k, ncols, ydt, epi;
  int ut;             // row tiles per CTA (warps split the ranks 16/ut ways)
  int act_words[2];   // max over projections of 4*ceil(words/4)
  int wtile_words;    // per-tile weight region (words)
  int ugm;            // max quantisation groups of a branch (scratch arrays [2][ugm][k])
  int s_bytes;        // shared-memory scratch region of a standalone launch (weights follow)
  // fused all-gather of a row-sharded layer (one projection): every result
  // goes to each rank's exchange buffer as one 8-byte word (call number << 32
  // | fp32 bits); the buffer half is the call number's parity
  int npeer;
  const unsigned *seq;  // completed calls of this rank (written by the unpack kernel)
  long long xhalf;      // words per exchange-buffer half
  unsigned long long *xbuf[LBX_MAX_PEERS];
};

// ---------------------------------------------------------------------------
// shared contraction: one warp, rows g and g+8 of a 16-row sign tile
// ---------------------------------------------------------------------------
// Consumes groups [g0, g1) of 4 words.  Thread (g,q) reads word 4G+q of its two
// rows; its 8 prmt expansions feed 4 MMA k-steps.  The activation layout puts,
// for word w, slot s=(h*4+j), column c, the 4 digits of reduction positions
// 32w+16h+j+{0,4,8,12} into one uint32, matching the A-fragment bytes.
// Single-column-block form (k <= 4 tokens): NG groups run side by side, their
// MMAs issued interleaved k-step by k-step so that the NG accumulator chains
// overlap in the tensor pipe; the A fragments come from the shift-light table
// expansion.
template <int R, int NG>
LBX_DEV void sign_kstep1(int (&acc)[NG][4], const uint32_t (&wa)[NG], const uint32_t (&wb)[NG],
                         const uint32_t *const (&aw)[NG], int ncols, int n8) {
  constexpr int slot = 4 * (R >> 1) + 2 * (R & 1);
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    uint32_t a0, a1, a2, a3;
    sign_frag<R>(wa[i], a0, a2);
    sign_frag<R>(wb[i], a1, a3);
    uint32_t b0 = 0, b1 = 0;
    if (n8 < ncols) {
      b0 = aw[i][slot * ncols + n8];
      b1 = aw[i][(slot + 1) * ncols + n8];
    }
    mma_s8(acc[i], a0, a1, a2, a3, b0, b1);
  }
}
// swz: the sign rows' words are stored permuted (word w of the rows at w ^ swz;
// the fused chain's V tiles swap the two 4-word halves of rows 4-7 and 12-15
// so that the fragment loads hit distinct banks without a padded pitch)
template <int NG>
LBX_DEV void sign_mma1(int (&acc)[NG][4], const uint32_t *rowg, const uint32_t *rowg8,
                       const uint32_t *act, int ws, int ncols, const int (&G)[NG], int lane, int swz = 0) {
  const int q = lane & 3, n8 = lane >> 2;
  uint32_t wa[NG], wb[NG];
  const uint32_t *aw[NG];
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    const int w = 4 * G[i] + q;
    wa[i] = rowg[w ^ swz];
    wb[i] = rowg8[w ^ swz];
    aw[i] = act + w * ws;
  }
  sign_kstep1<0, NG>(acc, wa, wb, aw, ncols, n8);
  sign_kstep1<1, NG>(acc, wa, wb, aw, ncols, n8);
  sign_kstep1<2, NG>(acc, wa, wb, aw, ncols, n8);
  sign_kstep1<3, NG>(acc, wa, wb, aw, ncols, n8);
}

// Groups [g0, g1) summed into acc.  One column block: pairs of groups as two
// interleaved chains.  Two or four blocks (already 2 or 4 independent chains
// per k-step): even and odd groups into separate accumulators with the
// per-bit-shift expansion, whose fewer live registers keep these widths from
// spilling.  The int32 sums are exact, so none of this changes a bit.
template <int NCB>
LBX_DEV void sign_mma(int (&acc)[NCB][4], const uint32_t *rowg, const uint32_t *rowg8,
                      const uint32_t *act, int ws, int ncols, int g0, int g1, int lane) {
  if constexpr (NCB == 1) {
    int G = g0;
    for (; G + 1 < g1; G += 2) {
      int a2[2][4] = {};
      const int gg[2] = {G, G + 1};
      sign_mma1<2>(a2, rowg, rowg8, act, ws, ncols, gg, lane);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[0][e] += a2[0][e] + a2[1][e];
    }
    if (G < g1) {
      const int gg[1] = {G};
      sign_mma1<1>(acc, rowg, rowg8, act, ws, ncols, gg, lane);
    }
    return;
  }
  const int q = lane & 3;
  const int n8 = lane >> 2;
  int acc2[NCB][4];
#pragma unroll
  for (int cb = 0; cb < NCB; ++cb) acc2[cb][0] = acc2[cb][1] = acc2[cb][2] = acc2[cb][3] = 0;
  auto group = [&](int G, int (&ac)[NCB][4]) {
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
        mma_s8(ac[cb], a0, a1, a2, a3, b0, b1);
      }
    }
  };
  int G = g0;
  for (; G + 1 < g1; G += 2) {
    group(G, acc);
    group(G + 1, acc2);
  }
  if (G < g1) group(G, acc);
#pragma unroll
  for (int cb = 0; cb < NCB; ++cb)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[cb][e] += acc2[cb][e];
}

LBX_DEV uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) |
         ((uint32_t)(d & 255) << 24);
}

// activations (written by the preceding kernel): L2 loads
LBX_DEV void load8(const void *p, int dtype, int64_t i, float (&v)[8]) {
  if (dtype == LBX_F32) {
    const float4 *s = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + i);
    const float4 a = __ldcg(s), b = __ldcg(s + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = __ldcg(reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(p) + i));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[2 * e] = __uint_as_float(w[e] << 16);
      v[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
    }
  }
}

LBX_DEV void load8f(const float *p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
  const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// partial-sum loads of data written by the preceding kernel: L2 only
LBX_DEV void load8cg(const float *p, float (&v)[8]) {
  const float4 a = __ldcg(reinterpret_cast<const float4 *>(p));
  const float4 b = __ldcg(reinterpret_cast<const float4 *>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// ---------------------------------------------------------------------------
// per-CTA state shared by the stage bodies (static shared memory of the
// launching kernel): scale scratch and the mbarriers of the weight copies.
// bar[0..UT_MAX) serve the U-stage tiles, bar[UT_MAX] the V-stage; par[] is
// the phase parity each barrier will complete next, so one barrier serves any
// number of units of a persistent CTA.
// ---------------------------------------------------------------------------
struct LinShm {
  float v_inv[VWARPS][LBX_MAX_TOKENS];
  int v_sq[VWARPS][LBX_MAX_TOKENS];
  float v_ssq[VWARPS][LBX_MAX_TOKENS];
  int v_zmax[2][LBX_MAX_TOKENS];
  int u_ec[2][LBX_MAX_TOKENS];  // per (branch, token): the coarsest group exponent
  __align__(8) uint64_t bar[UT_MAX + 1];
  uint32_t par[UT_MAX + 1];
};

LBX_DEV void linshm_init(LinShm &sh) {
  if (threadIdx.x <= UT_MAX) {
    mbar_init(&sh.bar[threadIdx.x], 1);
    sh.par[threadIdx.x] = 0;
    fence_mbar_init();
  }
  __syncthreads();
}

// shared-memory regions of a V-stage unit: W (weights, filled by bulk copies
// that may be issued long before the unit runs) and S (scratch of the run)
struct VLayout {
  uint32_t *wbuf;  // 16 vt x vpitch sign words
  float *sv2;      // vcap
  float *snw;      // vcap (RMSNorm prologue)
  float *smid;     // 2 x 16 vt (mid0 rows, then mid1 rows)
  uint32_t *act;   // PASS_WORDS x ws
  float *red;      // VWARPS x 16 x k
};

LBX_DEV VLayout vlayout(const VParams &p, uint8_t *W, uint8_t *S) {
  VLayout L;
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  L.wbuf = reinterpret_cast<uint32_t *>(W);
  L.sv2 = reinterpret_cast<float *>(L.wbuf + 16 * p.vt * p.vpitch);
  L.snw = L.sv2 + p.vcap;
  L.smid = L.snw + (rms ? p.vcap : 0);
  L.act = reinterpret_cast<uint32_t *>(S);
  L.red = reinterpret_cast<float *>(L.act + PASS_WORDS * act_ws(p.ncols));
  return L;
}

LBX_DEV int vseg_of(const VParams &p, int unit) {
  int s = 0;
  while (s + 1 < p.nseg && unit >= p.seg[s + 1].unit0) ++s;
  return s;
}

// the weights of V-stage unit `unit` (sign rows, v2, norm_w, mid): independent
// of every activation, so they may be requested before the inputs exist
LBX_DEV void vstage_issue(const VParams &p, int unit, uint8_t *W, LinShm &sh) {
  const int tid = threadIdx.x;
  const VSeg &sg = p.seg[vseg_of(p, unit)];
  const int row0 = (unit - sg.unit0) * 16 * p.vt;
  const int rows = min(16 * p.vt, sg.rank - row0);
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const VLayout L = vlayout(p, W, nullptr);
  const int vcap = p.vcap;
  uint64_t *bar = &sh.bar[UT_MAX];
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)rows * p.Wv * 4u + (uint32_t)vcap * 4u * (rms ? 2u : 1u) +
                           (uint32_t)rows * 4u * (sg.mid1 ? 2u : 1u);
    mbar_arrive_expect_tx(bar, bytes);
  }
  __syncthreads();
  if (tid < rows)
    bulk_g2s(L.wbuf + tid * p.vpitch, sg.v_sign + (int64_t)(row0 + tid) * p.Wv, (uint32_t)p.Wv * 4u, bar);
  else if (tid == VTHREADS - 1)
    bulk_g2s(L.sv2, sg.v2, (uint32_t)vcap * 4u, bar);
  else if (tid == VTHREADS - 2 && rms)
    bulk_g2s(L.snw, p.norm_w, (uint32_t)vcap * 4u, bar);
  else if (tid == VTHREADS - 3)
    bulk_g2s(L.smid, sg.mid0 + row0, (uint32_t)rows * 4u, bar);
  else if (tid == VTHREADS - 4 && sg.mid1)
    bulk_g2s(L.smid + 16 * p.vt, sg.mid1 + row0, (uint32_t)rows * 4u, bar);
}

// One staging pass of the V-stage: every token's a = v2 ⊙ prologue(x) over
// the (up to) 4096 columns of pass `pass`, as int8 digit pairs in act, with
// the per-(warp, token) scale, digit sum and RMSNorm sum of squares in sh.
// Thread t stages columns 8*(t%4)..+8 of word t/4; warp w = one 256-column
// scale block.  on_first() runs once, after the first tokens' x loads are
// issued and before v2 is used (the V-stage waits for its weight copies
// there).  Columns below p.vcap take v2 / norm_w from the shared-memory
// copies sv2 / snw, the rest from global memory (same arithmetic).
// prologue kinds of the V-stage staging (compile-time: the second input
// array costs registers)
constexpr int PM_X = 0;     // x (optionally RMSNorm'd)
constexpr int PM_SILU = 1;  // silu(x) * x2
constexpr int PM_MUL = 2;   // x * x2
__host__ __device__ inline int pm_of(int prologue) {
  return prologue == LBX_PRO_SILU_MUL ? PM_SILU : prologue == LBX_PRO_MUL ? PM_MUL : PM_X;
}

template <int PM, class OnFirst>
// vcap_arg >= 0: columns below it read v2 / norm_w from sv2 / snw (the
// pass-split kernel passes shared-memory copies of its own pass)
LBX_DEV void vstage_stage(const VParams &p, const float *v2, const float *sv2, const float *snw,
                          int pass, uint32_t *act, LinShm &sh, OnFirst &&on_first, int vcap_arg = -1) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const int ws = act_ws(p.ncols);
  const int vcap = vcap_arg >= 0 ? vcap_arg : p.vcap;
  const int Wd = tid >> 2, qq = tid & 3;
  const int hh = qq >> 1;
  const bool low = (qq & 1) == 0;  // my digits are bytes 0,1 (else 2,3) of the slot words
  const int pw0 = pass * PASS_WORDS;
  const int pwords = min(PASS_WORDS, p.Wv - pw0);
  const bool wvalid = Wd < pwords;
  const int64_t col = (int64_t)(pw0 + Wd) * 32 + 8 * qq;
  float hw[8];
  for (int t0 = 0; t0 < p.k; t0 += TBATCH) {
    // issue the loads of a batch of tokens before using any of them
    float xv[TBATCH][8], uv[PM != PM_X ? TBATCH : 1][8];
#pragma unroll
    for (int j = 0; j < TBATCH; ++j) {
      if (wvalid && t0 + j < p.k) {
        load8(p.x, p.xdt, (int64_t)(t0 + j) * p.K + col, xv[j]);
        if constexpr (PM != PM_X) load8(p.x2, p.xdt, (int64_t)(t0 + j) * p.K + col, uv[j]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xv[j][i] = 0.f;
          if constexpr (PM != PM_X) uv[j][i] = 0.f;
        }
      }
    }

    if (t0 == 0) {
      on_first();
      if (!wvalid) {
#pragma unroll
        for (int i = 0; i < 8; ++i) hw[i] = 0.f;
      } else if (col < vcap) {
        const float4 *v4 = reinterpret_cast<const float4 *>(sv2 + col);
        const float4 a0 = v4[0], a1 = v4[1];
        hw[0] = a0.x; hw[1] = a0.y; hw[2] = a0.z; hw[3] = a0.w;
        hw[4] = a1.x; hw[5] = a1.y; hw[6] = a1.z; hw[7] = a1.w;
        if (rms) {
          const float4 *n4 = reinterpret_cast<const float4 *>(snw + col);
          const float4 b0 = n4[0], b1 = n4[1];
          hw[0] *= b0.x; hw[1] *= b0.y; hw[2] *= b0.z; hw[3] *= b0.w;
          hw[4] *= b1.x; hw[5] *= b1.y; hw[6] *= b1.z; hw[7] *= b1.w;
        }
      } else {  // columns beyond the shared-memory copy (very wide inputs)
        load8f(v2 + col, hw);
        if (rms) {
          float nw[8];
          load8f(p.norm_w + col, nw);
#pragma unroll
          for (int i = 0; i < 8; ++i) hw[i] *= nw[i];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < TBATCH; ++j) {
      const int t = t0 + j;
      if (t >= p.k) break;  // uniform across the CTA
      float a[8];
      float sq2 = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xx = xv[j][i];
        if constexpr (PM == PM_SILU) {
          a[i] = (xx / (1.0f + expf(-xx))) * uv[j][i] * hw[i];
        } else if constexpr (PM == PM_MUL) {
          a[i] = xx * uv[j][i] * hw[i];
        } else {
          sq2 = fmaf(xx, xx, sq2);
          a[i] = xx * hw[i];
        }
      }
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(a[i]));
      m = __int_as_float(__reduce_max_sync(0xffffffffu, __float_as_int(m)));
      const float sc = m > 0.f ? QMAX / m : 0.f;
      int hi[8], lo[8], sqi = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int qv = __float2int_rn(a[i] * sc);
        sqi += qv;
        split_digits(qv, hi[i], lo[i]);
      }
      // 16-bit halves of the 4 slot words (h, j): bytes = columns j and j+4
      uint32_t H[2], Lw[2];
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        const int j0 = 2 * jp, j1 = 2 * jp + 1;
        H[jp] = ((hi[j0] & 255) | ((hi[j0 + 4] & 255) << 8)) |
                (((hi[j1] & 255) | ((hi[j1 + 4] & 255) << 8)) << 16);
        Lw[jp] = ((lo[j0] & 255) | ((lo[j0 + 4] & 255) << 8)) |
                 (((lo[j1] & 255) | ((lo[j1 + 4] & 255) << 8)) << 16);
      }
      const uint32_t PH0 = __shfl_xor_sync(0xffffffffu, H[0], 1);
      const uint32_t PH1 = __shfl_xor_sync(0xffffffffu, H[1], 1);
      const uint32_t PL0 = __shfl_xor_sync(0xffffffffu, Lw[0], 1);
      const uint32_t PL1 = __shfl_xor_sync(0xffffffffu, Lw[1], 1);
      uint32_t *aw = act + Wd * ws + 2 * t;
      if (low) {  // slots j = 0, 1: my half low, partner's high
        aw[(4 * hh + 0) * p.ncols] = (H[0] & 0xFFFFu) | (PH0 << 16);
        aw[(4 * hh + 0) * p.ncols + 1] = (Lw[0] & 0xFFFFu) | (PL0 << 16);
        aw[(4 * hh + 1) * p.ncols] = (H[0] >> 16) | (PH0 & 0xFFFF0000u);
        aw[(4 * hh + 1) * p.ncols + 1] = (Lw[0] >> 16) | (PL0 & 0xFFFF0000u);
      } else {    // slots j = 2, 3: partner's half low, mine high
        aw[(4 * hh + 2) * p.ncols] = (PH1 & 0xFFFFu) | (H[1] << 16);
        aw[(4 * hh + 2) * p.ncols + 1] = (PL1 & 0xFFFFu) | (Lw[1] << 16);
        aw[(4 * hh + 3) * p.ncols] = (PH1 >> 16) | (H[1] & 0xFFFF0000u);
        aw[(4 * hh + 3) * p.ncols + 1] = (PL1 >> 16) | (Lw[1] & 0xFFFF0000u);
      }
      sqi = __reduce_add_sync(0xffffffffu, sqi);
      if (rms) sq2 = warp_sum(sq2);
      if (lane == 0) {
        sh.v_inv[warp][t] = m / QMAX;
        sh.v_sq[warp][t] = sqi;
        sh.v_ssq[warp][t] += sq2;
      }
    }
  }
}

// z = mid ⊙ (V_sign · a) for the 16 rows of unit `unit`; returns false (on
// every thread) if the weight copies did not arrive in time
// PM: the prologue kind (PM_X / PM_SILU / PM_MUL).  VT: 16-row tiles per unit
// (p.vt); every tile gets exactly the one-tile arithmetic, x is staged once.
template <int NCB, int PM, int VT = 1>
LBX_DEV bool vstage_run(const VParams &p, int unit, uint8_t *W, uint8_t *S, LinShm &sh, bool zero = true) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const VSeg &sg = p.seg[vseg_of(p, unit)];
  const int row0 = (unit - sg.unit0) * 16 * VT;
  const int ntl = min(VT, (sg.rank - row0 + 15) / 16);
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const int ws = act_ws(p.ncols);
  const VLayout L = vlayout(p, W, S);
  uint32_t *wbuf = L.wbuf, *act = L.act;
  float *sv2 = L.sv2, *snw = L.snw, *red = L.red;
  const uint32_t par = sh.par[UT_MAX];
  if (zero) {  // per-unit scratch (standalone kernels clear it before their wait)
    if (tid < VWARPS * LBX_MAX_TOKENS) (&sh.v_ssq[0][0])[tid] = 0.f;
    if (tid < 2 * LBX_MAX_TOKENS) (&sh.v_zmax[0][0])[tid] = 0;
    __syncthreads();
  }
  LBX_PROBE(1);

  float tacc[VT][NCB][2];
#pragma unroll
  for (int tl = 0; tl < VT; ++tl)
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) tacc[tl][cb][0] = tacc[tl][cb][1] = 0.f;
  bool ok = true;
  const int npass = (p.Wv + PASS_WORDS - 1) / PASS_WORDS;
  for (int pass = 0; pass < npass; ++pass) {
    const int pw0 = pass * PASS_WORDS;
    const int pwords = min(PASS_WORDS, p.Wv - pw0);
    vstage_stage<PM>(p, sg.v2, sv2, snw, pass, act, sh, [&] {
      if (pass == 0) {
        ok = __syncthreads_and(mbar_wait_bounded(&sh.bar[UT_MAX], par, 0x101));
        LBX_PROBE(2);
      }
    });
    __syncthreads();
    LBX_PROBE(3);
    // MMA: warp w contracts its own 256-column block of this pass, every tile
    if (ok && BLK_WORDS * warp < pwords) {
      const int wb = pw0 + BLK_WORDS * warp;
      const int ng = min(BLK_WORDS, pwords - BLK_WORDS * warp) / 4;
#pragma unroll
      for (int tl = 0; tl < VT; ++tl) {
        if (tl < ntl) {
          int acc[NCB][4];
#pragma unroll
          for (int cb = 0; cb < NCB; ++cb) acc[cb][0] = acc[cb][1] = acc[cb][2] = acc[cb][3] = 0;
          const uint32_t *wt = wbuf + tl * 16 * p.vpitch + wb;
          sign_mma<NCB>(acc, wt + g * p.vpitch, wt + (g + 8) * p.vpitch, act + BLK_WORDS * warp * ws, ws,
                        p.ncols, 0, ng, lane);
#pragma unroll
          for (int cb = 0; cb < NCB; ++cb) {
            const int t = cb * 4 + q;
            if (t < p.k) {
              // each pass's product is rounded on its own before it joins the
              // running sum (no fused multiply-add), so a sum of the per-pass
              // partials in pass order (the pass-split kernel) gives these bits
              const int sq = sh.v_sq[warp][t];
              const float inv = sh.v_inv[warp][t];
              tacc[tl][cb][0] += __fmul_rn(__int2float_rn(sq + 2 * (256 * acc[cb][0] + acc[cb][1])), inv);
              tacc[tl][cb][1] += __fmul_rn(__int2float_rn(sq + 2 * (256 * acc[cb][2] + acc[cb][3])), inv);
            }
          }
        }
      }
    }
    __syncthreads();
  }
  // the weight barrier completed its phase (or timed out on every thread)
  if (tid == 0) sh.par[UT_MAX] = par ^ 1u;
  if (!ok) return false;
  // ---- per tile: fixed-order reduction over the 16 warps, then scales
  const float *smid = L.smid;
#pragma unroll
  for (int tl = 0; tl < VT; ++tl) {
    if (tl >= ntl) break;  // uniform across the CTA
    const int trow = row0 + tl * 16;
    const int rows = min(16, sg.rank - trow);
    float *rw = red + warp * 16 * p.k;
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) {
      const int t = cb * 4 + q;
      if (t < p.k) {
        rw[g * p.k + t] = tacc[tl][cb][0];
        rw[(g + 8) * p.k + t] = tacc[tl][cb][1];
      }
    }
    __syncthreads();
    LBX_PROBE(4);
    for (int i = tid; i < rows * p.k; i += VTHREADS) {
      const int rr = i / p.k, t = i - rr * p.k;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < VWARPS; ++w) v += red[(w * 16 + rr) * p.k + t];
      if (rms) {
        float s2 = 0.f;
#pragma unroll
        for (int w = 0; w < VWARPS; ++w) s2 += sh.v_ssq[w][t];
        v *= rsqrtf(s2 / (float)p.K + p.eps);
      }
      const float z0 = smid[tl * 16 + rr] * v;
      sg.z0[(int64_t)t * sg.rank + trow + rr] = z0;
      atomicMax(&sh.v_zmax[0][t], __float_as_int(fabsf(z0)));
      if (sg.z1) {
        const float z1 = smid[16 * VT + tl * 16 + rr] * v;
        sg.z1[(int64_t)t * sg.rank + trow + rr] = z1;
        atomicMax(&sh.v_zmax[1][t], __float_as_int(fabsf(z1)));
      }
    }
    __syncthreads();
    if (tid < p.k) {  // this tile's maxima: plain stores, overwritten by every call (nothing to reset)
      int *tm = sg.tmax + (int64_t)(trow / 16) * 2 * p.k;
      tm[tid] = sh.v_zmax[0][tid];
      if (sg.z1) tm[p.k + tid] = sh.v_zmax[1][tid];
      sh.v_zmax[0][tid] = sh.v_zmax[1][tid] = 0;  // (read and cleared by the same thread)
    }
  }
  LBX_PROBE(5);
  return true;
}

template <int NCB, int PM, int VT>
__global__ void __launch_bounds__(VTHREADS, 2) vstage_kernel(const __grid_constant__ VParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ LinShm sh;
  LBX_PROBE(0);
  if (threadIdx.x < VWARPS * LBX_MAX_TOKENS) (&sh.v_ssq[0][0])[threadIdx.x] = 0.f;
  if (threadIdx.x < 2 * LBX_MAX_TOKENS) (&sh.v_zmax[0][0])[threadIdx.x] = 0;
  linshm_init(sh);  // (ends with a CTA barrier)
  // scratch first, weights after: measured faster than the reverse order
  uint8_t *S = smem_raw;
  uint8_t *W = smem_raw + p.s_bytes;
  vstage_issue(p, blockIdx.x, W, sh);
  pdl_trigger();
  pdl_wait();
  vstage_run<NCB, PM, VT>(p, blockIdx.x, W, S, sh, false);
}

// ---------------------------------------------------------------------------
// U-stage
// ---------------------------------------------------------------------------
struct ULayout {
  uint32_t *wt;   // ut x wtile_words
  float *su1;     // ut x 48 (u1_0, u1_1, bias)
  uint32_t *act0, *act1;
  int *ue, *usq;  // [2][ugm][k]: group exponent (UE_NONE: all-zero group), group digit sum
  int *xch;       // [warps][32][2*NCB*4]
};

LBX_DEV ULayout ulayout(const UParams &p, uint8_t *W, uint8_t *S) {
  ULayout L;
  L.wt = reinterpret_cast<uint32_t *>(W);
  L.su1 = reinterpret_cast<float *>(L.wt + p.ut * p.wtile_words);
  const int ws = act_ws(p.ncols);
  L.act0 = reinterpret_cast<uint32_t *>(S);
  L.act1 = L.act0 + p.act_words[0] * ws;
  L.ue = reinterpret_cast<int *>(L.act1 + p.act_words[1] * ws);
  L.usq = L.ue + 2 * p.ugm * p.k;
  L.xch = L.usq + 2 * p.ugm * p.k;
  return L;
}

constexpr int UE_NONE = 0x7fffffff;  // exponent of an all-zero quantisation group

// largest e with m * 2^e <= QMAX (m > 0), within the normal exponents
LBX_DEV int u_group_exp(float m) {
  int em;
  frexpf(m, &em);  // m = f * 2^em, f in [0.5, 1)
  int e = 15 - em;
  if (e > 127) return 127;
  if (ldexpf(m, e) > QMAX) --e;
  return max(e, -126);
}
LBX_DEV float pow2f(int e) { return __int_as_float((e + 127) << 23); }  // e in [-126, 127]
// v / 2^s rounded half up, s >= 0 (|v| < 2^24)
LBX_DEV int rshr(int v, int s) { return s == 0 ? v : s > 30 ? 0 : (v + (1 << (s - 1))) >> s; }

// 2^n as a float for n in [-149, 127] (subnormal below -126), exactly
LBX_DEV float pow2_exact(int n) {
  return n >= -126 ? __int_as_float((n + 127) << 23) : __int_as_float(1 << (n + 149));
}

// One output value from the exact branch sums I_b at exponents e_b: the single
// expression every executor evaluates, so that all of them round alike.  The
// exponents lie in [-126, 127], so each scaling I_b * 2^-e_b is one correctly
// rounded multiply by an exact power of two: the value of ldexpf(I_b, -e_b)
// (which is also correctly rounded), at a fraction of its instructions.
LBX_DEV float u_result(float u1a, int I0, int e0, bool two, float u1b, int I1, int e1, bool has_bias,
                       float bias) {
  float v = u1a * (__int2float_rn(I0) * pow2_exact(-e0));
  if (two) v += u1b * (__int2float_rn(I1) * pow2_exact(-e1));
  if (has_bias) v += bias;
  return v;
}

LBX_DEV int useg_of(const UParams &p, int unit) {
  int s = 0;
  while (s + 1 < p.nseg && unit >= p.seg[s + 1].cta0) ++s;
  return s;
}

LBX_DEV void ustage_issue(const UParams &p, int unit, uint8_t *W, LinShm &sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ut = p.ut;
  const int tile = warp % ut, split = warp / ut;
  const USeg &sg = p.seg[useg_of(p, unit)];
  const int n0 = (unit - sg.cta0) * (16 * ut) + 16 * tile;
  const bool active = n0 < sg.out;
  const ULayout L = ulayout(p, W, nullptr);
  uint32_t *mywt0 = L.wt + tile * p.wtile_words;
  uint32_t *mywt1 = mywt0 + 16 * sg.pitch[0] + 4;
  float *myu1 = L.su1 + tile * 48;
  uint64_t *bar = &sh.bar[tile];
  if (active && split == 0) {
    uint32_t bytes = 0;
    for (int b = 0; b < sg.nbr; ++b) bytes += 16u * sg.words[b] * 4u + 64u;
    if (sg.bias) bytes += 64u;
    if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
    __syncwarp();
    for (int b = 0; b < sg.nbr; ++b) {
      uint32_t *dst = b == 0 ? mywt0 : mywt1;
      const int32_t *src = sg.u_sign[b] + (int64_t)n0 * sg.words[b];
      if (sg.perrow[b]) {
        if (lane < 16)
          bulk_g2s(dst + lane * sg.pitch[b], src + (int64_t)lane * sg.words[b],
                   (uint32_t)sg.words[b] * 4u, bar);
      } else if (lane == 0) {
        bulk_g2s(dst, src, 16u * sg.words[b] * 4u, bar);
      }
      if (lane == 16 + b) bulk_g2s(myu1 + 16 * b, sg.u1[b] + n0, 64u, bar);
    }
    if (lane == 18 && sg.bias) bulk_g2s(myu1 + 32, sg.bias + n0, 64u, bar);
  }
}

template <int NCB, bool PEER = false>
LBX_DEV bool ustage_run(const UParams &p, int unit, int nunits, uint8_t *W, uint8_t *S, LinShm &sh,
                        bool zero = true) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int ut = p.ut, nsplit = UWARPS / ut;
  const int tile = warp % ut, split = warp / ut;
  const int si = useg_of(p, unit);
  const USeg &sg = p.seg[si];
  const int n0 = (unit - sg.cta0) * (16 * ut) + 16 * tile;
  const bool active = n0 < sg.out;
  const int ws = act_ws(p.ncols);
  const ULayout L = ulayout(p, W, S);
  uint32_t *act0 = L.act0, *act1 = L.act1;
  int *xch = L.xch;
  uint32_t *mywt0 = L.wt + tile * p.wtile_words;
  uint32_t *mywt1 = mywt0 + 16 * sg.pitch[0] + 4;
  float *myu1 = L.su1 + tile * 48;
  const int r0 = sg.rank[0], r1 = sg.nbr > 1 ? sg.rank[1] : 0;
  const uint32_t par = sh.par[tile];
  unsigned call = 0;  // this call's number (fused all-gather); loaded early, used in the epilogue
  if constexpr (PEER) call = __ldcg(p.seq) + 1u;
  LBX_PROBE(11);

  // items (t, b, W, slot): each (t, b) segment is a multiple of 32 items, so a
  // warp's 32 items always share (t, b) and reduce with one redux
  const int nw0 = 4 * ((sg.words[0] + 3) / 4);
  const int nw1 = sg.nbr > 1 ? 4 * ((sg.words[1] + 3) / 4) : 0;
  const int per = (nw0 + nw1) * 8;
  const int total = p.k * per;
  constexpr int UB = 2;  // items per thread whose z loads are in flight together
  float zv[UB][4], zn[UB][4];
  auto load_batch = [&](int base0, float (&zd)[UB][4]) {
#pragma unroll
    for (int ib = 0; ib < UB; ++ib) {
      const int i = base0 + ib * UTHREADS + lane;
#pragma unroll
      for (int e = 0; e < 4; ++e) zd[ib][e] = 0.f;
      if (base0 + ib * UTHREADS < total) {  // uniform across the warp
        const int t = i / per, rem = i - t * per;
        const int b = rem < nw0 * 8 ? 0 : 1;
        const int rr = b ? rem - nw0 * 8 : rem;
        const int Wd = rr >> 3, slot = rr & 7;
        const int hh = slot >> 2, jj = slot & 3;
        const int r = b ? r1 : r0;
        const float *zrow = sg.z[b] + (int64_t)t * r;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int pos = 32 * Wd + 16 * hh + jj + 4 * e;
          // standalone: z is read-only in this grid and written by the previous
          // one, so the L1 path absorbs the 4x sector reuse of this pattern;
          // inside a persistent program z is produced in the same launch: L2 only
          if (pos < r) zd[ib][e] = zero ? __ldcg(zrow + pos) : __ldg(zrow + pos);
        }
      }
    }
  };
  // the first batch of z is requested before the scales: both reads share
  // one L2 round trip
  load_batch(warp * 32, zv);

  // ---- quantisation scales: a power of two per (branch, 128-rank group,
  // token) from the V-stage maxima, and per (branch, token) the coarsest one
  const int ng0 = (sg.words[0] + 3) / 4, ng1 = sg.nbr > 1 ? (sg.words[1] + 3) / 4 : 0;
  int *ue = L.ue, *usq = L.usq;
  const int gk = p.ugm * p.k;
  for (int i = tid; i < (ng0 + ng1) * p.k; i += UTHREADS) {
    const int b = i < ng0 * p.k ? 0 : 1;
    const int j = b ? i - ng0 * p.k : i;  // group * k + token
    const int grp = j / p.k, tk = j - grp * p.k;
    // max over the group's (up to) 8 V units: all loads in flight together
    const int nt = (sg.rank[b] + 15) / 16;
    const int *tm = sg.tmax[b] + sg.tsel[b] * p.k + tk;
    int v[UGRP / 16];
#pragma unroll
    for (int e = 0; e < UGRP / 16; ++e) {
      const int tile = grp * (UGRP / 16) + e;
      v[e] = tile < nt ? __ldcg(tm + (int64_t)tile * 2 * p.k) : 0;
    }
    int mm = 0;
#pragma unroll
    for (int e = 0; e < UGRP / 16; ++e) mm = max(mm, v[e]);
    const float m = __int_as_float(mm);
    ue[b * gk + j] = m > 0.f ? u_group_exp(m) : UE_NONE;
    usq[b * gk + j] = 0;
  }
  __syncthreads();
  if (tid < 2 * p.k) {
    const int b = tid / p.k, t = tid - b * p.k;
    const int ng = b ? ng1 : ng0;
    int ec = UE_NONE;
    for (int G = 0; G < ng; ++G) ec = min(ec, ue[b * gk + G * p.k + t]);
    sh.u_ec[b][t] = ec == UE_NONE ? 0 : ec;
  }
  LBX_PROBE(12);
  for (int base0 = warp * 32; base0 < total; base0 += UB * UTHREADS) {
    // the next batch's z loads are in flight while this batch is quantised
    const bool more = base0 + UB * UTHREADS < total;
    if (more) load_batch(base0 + UB * UTHREADS, zn);
#pragma unroll
    for (int ib = 0; ib < UB; ++ib) {
      const int base = base0 + ib * UTHREADS;
      if (base >= total) break;  // uniform across the warp
      const int i = base + lane;
      const int t = i / per, rem = i - t * per;
      const int b = rem < nw0 * 8 ? 0 : 1;
      const int rr = b ? rem - nw0 * 8 : rem;
      const int Wd = rr >> 3, slot = rr & 7;
      const int gi = b * gk + (Wd >> 2) * p.k + t;  // a warp's 32 items are one group
      const int ex = ue[gi];
      const float sc = ex == UE_NONE ? 0.f : pow2f(ex);
      int hi[4], lo[4], sq = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qv = __float2int_rn(zv[ib][e] * sc);
        sq += qv;
        split_digits(qv, hi[e], lo[e]);
      }
      uint32_t *aw = (b ? act1 : act0) + Wd * ws + 2 * t;
      aw[slot * p.ncols] = pack4(hi[0], hi[1], hi[2], hi[3]);
      aw[slot * p.ncols + 1] = pack4(lo[0], lo[1], lo[2], lo[3]);
      sq = __reduce_add_sync(0xffffffffu, sq);
      if (lane == 0) atomicAdd(&usq[gi], sq);
    }
    if (more) {
#pragma unroll
      for (int ib = 0; ib < UB; ++ib)
#pragma unroll
        for (int e = 0; e < 4; ++e) zv[ib][e] = zn[ib][e];
    }
  }
  __syncthreads();

  LBX_PROBE(13);
  bool ok = true;
  if (active) ok = mbar_wait_bounded(&sh.bar[tile], par, 0x201);
  ok = __syncthreads_and(ok);
  // every armed barrier (one per active tile) completed this phase
  if (tid < ut && (unit - sg.cta0) * (16 * ut) + 16 * tid < sg.out) sh.par[tid] ^= 1u;
  LBX_PROBE(14);

  // ---- contraction: every 128-rank group on its own (exact int32), rounded
  // to its branch's coarsest exponent by an integer shift; the rounded values
  // add exactly, so any split of the groups over warps, CTAs or clusters gives
  // the same bits
  int I0[NCB][2], I1[NCB][2];
#pragma unroll
  for (int cb = 0; cb < NCB; ++cb) I0[cb][0] = I0[cb][1] = I1[cb][0] = I1[cb][1] = 0;
  const int ngt = ng0 + ng1;  // this warp's share of the flattened (branch, group) list
  const int ga = (split * ngt) / nsplit, gb = ((split + 1) * ngt) / nsplit;
  if (active && ok) {
    // per branch, this warp's share of the groups; each group is rounded on
    // its own (with one column block, two groups at a time as two
    // interleaved MMA chains)
    auto branch_groups = [&](const int b, int (&Ib)[NCB][2]) {
      const int lo = b ? max(ga, ng0) - ng0 : ga;
      const int hi = b ? gb - ng0 : min(gb, ng0);
      const uint32_t *wt = b ? mywt1 : mywt0;
      const int pt = sg.pitch[b];
      const uint32_t *actb = b ? act1 : act0;
      auto round_add = [&](const int (&acc)[NCB][4], int Gl) {
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
          const int t = cb * 4 + q;
          if (t < p.k) {
            const int gi = b * gk + Gl * p.k + t;
            const int ex = ue[gi];
            if (ex != UE_NONE) {
              const int sft = ex - sh.u_ec[b][t];
              const int sq = usq[gi];
              Ib[cb][0] += rshr(sq + 2 * (256 * acc[cb][0] + acc[cb][1]), sft);
              Ib[cb][1] += rshr(sq + 2 * (256 * acc[cb][2] + acc[cb][3]), sft);
            }
          }
        }
      };
      int G = lo;
      if constexpr (NCB == 1) {
        for (; G + 1 < hi; G += 2) {
          int acc[2][4] = {};
          const int gg[2] = {G, G + 1};
          sign_mma1<2>(acc, wt + g * pt, wt + (g + 8) * pt, actb, ws, p.ncols, gg, lane);
          round_add(reinterpret_cast<const int(&)[NCB][4]>(acc[0]), G);
          round_add(reinterpret_cast<const int(&)[NCB][4]>(acc[1]), G + 1);
        }
      }
      for (; G < hi; ++G) {
        int acc[NCB][4] = {};
        sign_mma<NCB>(acc, wt + g * pt, wt + (g + 8) * pt, actb, ws, p.ncols, G, G + 1, lane);
        round_add(acc, G);
      }
    };
    if constexpr (NCB == 1) {
      branch_groups(0, I0);
      if (ng1) branch_groups(1, I1);
    } else {  // one loop over the flattened (branch, group) list: fewer live registers
      for (int G = ga; G < gb; ++G) {
        const int b = G < ng0 ? 0 : 1;
        const int Gl = b ? G - ng0 : G;
        const uint32_t *wt = b ? mywt1 : mywt0;
        const int pt = sg.pitch[b];
        int acc[NCB][4] = {};
        sign_mma<NCB>(acc, wt + g * pt, wt + (g + 8) * pt, b ? act1 : act0, ws, p.ncols, Gl, Gl + 1, lane);
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
          const int t = cb * 4 + q;
          if (t < p.k) {
            const int gi = b * gk + Gl * p.k + t;
            const int ex = ue[gi];
            if (ex != UE_NONE) {
              const int sft = ex - sh.u_ec[b][t];
              const int sq = usq[gi];
              const int va = rshr(sq + 2 * (256 * acc[cb][0] + acc[cb][1]), sft);
              const int vb = rshr(sq + 2 * (256 * acc[cb][2] + acc[cb][3]), sft);
              if (b) {
                I1[cb][0] += va;
                I1[cb][1] += vb;
              } else {
                I0[cb][0] += va;
                I0[cb][1] += vb;
              }
            }
          }
        }
      }
    }
  }
  if (nsplit > 1) {
    int *xw = xch + (warp * 32 + lane) * (8 * NCB);
    if (split > 0) {
#pragma unroll
      for (int cb = 0; cb < NCB; ++cb) {
        xw[cb * 4 + 0] = I0[cb][0];
        xw[cb * 4 + 1] = I0[cb][1];
        xw[cb * 4 + 2] = I1[cb][0];
        xw[cb * 4 + 3] = I1[cb][1];
      }
    }
    __syncthreads();
    if (split == 0) {
      for (int sp = 1; sp < nsplit; ++sp) {
        const int *xr = xch + ((sp * ut + tile) * 32 + lane) * (8 * NCB);
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
          I0[cb][0] += xr[cb * 4 + 0];
          I0[cb][1] += xr[cb * 4 + 1];
          I1[cb][0] += xr[cb * 4 + 2];
          I1[cb][1] += xr[cb * 4 + 3];
        }
      }
    }
  }
  LBX_PROBE(15);
  (void)nunits;
  if (!ok) return false;
  if (active && split == 0) {
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) {
      const int t = cb * 4 + q;
      if (t >= p.k) continue;
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const int nl = g + 8 * hrow;
        const int n = n0 + nl;
        float v = u_result(myu1[nl], I0[cb][hrow], sh.u_ec[0][t], sg.nbr > 1, myu1[16 + nl], I1[cb][hrow],
                           sh.u_ec[1][t], sg.bias != nullptr, myu1[32 + nl]);
        if (p.epi == LBX_EPI_SILU0 && si == 0) v = v / (1.0f + expf(-v));
        const int64_t off = (int64_t)t * sg.y_ld + n;
        if constexpr (PEER) {  // NVLink stores of (call number, value) words
          const unsigned long long wv = ((unsigned long long)call << 32) | __float_as_uint(v);
          const long long o = (call & 1u) * p.xhalf + off;
          for (int j = 0; j < p.npeer; ++j)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.xbuf[j] + o), "l"(wv) : "memory");
        } else if (p.ydt == LBX_F32) {
          float *y = reinterpret_cast<float *>(sg.y) + off;
          if (p.epi == LBX_EPI_ADD) v += *y;
          *y = v;
        } else {
          reinterpret_cast<uint16_t *>(sg.y)[off] = f32_to_bf16(v);
        }
      }
    }
  }
  return true;
}

template <int NCB, bool PEER = false>
__global__ void __launch_bounds__(UTHREADS, 2) ustage_kernel(const __grid_constant__ UParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ LinShm sh;
  LBX_PROBE(10);
  linshm_init(sh);  // (ends with a CTA barrier)
  // scratch first, weights after: measured faster than the reverse order
  uint8_t *S = smem_raw;
  uint8_t *W = smem_raw + p.s_bytes;
  ustage_issue(p, blockIdx.x, W, sh);
  pdl_trigger();
  pdl_wait();
  ustage_run<NCB, PEER>(p, blockIdx.x, gridDim.x, W, S, sh, false);
}

#include "slice.cuh"

// ---------------------------------------------------------------------------
// Pass-split V-stage for inputs wider than one staging pass (K > 4096): the
// passes of a unit run side by side in the CTAs of one thread-block cluster,
// CTA rank r staging and contracting pass r with its own slice of the sign
// rows, v2 and norm_w.  Rank 0 then adds the per-warp partial sums of every
// rank over distributed shared memory, in the one-CTA order (for each warp
// the passes in order from 0, then the warps in order), so z and the tile
// maxima are the bits vstage_run computes with all passes in one CTA.  The
// unit's latency becomes one pass instead of ceil(K / 4096).
// ---------------------------------------------------------------------------
constexpr int VSP_PITCH = PASS_WORDS + 4;  // row pitch (words) of a pass's sign rows
constexpr int VSP_COLS = PASS_WORDS * 32;  // columns of one pass

struct VSplitLayout {
  uint32_t *wbuf;  // 16 vt x VSP_PITCH sign words of this pass
  float *sv2;      // v2 of this pass's columns
  float *snw;      // norm_w of this pass's columns (RMSNorm prologue)
  float *smid;     // 2 x 16 vt
  uint32_t *act;   // PASS_WORDS x ws
  float *red;      // VWARPS x 16 x k: this rank's per-warp partial sums of one tile
  float *twa;      // VWARPS x 16 x k: rank 0, per-warp sums over the ranks
  float *ssqa;     // VWARPS x LBX_MAX_TOKENS: rank 0, per-warp sums of squares over the ranks
};

LBX_DEV VSplitLayout vsplit_layout(const VParams &p, uint8_t *W, uint8_t *S) {
  VSplitLayout L;
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  L.wbuf = reinterpret_cast<uint32_t *>(W);
  L.sv2 = reinterpret_cast<float *>(L.wbuf + 16 * p.vt * VSP_PITCH);
  L.snw = L.sv2 + VSP_COLS;
  L.smid = L.snw + (rms ? VSP_COLS : 0);
  L.act = reinterpret_cast<uint32_t *>(S);
  L.red = reinterpret_cast<float *>(L.act + PASS_WORDS * act_ws(p.ncols));
  L.twa = L.red + VWARPS * 16 * p.k;
  L.ssqa = L.twa + VWARPS * 16 * p.k;
  return L;
}

// the weights of pass `pass` of unit `unit` (independent of the activations)
LBX_DEV void vsplit_issue(const VParams &p, int unit, int pass, uint8_t *W, LinShm &sh) {
  const int tid = threadIdx.x;
  const VSeg &sg = p.seg[vseg_of(p, unit)];
  const int row0 = (unit - sg.unit0) * 16 * p.vt;
  const int rows = min(16 * p.vt, sg.rank - row0);
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const int pw0 = pass * PASS_WORDS;
  const int pwords = min(PASS_WORDS, p.Wv - pw0);
  const int c0 = pw0 * 32, ncols = pwords * 32;
  const VSplitLayout L = vsplit_layout(p, W, nullptr);
  uint64_t *bar = &sh.bar[UT_MAX];
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)rows * pwords * 4u + (uint32_t)ncols * 4u * (rms ? 2u : 1u) +
                           (uint32_t)rows * 4u * (sg.mid1 ? 2u : 1u);
    mbar_arrive_expect_tx(bar, bytes);
  }
  __syncthreads();
  if (tid < rows)
    bulk_g2s(L.wbuf + tid * VSP_PITCH, sg.v_sign + (int64_t)(row0 + tid) * p.Wv + pw0, (uint32_t)pwords * 4u, bar);
  else if (tid == VTHREADS - 1)
    bulk_g2s(L.sv2, sg.v2 + c0, (uint32_t)ncols * 4u, bar);
  else if (tid == VTHREADS - 2 && rms)
    bulk_g2s(L.snw, p.norm_w + c0, (uint32_t)ncols * 4u, bar);
  else if (tid == VTHREADS - 3)
    bulk_g2s(L.smid, sg.mid0 + row0, (uint32_t)rows * 4u, bar);
  else if (tid == VTHREADS - 4 && sg.mid1)
    bulk_g2s(L.smid + 16 * p.vt, sg.mid1 + row0, (uint32_t)rows * 4u, bar);
}

template <int NCB, int PM, int VT>
LBX_DEV void vsplit_run(const VParams &p, int unit, int pass, int npass, uint8_t *W, uint8_t *S, LinShm &sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const VSeg &sg = p.seg[vseg_of(p, unit)];
  const int row0 = (unit - sg.unit0) * 16 * VT;
  const int ntl = min(VT, (sg.rank - row0 + 15) / 16);
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const int ws = act_ws(p.ncols);
  const VSplitLayout L = vsplit_layout(p, W, S);
  const int pw0 = pass * PASS_WORDS;
  const int pwords = min(PASS_WORDS, p.Wv - pw0);
  const int c0 = pw0 * 32;
  const uint32_t par = sh.par[UT_MAX];

  float tacc[VT][NCB][2];
#pragma unroll
  for (int tl = 0; tl < VT; ++tl)
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) tacc[tl][cb][0] = tacc[tl][cb][1] = 0.f;
  bool ok = true;
  // v2 / norm_w of this pass are in shared memory: index them by column
  vstage_stage<PM>(p, sg.v2, L.sv2 - c0, L.snw - c0, pass, L.act, sh, [&] {
    ok = __syncthreads_and(mbar_wait_bounded(&sh.bar[UT_MAX], par, 0x111));
  }, c0 + VSP_COLS);
  __syncthreads();
  if (tid == 0) sh.par[UT_MAX] = par ^ 1u;
  if (ok && BLK_WORDS * warp < pwords) {
    const int wb = BLK_WORDS * warp;
    const int ng = min(BLK_WORDS, pwords - wb) / 4;
#pragma unroll
    for (int tl = 0; tl < VT; ++tl) {
      if (tl < ntl) {
        int acc[NCB][4];
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) acc[cb][0] = acc[cb][1] = acc[cb][2] = acc[cb][3] = 0;
        const uint32_t *wt = L.wbuf + tl * 16 * VSP_PITCH + wb;
        sign_mma<NCB>(acc, wt + g * VSP_PITCH, wt + (g + 8) * VSP_PITCH, L.act + wb * ws, ws, p.ncols, 0, ng,
                      lane);
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
          const int t = cb * 4 + q;
          if (t < p.k) {
            const int sq = sh.v_sq[warp][t];
            const float inv = sh.v_inv[warp][t];
            tacc[tl][cb][0] += __fmul_rn(__int2float_rn(sq + 2 * (256 * acc[cb][0] + acc[cb][1])), inv);
            tacc[tl][cb][1] += __fmul_rn(__int2float_rn(sq + 2 * (256 * acc[cb][2] + acc[cb][3])), inv);
          }
        }
      }
    }
  }
  // ---- per tile: rank 0 adds the ranks' partials in the one-CTA order.  Every
  // rank takes both cluster barriers of every tile, whatever its status.
  const float *smid = L.smid;
#pragma unroll
  for (int tl = 0; tl < VT; ++tl) {
    if (tl >= ntl) break;  // uniform across the cluster
    const int trow = row0 + tl * 16;
    const int rows = min(16, sg.rank - trow);
    float *rw = L.red + warp * 16 * p.k;
#pragma unroll
    for (int cb = 0; cb < NCB; ++cb) {
      const int t = cb * 4 + q;
      if (t < p.k) {
        rw[g * p.k + t] = tacc[tl][cb][0];
        rw[(g + 8) * p.k + t] = tacc[tl][cb][1];
      }
    }
    cl_arrive();
    cl_wait();  // every rank's partials (and sums of squares) are written
    if (pass == 0) {
      const int nk = rows * p.k;
      for (int i = tid; i < VWARPS * nk; i += VTHREADS) {
        const int w = i / nk, rem = i - w * nk;
        const int rr = rem / p.k, t = rem - rr * p.k;
        const float *src = L.red + (w * 16 + rr) * p.k + t;
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = r < npass ? *cl_map(src, r) : 0.f;
        float tw = 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r)
          if (r < npass) tw += v[r];
        L.twa[(w * 16 + rr) * p.k + t] = tw;
      }
      if (rms && tl == 0) {
        for (int i = tid; i < VWARPS * p.k; i += VTHREADS) {
          const int w = i / p.k, t = i - w * p.k;
          const float *src = &sh.v_ssq[w][t];
          float v[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) v[r] = r < npass ? *cl_map(src, r) : 0.f;
          float sw = 0.f;
#pragma unroll
          for (int r = 0; r < 8; ++r)
            if (r < npass) sw += v[r];
          L.ssqa[w * LBX_MAX_TOKENS + t] = sw;
        }
      }
      __syncthreads();
      for (int i = tid; i < nk; i += VTHREADS) {
        const int rr = i / p.k, t = i - rr * p.k;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < VWARPS; ++w) v += L.twa[(w * 16 + rr) * p.k + t];
        if (rms) {
          float s2 = 0.f;
#pragma unroll
          for (int w = 0; w < VWARPS; ++w) s2 += L.ssqa[w * LBX_MAX_TOKENS + t];
          v *= rsqrtf(s2 / (float)p.K + p.eps);
        }
        const float z0 = smid[tl * 16 + rr] * v;
        sg.z0[(int64_t)t * sg.rank + trow + rr] = z0;
        atomicMax(&sh.v_zmax[0][t], __float_as_int(fabsf(z0)));
        if (sg.z1) {
          const float z1 = smid[16 * VT + tl * 16 + rr] * v;
          sg.z1[(int64_t)t * sg.rank + trow + rr] = z1;
          atomicMax(&sh.v_zmax[1][t], __float_as_int(fabsf(z1)));
        }
      }
      __syncthreads();
      if (tid < p.k) {
        int *tm = sg.tmax + (int64_t)(trow / 16) * 2 * p.k;
        tm[tid] = sh.v_zmax[0][tid];
        if (sg.z1) tm[p.k + tid] = sh.v_zmax[1][tid];
        sh.v_zmax[0][tid] = sh.v_zmax[1][tid] = 0;
      }
    }
    cl_arrive();
    cl_wait();  // rank 0 has read every rank's partials: they may be overwritten, or the CTAs leave
  }
}

template <int NCB, int PM, int VT>
__global__ void __launch_bounds__(VTHREADS, 2) vsplit_kernel(const __grid_constant__ VParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ LinShm sh;
  const int npass = (p.Wv + PASS_WORDS - 1) / PASS_WORDS;
  const int pass = cl_rank();  // clusters of npass CTAs along x
  const int unit = blockIdx.x / npass;
  if (threadIdx.x < VWARPS * LBX_MAX_TOKENS) (&sh.v_ssq[0][0])[threadIdx.x] = 0.f;
  if (threadIdx.x < 2 * LBX_MAX_TOKENS) (&sh.v_zmax[0][0])[threadIdx.x] = 0;
  linshm_init(sh);  // (ends with a CTA barrier)
  uint8_t *S = smem_raw;
  uint8_t *W = smem_raw + p.s_bytes;
  vsplit_issue(p, unit, pass, W, sh);
  pdl_trigger();
  pdl_wait();
  vsplit_run<NCB, PM, VT>(p, unit, pass, npass, W, S, sh);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// scratch: [header: the cluster executor's range tickets and the grid barrier
// of a persistent program (zero between calls, at fixed offsets)] then z
// [k][rank] of every (projection, branch) and the per-unit maxima [tile][2][k]
// of every V segment (both overwritten by every call)
constexpr size_t WS_GRIDBAR = 400;  // byte offset of the grid barrier words in the header
constexpr size_t WS_HDR = 512;

static int u_groups(int rank) { return (rank + UGRP - 1) / UGRP; }

constexpr size_t WS_SLTICKET = 16;  // byte offset of the cluster executor's range tickets
static_assert(WS_SLTICKET + LBX_MAX_PROJ * SL_S * 4 <= WS_GRIDBAR, "header layout");

// cluster executor scratch after the header: per projection the exact group
// sums [groups][k][out] and the group exponents [2][ZGMAX][LBX_MAX_TOKENS]
static size_t slice_ws_bytes(const lbx_proj *projs, int n_proj, int k) {
  size_t tot = WS_HDR;
  for (int i = 0; i < n_proj; ++i) {
    size_t ng = 0;
    for (int b = 0; b < projs[i].n_branches; ++b) ng += (projs[i].br[b].rank + UGRP - 1) / UGRP;
    tot += al256(ng * k * projs[i].out_features * 4) + al256((size_t)2 * ZGMAX * LBX_MAX_TOKENS * 4);
  }
  return tot;
}

// scratch of the two stage grids
static size_t stage_ws_bytes(const lbx_proj *projs, int n_proj, int k) {
  size_t tot = WS_HDR;
  for (int i = 0; i < n_proj; ++i)
    for (int b = 0; b < projs[i].n_branches; ++b) {
      tot += al256((size_t)k * projs[i].br[b].rank * 4);
      if (projs[i].br[b].v_sign) tot += al256((size_t)(projs[i].br[b].rank + 15) / 16 * 2 * k * 4);
    }
  return tot;
}

// scratch of a call on any executor (the public workspace size)
static size_t ws_bytes_for(const lbx_proj *projs, int n_proj, int k) {
  return std::max(stage_ws_bytes(projs, n_proj, k), slice_ws_bytes(projs, n_proj, k));
}

// scratch of this call on the executor it selects
static size_t ws_bytes_call(const lbx_proj *projs, const lbx_linear_args *a) {
  const int k = a->n_tokens < LBX_MAX_TOKENS ? a->n_tokens : LBX_MAX_TOKENS;
  return a->exec == LBX_EXEC_CLUSTER ? ws_bytes_for(projs, a->n_proj, k)
                                     : stage_ws_bytes(projs, a->n_proj, k);
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
      LBX_CHECK_SUP(br.rank > 0 && br.rank % 8 == 0, "rank must be a positive multiple of 8 (got %d)",
                    br.rank);
      LBX_CHECK_SUP(br.rank <= UGRP * ZGMAX, "rank must be at most %d (got %d)", UGRP * ZGMAX, br.rank);
      LBX_CHECK_ARG(br.mid && br.u_sign && br.u1, "branch %d: mid/u_sign/u1 required", b);
      LBX_CHECK_ARG(aligned16(br.u_sign) && aligned16(br.mid), "u_sign/mid must be 16-byte aligned");
      if (br.v_sign) {
        LBX_CHECK_ARG(br.v2, "branch %d: v2 required with v_sign", b);
        LBX_CHECK_ARG(aligned16(br.v_sign) && aligned16(br.v2), "v_sign/v2 must be 16-byte aligned");
      } else {
        LBX_CHECK_ARG(b == 1 && pr.br[0].v_sign && br.rank == pr.br[0].rank,
                      "a shared-V branch must be the residual with the main branch's rank");
      }
    }
  }
  return LBX_OK;
}

static int check_args(const lbx_proj *projs, const lbx_linear_args *a) {
  LBX_CHECK_ARG(a, "args is NULL");
  int rc = validate(projs, a->n_proj);
  if (rc) return rc;
  LBX_CHECK_ARG(a->n_tokens >= 1, "n_tokens must be >= 1");
  LBX_CHECK_ARG(a->x, "x is NULL");
  LBX_CHECK_ARG(a->x_dtype == LBX_F32 || a->x_dtype == LBX_BF16, "bad x_dtype");
  LBX_CHECK_ARG(a->y_dtype == LBX_F32 || a->y_dtype == LBX_BF16, "bad y_dtype");
  LBX_CHECK_ARG(aligned16(a->x) && (!a->x2 || aligned16(a->x2)), "x/x2 must be 16-byte aligned");
  LBX_CHECK_ARG(a->prologue >= LBX_PRO_NONE && a->prologue <= LBX_PRO_MUL, "bad prologue");
  LBX_CHECK_ARG(a->prologue != LBX_PRO_RMSNORM || (a->norm_w && aligned16(a->norm_w)),
                "RMSNorm prologue needs a 16-byte aligned norm_w");
  LBX_CHECK_ARG((a->prologue != LBX_PRO_SILU_MUL && a->prologue != LBX_PRO_MUL) || a->x2,
                "SiLU-mul and mul prologues need x2");
  LBX_CHECK_ARG(a->epilogue == LBX_EPI_STORE || a->epilogue == LBX_EPI_SILU0 ||
                    (a->epilogue == LBX_EPI_ADD && a->y_dtype == LBX_F32),
                "bad epilogue (ADD needs fp32 y)");
  for (int i = 0; i < a->n_proj; ++i) LBX_CHECK_ARG(a->y[i], "y[%d] is NULL", i);
  LBX_CHECK_ARG(a->exec == LBX_EXEC_AUTO || a->exec == LBX_EXEC_KERNELS || a->exec == LBX_EXEC_CLUSTER ||
                    a->exec == LBX_EXEC_KERNELS_ONE_CTA_V || a->exec == LBX_EXEC_TC ||
                    a->exec == LBX_EXEC_NO_TC,
                "bad exec (LBX_EXEC_AUTO, _KERNELS, _CLUSTER, _KERNELS_ONE_CTA_V, _TC or _NO_TC)");
  return LBX_OK;
}

using VKern = void (*)(VParams);
template <int PM, int VT>
static VKern vstage_for_pv(int ncb) {
  return ncb == 1 ? vstage_kernel<1, PM, VT> : ncb == 2 ? vstage_kernel<2, PM, VT> : vstage_kernel<4, PM, VT>;
}
template <int VT>
static VKern vstage_for_vt(int ncb, int pm) {
  return pm == PM_SILU ? vstage_for_pv<PM_SILU, VT>(ncb)
         : pm == PM_MUL ? vstage_for_pv<PM_MUL, VT>(ncb)
                        : vstage_for_pv<PM_X, VT>(ncb);
}
static VKern vstage_for(int ncb, int pm, int vt) {
  return vt == 2 ? vstage_for_vt<2>(ncb, pm) : vstage_for_vt<1>(ncb, pm);
}
template <int PM, int VT>
static VKern vsplit_for_pv(int ncb) {
  return ncb == 1 ? vsplit_kernel<1, PM, VT> : ncb == 2 ? vsplit_kernel<2, PM, VT> : vsplit_kernel<4, PM, VT>;
}
template <int VT>
static VKern vsplit_for_vt(int ncb, int pm) {
  return pm == PM_SILU ? vsplit_for_pv<PM_SILU, VT>(ncb)
         : pm == PM_MUL ? vsplit_for_pv<PM_MUL, VT>(ncb)
                        : vsplit_for_pv<PM_X, VT>(ncb);
}
static VKern vsplit_for(int ncb, int pm, int vt) {
  return vt == 2 ? vsplit_for_vt<2>(ncb, pm) : vsplit_for_vt<1>(ncb, pm);
}

static int sm_count() { return device_sm_count(); }

#ifndef LBX_U_GROUPS
#define LBX_U_GROUPS 136  // quantisation groups per U-stage CTA at most (measured on 7B- and 70B-shaped calls)
#endif
#ifndef LBX_U_MIN_CTAS
#define LBX_U_MIN_CTAS 60  // U-stage CTAs to aim for when choosing tiles per CTA (measured: 4 tiles per CTA beat 2 and 8 at C2)
#endif

// dynamic shared memory the stage kernels may use (after their static
// shared memory); established once per device, before any graph capture
struct StageSmem {
  size_t v, u;
};
static int stage_smem_limits(size_t &vmax, size_t &umax) {
  static DevCache<StageSmem> cache;
  StageSmem lim{};
  const int rc = cache.get(lim, [](StageSmem &out) {
    size_t m = 0, vv = (size_t)-1, uu = (size_t)-1;
    VKern all[36];
    int na = 0;
    for (int vt = 1; vt <= 2; ++vt)
      for (int pm = 0; pm < 3; ++pm)
        for (int ncb : {1, 2, 4}) {
          all[na++] = vstage_for(ncb, pm, vt);
          all[na++] = vsplit_for(ncb, pm, vt);
        }
    for (VKern kk : all) {
      cudaError_t e = allow_max_smem(kk, &m);
      if (e != cudaSuccess) return cuda_status(e, "vstage smem attribute");
      vv = std::min(vv, m);
    }
    for (auto kk : {ustage_kernel<1>, ustage_kernel<2>, ustage_kernel<4>}) {
      cudaError_t e = allow_max_smem(kk, &m);
      if (e != cudaSuccess) return cuda_status(e, "ustage smem attribute");
      uu = std::min(uu, m);
    }
    out.v = vv;
    out.u = uu;
    return (int)LBX_OK;
  });
  vmax = lim.v;
  umax = lim.u;
  return rc;
}

// one batch of k <= LBX_MAX_TOKENS tokens of a linear call, as the parameters
// of its two stages
struct LinPrep {
  VParams vp;
  UParams up;
  int ncb, vunits, uunits;
  size_t v_w, v_s, u_w, u_s;  // weight (W) and scratch (S) shared-memory bytes of each stage
};

// multi_tile: V units of two tiles when one-tile units would not all be
// resident at once (the persistent program keeps one tile per unit)
static int prep_linear(const lbx_proj *projs, const lbx_linear_args *a, int tok0, int k, void *ws,
                       size_t vmax, size_t umax, LinPrep &P, bool multi_tile = true) {
  const int n_proj = a->n_proj;
  const int K = projs[0].in_features;
  const int ncols = 2 * k;
  // MMA column blocks the stage code is instantiated for (1, 2 or 4); every
  // size below must use this, not the bare ceil(ncols/8)
  const int ncb_need = (ncols + 7) / 8;
  const int ncb = ncb_need <= 1 ? 1 : ncb_need <= 2 ? 2 : 4;
  const int esz_x = a->x_dtype == LBX_F32 ? 4 : 2;
  const int esz_y = a->y_dtype == LBX_F32 ? 4 : 2;
  const int Wv = K / 32;
  const bool rms = a->prologue == LBX_PRO_RMSNORM;

  // scratch: header, then z of every (projection, branch), [k][rank], and the
  // per-unit maxima of every V segment, [tile][2][k]
  float *zp[LBX_MAX_PROJ][2] = {};
  int *tm[LBX_MAX_PROJ][2] = {};
  {
    uint8_t *w = reinterpret_cast<uint8_t *>(ws) + WS_HDR;
    for (int i = 0; i < n_proj; ++i)
      for (int b = 0; b < projs[i].n_branches; ++b) {
        zp[i][b] = reinterpret_cast<float *>(w);
        w += al256((size_t)k * projs[i].br[b].rank * 4);
        if (projs[i].br[b].v_sign) {
          tm[i][b] = reinterpret_cast<int *>(w);
          w += al256((size_t)(projs[i].br[b].rank + 15) / 16 * 2 * k * 4);
        }
      }
  }

  // ---------------- V-stage
  VParams &vp = P.vp;
  vp = VParams{};
  vp.K = K;
  vp.Wv = Wv;
  vp.vpitch = row_pitch(Wv);
  vp.vcap = std::min(K, VCAP_MAX);
  vp.k = k;
  vp.ncols = ncols;
  vp.xdt = a->x_dtype;
  vp.prologue = a->prologue;
  vp.eps = a->eps;
  vp.x = reinterpret_cast<const uint8_t *>(a->x) + (size_t)tok0 * K * esz_x;
  vp.x2 = a->x2 ? reinterpret_cast<const uint8_t *>(a->x2) + (size_t)tok0 * K * esz_x : nullptr;
  vp.norm_w = a->norm_w;
  int ttiles = 0;
  for (int i = 0; i < n_proj; ++i)
    for (int b = 0; b < projs[i].n_branches; ++b)
      if (projs[i].br[b].v_sign) ttiles += (projs[i].br[b].rank + 15) / 16;
  vp.vt = multi_tile && ttiles > 2 * sm_count() ? 2 : 1;
  int vunits = 0;
  for (int i = 0; i < n_proj; ++i) {
    const lbx_proj &pr = projs[i];
    for (int b = 0; b < pr.n_branches; ++b) {
      if (!pr.br[b].v_sign) continue;
      VSeg &sg = vp.seg[vp.nseg++];
      sg.v_sign = pr.br[b].v_sign;
      sg.v2 = pr.br[b].v2;
      sg.mid0 = pr.br[b].mid;
      sg.z0 = zp[i][b];
      sg.tmax = tm[i][b];
      sg.rank = pr.br[b].rank;
      if (b == 0 && pr.n_branches == 2 && !pr.br[1].v_sign) {
        sg.mid1 = pr.br[1].mid;
        sg.z1 = zp[i][1];

      }
      sg.unit0 = vunits;
      vunits += ((sg.rank + 15) / 16 + vp.vt - 1) / vp.vt;
    }
  }
  P.v_w = al256((size_t)16 * vp.vt * vp.vpitch * 4 + (size_t)vp.vcap * 4 * (rms ? 2 : 1) + 32 * vp.vt * 4);
  P.v_s = (size_t)PASS_WORDS * act_ws(ncols) * 4 + (size_t)VWARPS * 16 * k * 4;
  P.v_s = (P.v_s + 255) & ~(size_t)255;
  vp.s_bytes = (int)P.v_s;
  LBX_CHECK_SUP(P.v_w + P.v_s <= vmax, "V-stage needs %zu bytes of shared memory (max %zu)",
                P.v_w + P.v_s, vmax);

  // ---------------- U-stage
  UParams &up = P.up;
  up = UParams{};
  up.k = k;
  up.ncols = ncols;
  up.ydt = a->y_dtype;
  up.epi = a->epilogue;
  int maxw[2] = {0, 0}, maxtile = 0, tiles = 0, ugm = 1, ngt_max = 1;
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
      sg.tmax[b] = pr.br[b].v_sign ? tm[i][b] : tm[i][0];  // a shared-V residual: the main segment's units
      sg.tsel[b] = pr.br[b].v_sign ? 0 : 1;
      sg.rank[b] = pr.br[b].rank;
      sg.words[b] = (pr.br[b].rank + 31) / 32;
      sg.perrow[b] = (sg.words[b] % 4) == 0;
      sg.pitch[b] = sg.perrow[b] ? row_pitch(sg.words[b]) : sg.words[b];
      maxw[b] = std::max(maxw[b], 4 * ((sg.words[b] + 3) / 4));
      ugm = std::max(ugm, u_groups(sg.rank[b]));
      tw += 16 * sg.pitch[b] + 4;
    }
    maxtile = std::max(maxtile, tw);
    tiles += pr.out_features / 16;
    int ng = 0;  // quantisation groups of one output tile (both branches)
    for (int b = 0; b < pr.n_branches; ++b) ng += (sg.words[b] + 3) / 4;
    ngt_max = std::max(ngt_max, ng);
  }
  up.act_words[0] = maxw[0];
  up.act_words[1] = maxw[1];
  up.ugm = ugm;
  up.wtile_words = (maxtile + 3) & ~3;
  // row tiles per CTA: enough CTAs to cover the SMs, within shared memory; the
  // remaining warps of a CTA split the ranks of its tiles
  // row tiles per CTA: at least LBX_U_MIN_CTAS CTAs, and no more than
  // LBX_U_GROUPS quantisation groups per CTA (heavy tiles spread over more
  // SMs), but not beyond two CTAs per SM
  int ut = UT_MAX;
  while (ut > 1 && (tiles / ut < LBX_U_MIN_CTAS || ut * ngt_max > LBX_U_GROUPS)) ut >>= 1;
  while (ut < UT_MAX && tiles / ut > 2 * sm_count()) ut <<= 1;
  const size_t u_s = al256((size_t)(maxw[0] + maxw[1]) * act_ws(ncols) * 4 + (size_t)4 * ugm * k * 4 +
                           (size_t)UWARPS * 32 * 8 * ncb * 4);
  for (; ut >= 1; ut >>= 1) {
    const size_t u_w = al256((size_t)ut * up.wtile_words * 4 + (size_t)ut * 48 * 4);
    if (u_w + u_s <= umax) break;
  }
  LBX_CHECK_SUP(ut >= 1, "U-stage needs too much shared memory (rank too large for k=%d)", k);
  up.ut = ut;

  P.u_w = al256((size_t)ut * up.wtile_words * 4 + (size_t)ut * 48 * 4);
  P.u_s = u_s;
  up.s_bytes = (int)P.u_s;
  int ctas = 0;
  for (int i = 0; i < n_proj; ++i) {
    up.seg[i].cta0 = ctas;
    ctas += (projs[i].out_features + 16 * ut - 1) / (16 * ut);
  }
  up.nseg = n_proj;
  P.ncb = ncb;
  P.vunits = vunits;
  P.uunits = ctas;
  return LBX_OK;
}

#ifndef LBX_SL_CLUSTERS
#define LBX_SL_CLUSTERS 9  // clusters per cluster-executor launch (9 x 16 CTAs on 148 SMs)
#endif

// dynamic shared memory the cluster kernel may use, and the cluster-size opt-in
static int slice_smem_limit(size_t &cmax) {
  static DevCache<size_t> cache;
  return cache.get(cmax, [](size_t &out) {
    size_t m = 0;
    cudaError_t e = allow_max_smem(slice_kernel<1>, &m);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(slice_kernel<1>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_status(e, "cluster kernel attributes");
    out = m;
    return (int)LBX_OK;
  });
}

static cudaLaunchConfig_t slice_cfg(cudaLaunchAttribute (&attr)[2], int nclusters, size_t smem,
                                    cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nclusters * SL_S);
  cfg.blockDim = dim3(VTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = SL_S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int na = 1;
  if (pdl) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cfg;
}

// clusters of the cluster kernel with `smem` bytes each that can be resident
// at once (cached per device and shared-memory size)
static int slice_active(size_t smem) {
  static int cache[LBX_MAX_DEVICES][256] = {};
  const int kb = (int)((smem + 1023) / 1024);
  const int dev = cur_device();
  if (kb >= 256) return 0;
  int scratch = 0;
  std::lock_guard<std::recursive_mutex> lk(dev_cache_mu());
  int &v = dev >= 0 && dev < LBX_MAX_DEVICES ? cache[dev][kb] : scratch;
  if (!v) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = slice_cfg(attr, LBX_SL_CLUSTERS, (size_t)kb * 1024, nullptr, false);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void *)slice_kernel<1>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    v = n + 1;
  }
  return v - 1;
}

// cluster-executor parameters; false (with the reason in `why`) when the call
// does not fit it
static bool prep_slice(const lbx_proj *projs, const lbx_linear_args *a, int k, const LinPrep &P,
                       void *ws, size_t cmax, SlParams &sp, size_t &smem, char (&why)[160]) {
  const VParams &vp = P.vp;
  const int n_proj = a->n_proj;
  why[0] = 0;
  if (P.ncb != 1 || vp.Wv > PASS_WORDS) {
    snprintf(why, sizeof why, "needs k <= 4 and in_features <= 4096");
    return false;
  }
  const int ncl_max = LBX_SL_CLUSTERS;
  if (vp.nseg > ncl_max) {
    snprintf(why, sizeof why, "%d V segments for %d clusters", vp.nseg, ncl_max);
    return false;
  }
  sp = SlParams{};
  sp.vp = vp;
  sp.vp.vcap = 0;  // v2 / norm_w straight from global memory (prefetched to L2)
  // segment -> (projection, branch, shared-V) in prep_linear's order
  int sproj[2 * LBX_MAX_PROJ], sbr[2 * LBX_MAX_PROJ], NG[2 * LBX_MAX_PROJ], nc[2 * LBX_MAX_PROJ];
  {
    int si = 0;
    for (int i = 0; i < n_proj; ++i)
      for (int b = 0; b < projs[i].n_branches; ++b)
        if (projs[i].br[b].v_sign) {
          sproj[si] = i;
          sbr[si] = b;
          NG[si] = (projs[i].br[b].rank + UGRP - 1) / UGRP;
          nc[si] = 1;
          ++si;
        }
  }
  // clusters: one per segment, the rest to the segment with the most groups per cluster
  for (int left = ncl_max - vp.nseg; left > 0; --left) {
    int best = -1;
    for (int i = 0; i < vp.nseg; ++i)
      if (nc[i] < NG[i] && (best < 0 || (NG[i] + nc[i] - 1) / nc[i] > (NG[best] + nc[best] - 1) / nc[best]))
        best = i;
    if (best < 0) break;
    ++nc[best];
  }
  int ncl = 0, ugmax = 1, zcap = 4;
  int pncl[LBX_MAX_PROJ] = {};
  for (int si = 0; si < vp.nseg; ++si) {
    const VSeg &vs = vp.seg[si];
    const int base = NG[si] / nc[si], extra = NG[si] % nc[si];
    for (int c = 0, g0 = 0; c < nc[si]; ++c) {
      const int ng = base + (c < extra ? 1 : 0);
      SlCluster &C = sp.cl[ncl++];
      C.proj = sproj[si];
      C.vseg = si;
      C.row0 = g0 * UGRP;
      C.rows = std::min(ng * UGRP, vs.rank - C.row0);
      C.tpc = ((C.rows + 15) / 16 + SL_S - 1) / SL_S;
      C.nplane = vs.mid1 ? 2 : 1;
      C.br[0] = sbr[si];
      C.br[1] = 1;
      if (C.tpc > SL_VT) {
        snprintf(why, sizeof why, "%d V tiles per CTA (max %d)", C.tpc, SL_VT);
        return false;
      }
      ugmax = std::max(ugmax, ng);
      zcap = std::max(zcap, C.rows);
      ++pncl[C.proj];
      g0 += ng;
    }
  }
  sp.ncl = ncl;
  // projections
  uint8_t *w = reinterpret_cast<uint8_t *>(ws) + WS_HDR;
  int rmax = 16, gmax = 1;
  for (int i = 0; i < n_proj; ++i) {
    const lbx_proj &pr = projs[i];
    SlProj &Pj = sp.pj[i];
    Pj.out = pr.out_features;
    Pj.nbr = pr.n_branches;
    int ng = 0;
    for (int b = 0; b < pr.n_branches; ++b) {
      Pj.u_sign[b] = pr.br[b].u_sign;
      Pj.words[b] = (pr.br[b].rank + 31) / 32;
      Pj.ngrp[b] = (pr.br[b].rank + UGRP - 1) / UGRP;
      Pj.u1[b] = pr.br[b].u1;
      ng += Pj.ngrp[b];
    }
    Pj.bias = pr.bias;
    Pj.y = P.up.seg[i].y;
    Pj.y_ld = P.up.seg[i].y_ld;
    Pj.rtiles = (pr.out_features / 16 + SL_S - 1) / SL_S;
    Pj.ncl = pncl[i];
    Pj.part = reinterpret_cast<int *>(w);
    w += al256((size_t)ng * k * pr.out_features * 4);
    Pj.gexp = reinterpret_cast<int *>(w);
    w += al256((size_t)2 * ZGMAX * LBX_MAX_TOKENS * 4);
    rmax = std::max(rmax, Pj.rtiles * 16);
    gmax = std::max(gmax, ng);
  }
  for (int c = 0; c < ncl; ++c) {
    const SlCluster &C = sp.cl[c];
    const int nug = C.nplane * ((C.rows + UGRP - 1) / UGRP);
    const int pairs = sp.pj[C.proj].rtiles * nug;
    if ((pairs + VWARPS - 1) / VWARPS > SL_UP) {
      snprintf(why, sizeof why, "%d output (tile, group) pairs per warp (max %d)",
               (pairs + VWARPS - 1) / VWARPS, SL_UP);
      return false;
    }
  }
  sp.ydt = a->y_dtype;
  sp.epi = a->epilogue;
  sp.ticket = reinterpret_cast<unsigned *>(reinterpret_cast<uint8_t *>(ws) + WS_SLTICKET);
  sp.zcap = zcap;
  sp.rmax = rmax;
  sp.ugmax = ugmax;
  // shared memory: V staging / U digits | V partials | gathered z | mid |
  // exponents, digit sums | U sign words | u1, bias
  const size_t ws_ = (size_t)act_ws(vp.ncols);
  sp.o_red = (int)al256((size_t)PASS_WORDS * ws_ * 4);
  sp.o_zall = (int)al256(sp.o_red + (size_t)SL_VT * VWARPS * 16 * k * 4);
  sp.o_mid = (int)al256(sp.o_zall + (size_t)2 * k * zcap * 4);
  sp.o_ue = (int)al256(sp.o_mid + (size_t)2 * SL_ZR * 4);
  sp.o_uw = (int)al256(sp.o_ue + (size_t)4 * ugmax * k * 4);
  sp.o_u1 = (int)al256(sp.o_uw + (size_t)SL_UP * VWARPS * 32 * 8);
  smem = al256(sp.o_u1 + (size_t)3 * rmax * 4);
  // the finalize staging overlays everything before u1: after the cluster
  // barrier no other CTA touches this CTA's shared memory, and the U
  // contraction is done
  sp.o_fin = 0;
  const size_t fe = (size_t)2 * ZGMAX * k * 4;
  const size_t room = (size_t)sp.o_u1 - fe;
  sp.fin_rows = std::min(rmax, (int)(room / ((size_t)gmax * k * 4)) / 16 * 16);
  if (sp.fin_rows < 16) {
    snprintf(why, sizeof why, "no room to combine %d groups", gmax);
    return false;
  }
  if (smem > cmax) {
    snprintf(why, sizeof why, "%zu bytes of shared memory (max %zu)", smem, cmax);
    return false;
  }
  const int act = slice_active(smem);
  if (act < ncl) {
    snprintf(why, sizeof why, "%d clusters resident at once (need %d)", act, ncl);
    return false;
  }
  return true;
}

#ifndef LBX_V_SPLIT
#define LBX_V_SPLIT 1  // 0: every V unit runs all of its staging passes in one CTA
#endif

// Whether one cluster of `npass` pass-split CTAs with `smem` bytes each can be
// resident on this device (a partitioned or heavily shared GPU may not offer a
// whole cluster); when it cannot, the call runs the one-CTA V-stage, which
// gives the same bits.  Cached per device, kernel, cluster size and size.
static bool vsplit_schedulable(VKern kern, int npass, size_t smem) {
  struct Key {
    int dev;
    VKern k;
    int npass;
    size_t smem;
  };
  static Key seen[256];
  static bool fits[256];
  static int nseen = 0;
  const int dev = cur_device();
  std::lock_guard<std::recursive_mutex> lk(dev_cache_mu());
  for (int i = 0; i < nseen; ++i)
    if (seen[i].dev == dev && seen[i].k == kern && seen[i].npass == npass && seen[i].smem == smem)
      return fits[i];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(npass);
  cfg.blockDim = dim3(VTHREADS);
  cfg.dynamicSmemBytes = smem;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = npass;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void *)kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  const bool ok = n >= 1;
  if (nseen < 256) {
    seen[nseen] = Key{dev, kern, npass, smem};
    fits[nseen++] = ok;
  }
  return ok;
}

static int run_batch(const lbx_proj *projs, const lbx_linear_args *a, int tok0, int k, void *ws,
                     cudaStream_t stream) {
  size_t vmax = 0, umax = 0;
  int rc = stage_smem_limits(vmax, umax);
  if (rc) return rc;
  LinPrep P;
  rc = prep_linear(projs, a, tok0, k, ws, vmax, umax, P);
  if (rc) return rc;
  const bool pdl = a->use_pdl != 0;
  if (a->exec == LBX_EXEC_CLUSTER) {
    size_t cmax = 0;
    rc = slice_smem_limit(cmax);
    if (rc) return rc;
    SlParams sp;
    size_t smem = 0;
    char why[160];
    if (prep_slice(projs, a, k, P, ws, cmax, sp, smem, why)) {
      cudaLaunchAttribute attr[2];
      const cudaLaunchConfig_t cfg = slice_cfg(attr, sp.ncl, smem, stream, pdl);
      return cuda_status(cudaLaunchKernelEx(&cfg, slice_kernel<1>, sp), "cluster kernel launch");
    }
    LBX_CHECK_SUP(false, "this call does not fit the cluster executor: %s", why);
  }
  auto uk = P.ncb == 1 ? ustage_kernel<1> : P.ncb == 2 ? ustage_kernel<2> : ustage_kernel<4>;
  cudaError_t e;
  // inputs wider than one staging pass on a small V grid: the pass-split
  // V-stage (a cluster of one CTA per pass for each unit), when all of its
  // CTAs fit at two per SM.  Measured: 7B draft down projection 12.5 -> 9.3 us,
  // 70B draft down 22.7 -> 16.0 us; on grids that already fill the GPU (the 7B
  // and 70B targets) it was slower, 19.5 -> 24.5 us for the 7B down call.
  const int npass = (P.vp.Wv + PASS_WORDS - 1) / PASS_WORDS;
  bool split = false;
  if (LBX_V_SPLIT && a->exec != LBX_EXEC_KERNELS_ONE_CTA_V && npass > 1 && npass <= 8 &&
      P.vunits * npass <= 2 * sm_count()) {
    const bool rms = a->prologue == LBX_PRO_RMSNORM;
    const size_t sw = al256((size_t)16 * P.vp.vt * VSP_PITCH * 4 + (size_t)VSP_COLS * 4 * (rms ? 2 : 1) +
                            (size_t)32 * P.vp.vt * 4);
    const size_t ss = al256((size_t)PASS_WORDS * act_ws(P.vp.ncols) * 4 + (size_t)2 * VWARPS * 16 * k * 4 +
                            (size_t)VWARPS * LBX_MAX_TOKENS * 4);
    if (sw + ss <= vmax && vsplit_schedulable(vsplit_for(P.ncb, pm_of(a->prologue), P.vp.vt), npass, sw + ss)) {
      VParams vp = P.vp;
      vp.split = 1;
      vp.s_bytes = (int)ss;
      cudaLaunchAttribute attr[2];
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(P.vunits * npass);
      cfg.blockDim = dim3(VTHREADS);
      cfg.dynamicSmemBytes = sw + ss;
      cfg.stream = stream;
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = npass;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      int na = 1;
      if (pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        na = 2;
      }
      cfg.attrs = attr;
      cfg.numAttrs = na;
      e = cudaLaunchKernelEx(&cfg, vsplit_for(P.ncb, pm_of(a->prologue), P.vp.vt), vp);
      if (e != cudaSuccess) return cuda_status(e, "pass-split vstage launch");
      split = true;
    }
  }
  if (!split) {
    auto vk = vstage_for(P.ncb, pm_of(a->prologue), P.vp.vt);
    e = launch(vk, dim3(P.vunits), dim3(VTHREADS), P.v_w + P.v_s, stream, pdl, P.vp);
    if (e != cudaSuccess) return cuda_status(e, "vstage launch");
  }
  e = launch(uk, dim3(P.uunits), dim3(UTHREADS), P.u_w + P.u_s, stream, pdl, P.up);
  if (e != cudaSuccess) return cuda_status(e, "ustage launch");
  return LBX_OK;
}

}  // namespace lbx

// the tensor-core executor (wide.cu)
namespace lbx {
static bool wide_auto(const lbx_proj *projs, int n_proj, int n_tokens);
static size_t wide_ws_bytes(const lbx_proj *projs, int n_proj, int k);
static int wide_try(const lbx_proj *projs, const lbx_linear_args *a, void *ws, size_t ws_bytes,
                    cudaStream_t stream, bool &handled);
}  // namespace lbx

extern "C" size_t lbx_linear_workspace_size(const lbx_proj *projs, int32_t n_proj,
                                            int32_t n_tokens) {
  if (!projs || n_proj < 1 || n_proj > LBX_MAX_PROJ || n_tokens < 1) return 0;
  const int k = n_tokens < LBX_MAX_TOKENS ? n_tokens : LBX_MAX_TOKENS;
  size_t s = lbx::ws_bytes_for(projs, n_proj, k);
  if (lbx::wide_auto(projs, n_proj, n_tokens)) s = std::max(s, lbx::wide_ws_bytes(projs, n_proj, n_tokens));
  return s;
}

extern "C" int lbx_linear_verify(const lbx_proj *projs, const lbx_linear_args *a, void *ws,
                                 size_t ws_bytes, cudaStream_t stream) {
  using namespace lbx;
  int rc = check_args(projs, a);
  if (rc) return rc;
  bool handled = false;
  rc = wide_try(projs, a, ws, ws_bytes, stream, handled);
  if (handled) return rc;
  const size_t need = ws_bytes_call(projs, a);
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  // token batches: up to LBX_MAX_TOKENS, fewer when a batch's stages would not
  // fit in shared memory (large ranks); tokens never interact, so the split
  // does not change any token's bits
  int kb = std::min(LBX_MAX_TOKENS, a->n_tokens);
  {
    size_t vmax = 0, umax = 0;
    rc = stage_smem_limits(vmax, umax);
    if (rc) return rc;
    while (kb > 1) {
      LinPrep P;
      if (prep_linear(projs, a, 0, kb, ws, vmax, umax, P) != LBX_EUNSUPPORTED) {
        // a batch whose digits leave room for fewer U tiles per CTA than half
        // the batch would get runs as halves: each CTA quantises every token
        // once per tile group, so the small-tile grid does that work many
        // times over (70B q/k/v at 16 tokens: 196 -> 119 us as two batches)
        LinPrep H;
        if (prep_linear(projs, a, 0, kb / 2, ws, vmax, umax, H) != LBX_OK || H.up.ut <= P.up.ut) break;
      }
      kb >>= 1;
    }
  }
  for (int t0 = 0; t0 < a->n_tokens; t0 += kb) {
    const int k = std::min(kb, a->n_tokens - t0);
    rc = run_batch(projs, a, t0, k, ws, stream);
    if (rc) return rc;
  }
  return LBX_OK;
}

extern "C" int lbx_linear(const lbx_proj *projs, const lbx_linear_args *a, void *ws,
                          size_t ws_bytes, cudaStream_t stream) {
  return lbx_linear_verify(projs, a, ws, ws_bytes, stream);
}

// ---------------------------------------------------------------------------
// Launch floor of a linear call (a benchmarking aid): the call's two stage
// grids with their launch shapes, shared memory and PDL chaining, each CTA
// doing no arithmetic.  MODE 0: trigger, wait for the preceding grid, one
// dependent load and one store per CTA.  MODE 1: also every unit's weight
// bulk copies and the wait for them (the HBM latency a stage has to cover).
// The time of a chain of these against a chain of real calls separates the
// cost of the grid boundaries from the cost of the stage bodies.
// ---------------------------------------------------------------------------
namespace lbx {
template <int MODE>
__global__ void __launch_bounds__(VTHREADS, 2) vfloor_kernel(const __grid_constant__ VParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ LinShm sh;
  linshm_init(sh);
  uint8_t *W = smem_raw + p.s_bytes;
  if (MODE) vstage_issue(p, blockIdx.x, W, sh);
  pdl_trigger();
  pdl_wait();
  bool ok = true;
  if (MODE) ok = __syncthreads_and(mbar_wait_bounded(&sh.bar[UT_MAX], 0, 0x121));
  if (threadIdx.x == 0) {
    const VSeg &sg = p.seg[vseg_of(p, blockIdx.x)];
    const int row0 = (blockIdx.x - sg.unit0) * 16 * p.vt;
    sg.z0[row0] = load_act(p.x, p.xdt, 0) + (ok ? 0.f : 1.f);
  }
}

template <int MODE>
__global__ void __launch_bounds__(UTHREADS, 2) ufloor_kernel(const __grid_constant__ UParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ LinShm sh;
  linshm_init(sh);
  uint8_t *W = smem_raw + p.s_bytes;
  if (MODE) ustage_issue(p, blockIdx.x, W, sh);
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, tile = warp % p.ut;
  const USeg &sg = p.seg[useg_of(p, blockIdx.x)];
  const int n0 = (blockIdx.x - sg.cta0) * (16 * p.ut) + 16 * tile;
  bool ok = true;
  if (MODE && n0 < sg.out) ok = mbar_wait_bounded(&sh.bar[tile], 0, 0x221);
  ok = __syncthreads_and(ok);
  if (threadIdx.x == 0) {
    const float v = __ldcg(sg.z[0]) + (ok ? 0.f : 1.f);
    const int64_t off = (int64_t)(blockIdx.x - sg.cta0) * 16 * p.ut;
    if (p.ydt == LBX_F32)
      reinterpret_cast<float *>(sg.y)[off] = v;
    else
      reinterpret_cast<uint16_t *>(sg.y)[off] = f32_to_bf16(v);
  }
}
}  // namespace lbx

extern "C" int lbx_linear_floor(const lbx_proj *projs, const lbx_linear_args *a, int32_t mode, void *ws,
                                size_t ws_bytes, cudaStream_t stream) {
  using namespace lbx;
  int rc = check_args(projs, a);
  if (rc) return rc;
  LBX_CHECK_ARG(mode == 0 || mode == 1, "mode must be 0 (launches only) or 1 (with weight copies)");
  const size_t need = stage_ws_bytes(projs, a->n_proj, std::min(a->n_tokens, (int32_t)LBX_MAX_TOKENS));
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  size_t vmax = 0, umax = 0;
  rc = stage_smem_limits(vmax, umax);
  if (rc) return rc;
  static DevCache<int> attr;
  int done = 0;
  rc = attr.get(done, [](int &out) {
    cudaError_t e = allow_max_smem(vfloor_kernel<0>);
    if (e == cudaSuccess) e = allow_max_smem(vfloor_kernel<1>);
    if (e == cudaSuccess) e = allow_max_smem(ufloor_kernel<0>);
    if (e == cudaSuccess) e = allow_max_smem(ufloor_kernel<1>);
    out = 1;
    return e != cudaSuccess ? cuda_status(e, "floor kernel attributes") : (int)LBX_OK;
  });
  if (rc) return rc;
  const bool pdl = a->use_pdl != 0;
  for (int t0 = 0; t0 < a->n_tokens; t0 += LBX_MAX_TOKENS) {
    const int k = std::min((int)LBX_MAX_TOKENS, a->n_tokens - t0);
    LinPrep P;
    rc = prep_linear(projs, a, t0, k, ws, vmax, umax, P);
    if (rc) return rc;
    cudaError_t e = launch(mode ? vfloor_kernel<1> : vfloor_kernel<0>, dim3(P.vunits), dim3(VTHREADS),
                           P.v_w + P.v_s, stream, pdl, P.vp);
    if (e == cudaSuccess)
      e = launch(mode ? ufloor_kernel<1> : ufloor_kernel<0>, dim3(P.uunits), dim3(UTHREADS), P.u_w + P.u_s,
                 stream, pdl, P.up);
    if (e != cudaSuccess) return cuda_status(e, "floor launch");
  }
  return LBX_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the scratch lives in a fixed device array
// ---------------------------------------------------------------------------
// Some callers cannot hand the library device memory: a host application that
// owns every device allocation through its own pool, a service that sets up all
// device memory at start-up and may not allocate while serving, or a plugin
// without access to any allocator.  lbx_linear_noalloc runs the same two
// kernels as lbx_linear_verify with its scratch in this module-level array.
// Device code could name the array directly; host code cannot (there the name
// is only a host-side stand-in), so its device address is fetched once per
// device with cudaGetSymbolAddress.

#include <mutex>

namespace lbx {
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(1) << 20;  // 1 MiB, held by every GPU that loads the library
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];
constexpr int NOALLOC_MAX_DEVICES = 64;
static void *g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};
static std::mutex g_noalloc_mu;
}  // namespace lbx

extern "C" size_t lbx_linear_noalloc_max_bytes(void) { return lbx::NOALLOC_SCRATCH_BYTES; }

extern "C" int lbx_linear_noalloc(const lbx_proj *projs, const lbx_linear_args *a,
                                  cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(a, "args is NULL");
  int rc = validate(projs, a->n_proj);
  if (rc) return rc;
  LBX_CHECK_ARG(a->n_tokens >= 1, "n_tokens must be >= 1");
  const size_t need = ws_bytes_call(projs, a);
  LBX_CHECK_SUP(need <= NOALLOC_SCRATCH_BYTES,
                "lbx_linear_noalloc: this call needs %zu bytes of scratch but the fixed buffer holds "
                "%zu; use lbx_linear with a caller-provided workspace",
                need, NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "lbx_linear_noalloc: cudaGetDevice");
  LBX_CHECK_SUP(dev >= 0 && dev < NOALLOC_MAX_DEVICES, "lbx_linear_noalloc: device %d out of range",
                dev);
  void *scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {  // first call on this device: resolve the array's device address
      void *p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_status(e, "lbx_linear_noalloc: cudaGetSymbolAddress");
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  // only the 512-byte header (the cluster executor's range tickets and the
  // grid barrier words) must start at zero: clear it rather than trusting
  // whatever an earlier (possibly failed) call left behind.  z and the per-unit
  // maxima after it are overwritten by every call.
  e = cudaMemsetAsync(scratch, 0, WS_HDR, stream);
  if (e != cudaSuccess) return cuda_status(e, "lbx_linear_noalloc: clear scratch");
  return lbx_linear_verify(projs, a, scratch, NOALLOC_SCRATCH_BYTES, stream);
}

// ---------------------------------------------------------------------------
// Row-sharded layer with its all-gather fused into the U-stage epilogue
// ---------------------------------------------------------------------------
// The exchange needs no fences and no separate signals: each result travels
// as one single-copy-atomic 8-byte word tagged with the call number, and the
// reader polls the words themselves (the flag-in-data scheme of low-latency
// collective protocols).  A per-unit system-scope fence + signal, measured on
// 2 GPUs, cost ~13 us per call at 224 units; the tagged words cost nothing
// beyond the stores.
extern "C" int lbx_linear_allgather(const lbx_proj *proj, const lbx_linear_args *a, int32_t n_peer,
                                    uint64_t *const *xbuf_peers, int64_t half_words, int32_t y_col0,
                                    int64_t ld, const uint32_t *state, void *ws, size_t ws_bytes,
                                    cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(a && proj && state, "NULL argument");
  LBX_CHECK_ARG(n_peer >= 1 && n_peer <= LBX_MAX_PEERS && xbuf_peers, "bad peer list");
  for (int j = 0; j < n_peer; ++j)
    LBX_CHECK_ARG(xbuf_peers[j] && ((uintptr_t)xbuf_peers[j] & 7) == 0,
                  "exchange buffer %d is NULL or not 8-byte aligned", j);
  LBX_CHECK_ARG(a->n_proj == 1, "one projection");
  LBX_CHECK_SUP(a->n_tokens >= 1 && a->n_tokens <= LBX_MAX_TOKENS, "1..%d tokens", LBX_MAX_TOKENS);
  LBX_CHECK_ARG(a->y_dtype == LBX_F32 && a->epilogue == LBX_EPI_STORE, "fp32 y, store epilogue");
  LBX_CHECK_ARG(y_col0 >= 0 && ld >= (int64_t)y_col0 + proj->out_features, "bad output window");
  LBX_CHECK_ARG(half_words >= (int64_t)a->n_tokens * ld, "exchange half too small");
  lbx_linear_args b = *a;
  b.y[0] = xbuf_peers[0];  // the results go to the exchange buffers; y[0] only stands in for the checks
  b.y_ld[0] = ld;
  int rc = check_args(proj, &b);
  if (rc) return rc;
  const size_t need = lbx_linear_workspace_size(proj, 1, a->n_tokens);
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  size_t vmax = 0, umax = 0;
  rc = stage_smem_limits(vmax, umax);
  if (rc) return rc;
  LinPrep P;
  rc = prep_linear(proj, &b, 0, a->n_tokens, ws, vmax, umax, P);
  if (rc) return rc;
  P.up.npeer = n_peer;
  P.up.seq = state;
  P.up.xhalf = half_words;
  for (int j = 0; j < n_peer; ++j)
    P.up.xbuf[j] = reinterpret_cast<unsigned long long *>(xbuf_peers[j]) + y_col0;
  const bool pdl = a->use_pdl != 0;
  auto vk = vstage_for(P.ncb, pm_of(a->prologue), P.vp.vt);
  auto uk = P.ncb == 1   ? ustage_kernel<1, true>
            : P.ncb == 2 ? ustage_kernel<2, true>
                         : ustage_kernel<4, true>;
  static DevCache<int> attr;
  int done = 0;
  rc = attr.get(done, [](int &out) {
    for (auto kk : {ustage_kernel<1, true>, ustage_kernel<2, true>, ustage_kernel<4, true>}) {
      const cudaError_t e0 = allow_max_smem(kk);
      if (e0 != cudaSuccess) return cuda_status(e0, "ustage smem attribute");
    }
    out = 1;
    return (int)LBX_OK;
  });
  if (rc) return rc;
  cudaError_t e = launch(vk, dim3(P.vunits), dim3(VTHREADS), P.v_w + P.v_s, stream, pdl, P.vp);
  if (e != cudaSuccess) return cuda_status(e, "vstage launch");
  e = launch(uk, dim3(P.uunits), dim3(UTHREADS), P.u_w + P.u_s, stream, pdl, P.up);
  return cuda_status(e, "ustage launch");
}

namespace lbx {
constexpr int XU_THREADS = 256;
constexpr int XU_PER = 2;  // words per thread

// Exchange buffer -> plain fp32 y.  Waits (bounded, 1 s) for every word of
// this call; the last CTA advances the call counter state[0] (state[1] is its
// completion ticket, zero between calls).
__global__ void __launch_bounds__(XU_THREADS) allgather_unpack_kernel(
    const unsigned long long *xbuf, long long half, int k, int n, long long ld, float *y,
    long long y_ld, unsigned *state) {
  pdl_trigger();  // the consumer's weight prefetch may start
  pdl_wait();     // this rank's U-stage (and, through it, the previous call) is complete
  const unsigned call = __ldcg(state) + 1u;
  const unsigned long long *src = xbuf + (call & 1u) * half;
  const long long total = (long long)k * n;
  const long long base = ((long long)blockIdx.x * XU_THREADS + threadIdx.x) * XU_PER;
  long long idx[XU_PER];
  unsigned long long w[XU_PER];
  bool ready[XU_PER];
#pragma unroll
  for (int e = 0; e < XU_PER; ++e) {
    const long long i = base + e;
    ready[e] = i >= total;
    const long long t = i / n;
    idx[e] = ready[e] ? 0 : t * ld + (i - t * n);
  }
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    bool all = true;
#pragma unroll
    for (int e = 0; e < XU_PER; ++e)
      if (!ready[e]) {
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[e]) : "l"(src + idx[e]) : "memory");
        ready[e] = (unsigned)(w[e] >> 32) == call;
        all &= ready[e];
      }
    if (all) break;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > 1000000000ull) {  // 1 s: a rank did not deliver
      atomicCAS(&g_lbx_device_error, 0, 0x601);
      break;
    }
  }
#pragma unroll
  for (int e = 0; e < XU_PER; ++e) {
    const long long i = base + e;
    if (i < total) {
      const long long t = i / n;
      y[t * y_ld + (i - t * n)] = ready[e] ? __uint_as_float((unsigned)w[e]) : __int_as_float(0x7fc00000);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(state + 1, 1u);
    if (done == gridDim.x - 1) {  // every CTA has read the call number
      state[1] = 0u;
      state[0] = call;
      __threadfence();
    }
  }
}
}  // namespace lbx

extern "C" int lbx_allgather_unpack(const uint64_t *xbuf, int64_t half_words, int32_t n_tokens,
                                    int32_t n, int64_t ld, float *y, int64_t y_ld, uint32_t *state,
                                    int32_t use_pdl, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(xbuf && y && state, "NULL pointer");
  LBX_CHECK_ARG(((uintptr_t)xbuf & 7) == 0, "exchange buffer must be 8-byte aligned");
  LBX_CHECK_ARG(n_tokens >= 1 && n >= 1 && ld >= n && y_ld >= n, "bad shape");
  LBX_CHECK_ARG(half_words >= (int64_t)n_tokens * ld, "exchange half too small");
  const long long total = (long long)n_tokens * n;
  const int grid = (int)((total + XU_THREADS * XU_PER - 1) / (XU_THREADS * XU_PER));
  const cudaError_t e = launch(allgather_unpack_kernel, dim3(grid), dim3(XU_THREADS), 0, stream,
                               use_pdl != 0, (const unsigned long long *)xbuf, (long long)half_words,
                               (int)n_tokens, (int)n, (long long)ld, y, (long long)y_ld,
                               (unsigned *)state);
  return cuda_status(e, "allgather unpack launch");
}
