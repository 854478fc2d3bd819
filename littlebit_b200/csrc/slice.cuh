// Split-rank cluster executor: one LittleBit linear call in one launch.
//
// The grid is a set of clusters of SL_S CTAs.  Each cluster owns a contiguous
// run of 128-rank quantisation groups of one V segment (one own-V branch of
// one projection, both branches for a shared-V residual):
//   1. each CTA computes up to SL_VT 16-row tiles of z for those groups, with
//      the V-stage's staging, block order and fixed-order reductions;
//   2. each CTA stores its z rows into every cluster CTA's shared memory
//      (distributed shared memory); after one cluster barrier every CTA holds
//      the cluster's z, derives the group
//      exponents and int8 digits exactly as the U-stage does, and contracts
//      its range of the projection's output rows against the cluster's
//      groups: one exact int32 sum per (output row, token, group), written to
//      the workspace with the group exponents;
//   3. per (projection, output range) a ticket picks the last CTA to finish;
//      it combines every cluster's group sums with the U-stage's integer
//      rounding (rshr to the branch's coarsest exponent) and epilogue.
// No grid-wide barrier and no second kernel: the only synchronisation across
// clusters is the per-range ticket.  The rank is never replicated, so each
// packed weight is read once per call.  Results are bit-identical to the two
// stage grids (same integers, same float operations in the same order).
//
// Sign fragments are fetched before the dependent-launch wait, V into
// registers and U into shared memory, so the kernel needs no mbarriers, two
// CTAs fit on an SM, and the next call's prologue overlaps this call.

// address of the same shared-memory location in CTA `rank` of this cluster
template <class T>
LBX_DEV const T *cl_map(const T *p, int rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
  return reinterpret_cast<const T *>(r);
}
template <class T>
LBX_DEV T *cl_map_w(T *p, int rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
  return reinterpret_cast<T *>(r);
}
LBX_DEV void cl_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
LBX_DEV void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
LBX_DEV void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
LBX_DEV int cl_rank() {
  int r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

constexpr int SL_S = 16;      // CTAs per cluster (non-portable size)
constexpr int SL_VT = 4;      // V tiles per CTA
constexpr int SL_UP = 8;      // U (tile, group) pairs per warp
constexpr int SL_MAXCL = 16;  // clusters per launch
constexpr int SL_ZR = SL_VT * 16;

struct SlCluster {
  int proj, vseg;
  int row0, rows;  // V rows [row0, row0 + rows) of segment vseg (row0 a multiple of 128)
  int tpc;         // V tiles per CTA
  int nplane;      // z planes: 1, or 2 for a shared-V segment (plane 1 = the residual branch)
  int br[2];       // branch of each plane
};

struct SlProj {
  int out, nbr;
  const int32_t *u_sign[2];
  int words[2];  // sign words per U row
  int ngrp[2];   // quantisation groups per branch
  const float *u1[2];
  const float *bias;
  void *y;
  int64_t y_ld;
  int rtiles;    // output tiles per CTA range (range j: tiles [j*rtiles, (j+1)*rtiles))
  int ncl;       // clusters contributing to this projection
  int *part;     // [ngrp[0] + ngrp[1]][k][out] exact group sums
  int *gexp;     // [2][ZGMAX][LBX_MAX_TOKENS] group exponents
};

struct SlParams {
  VParams vp;  // staging and V segments (vcap = 0, z pointers unused)
  SlCluster cl[SL_MAXCL];
  SlProj pj[LBX_MAX_PROJ];
  int ncl;
  int ydt, epi;
  unsigned *ticket;  // [LBX_MAX_PROJ][SL_S], zero between calls
  int zcap;          // rows per gathered z plane
  int rmax;          // output rows per range
  int ugmax;         // z groups per cluster plane
  int fin_rows;      // output rows per finalize chunk
  // dynamic shared memory: [V staging | U digits | finalize staging] at 0
  int o_red, o_zall, o_mid, o_ue, o_u1, o_uw, o_fin;
};

// one 4-word group of a 16-row sign tile against the digits at aw (word
// 4*G + q of the group for thread q), sign words of rows g and g+8 in wa, wb
template <int NCB>
LBX_DEV void mma_group(int (&acc)[NCB][4], uint32_t wa, uint32_t wb, const uint32_t *aw, int ncols,
                       int lane) {
  const int n8 = lane >> 2;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int sh = 16 * (r >> 1) + 2 * (r & 1);
    const int slot = 4 * (r >> 1) + 2 * (r & 1);
    const uint32_t a0 = negbits4(wa >> sh);
    const uint32_t a2 = negbits4(wa >> (sh + 1));
    const uint32_t a1 = negbits4(wb >> sh);
    const uint32_t a3 = negbits4(wb >> (sh + 1));
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

LBX_DEV int sl_part_index(const SlProj &P, int b, int grp, int t, int k, int n) {
  return (((b ? P.ngrp[0] : 0) + grp) * k + t) * P.out + n;
}
LBX_DEV int sl_gexp_index(int b, int grp, int t) { return (b * ZGMAX + grp) * LBX_MAX_TOKENS + t; }

#ifndef LBX_SL_MINBLOCKS
#define LBX_SL_MINBLOCKS 2  // resident CTAs per SM the register budget allows
#endif

template <int NCB>
__global__ void __launch_bounds__(VTHREADS, LBX_SL_MINBLOCKS) slice_kernel(const __grid_constant__ SlParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ LinShm sh;
  __shared__ int s_last;
  __shared__ int s_ec[2][LBX_MAX_TOKENS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int cid = blockIdx.x / SL_S;
  const int j = cl_rank();
  const SlCluster &C = p.cl[cid];
  const VParams &vp = p.vp;
  const VSeg &sg = vp.seg[C.vseg];
  const SlProj &P = p.pj[C.proj];
  const int k = vp.k, ncols = vp.ncols, ws = act_ws(ncols), Wv = vp.Wv;
  uint32_t *act = reinterpret_cast<uint32_t *>(smem);  // V staging, then the U digits
  float *red = reinterpret_cast<float *>(smem + p.o_red);
  float *zall = reinterpret_cast<float *>(smem + p.o_zall);  // [plane][k][zcap], filled by the cluster
  uint2 *suw = reinterpret_cast<uint2 *>(smem + p.o_uw);      // [SL_UP][warp][lane] U sign words
  float *smid = reinterpret_cast<float *>(smem + p.o_mid);   // [plane][SL_ZR]
  int *sue = reinterpret_cast<int *>(smem + p.o_ue);          // [plane*ugmax][k] exponents
  int *ssq = sue + 2 * p.ugmax * k;                           // [plane*ugmax][k] digit sums
  float *su1 = reinterpret_cast<float *>(smem + p.o_u1);      // [3][rmax]: u1_0, u1_1, bias
  LBX_PROBE(30);

  // ---- this CTA's share: V tiles and output tiles
  const int ctiles = (C.rows + 15) / 16;
  const int t0 = j * C.tpc;
  const int ntl = max(0, min(C.tpc, ctiles - t0));
  const int myrow0 = C.row0 + t0 * 16;
  const int myrows = max(0, min(ntl * 16, C.rows - t0 * 16));
  const int ngc = (C.rows + UGRP - 1) / UGRP;  // groups per plane
  const int nug = C.nplane * ngc;
  const int rt0 = j * P.rtiles;
  const int nrt = max(0, min(P.rtiles, P.out / 16 - rt0));
  const int npair = nrt * nug;
  const bool vblk = BLK_WORDS * warp < Wv;

  // ---- prologue (independent of the inputs)
  if (tid < VWARPS * LBX_MAX_TOKENS) (&sh.v_ssq[0][0])[tid] = 0.f;
  uint32_t vw[SL_VT][2][2];
#pragma unroll
  for (int tl = 0; tl < SL_VT; ++tl)
#pragma unroll
    for (int G = 0; G < 2; ++G)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        vw[tl][G][h] = 0u;
        const int row = myrow0 + tl * 16 + g + 8 * h;
        const int w = BLK_WORDS * warp + 4 * G + q;
        if (tl < ntl && vblk && w < Wv && row < sg.rank) vw[tl][G][h] = __ldg(sg.v_sign + (int64_t)row * Wv + w);
      }
#pragma unroll
  for (int pi = 0; pi < SL_UP; ++pi) {  // U sign words of this CTA's (output tile, group) pairs
    const int pair = warp + pi * VWARPS;
    uint2 u = make_uint2(0u, 0u);
    if (pair < npair) {
      const int rt = pair / nug, ug = pair - rt * nug;
      const int pl = ug / ngc, gl = ug - pl * ngc;
      const int b = C.br[pl];
      const int w = (C.row0 / UGRP + gl) * 4 + q;
      const int n = (rt0 + rt) * 16 + g;
      if (w < P.words[b]) {
        u.x = __ldg(P.u_sign[b] + (int64_t)n * P.words[b] + w);
        u.y = __ldg(P.u_sign[b] + (int64_t)(n + 8) * P.words[b] + w);
      }
    }
    if (pi * VWARPS < npair) suw[(pi * VWARPS + warp) * 32 + lane] = u;
  }
  for (int r = tid; r < myrows; r += VTHREADS) {
    smid[r] = __ldg(sg.mid0 + myrow0 + r);
    if (sg.mid1) smid[SL_ZR + r] = __ldg(sg.mid1 + myrow0 + r);
  }
  for (int r = tid; r < nrt * 16; r += VTHREADS) {
    const int n = rt0 * 16 + r;
    su1[r] = __ldg(P.u1[0] + n);
    if (P.nbr > 1) su1[p.rmax + r] = __ldg(P.u1[1] + n);
    if (P.bias) su1[2 * p.rmax + r] = __ldg(P.bias + n);
  }
  {  // v2 / norm_w of the staging columns and this CTA's U sign rows into L2
    const int col = tid * 8;
    if (ntl > 0 && col < vp.K) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(sg.v2 + col));
      if (vp.prologue == LBX_PRO_RMSNORM) asm volatile("prefetch.global.L2 [%0];" ::"l"(vp.norm_w + col));
    }
  }
  __syncthreads();
  cl_arrive_relaxed();  // this CTA has started (its shared memory may receive stores)
  LBX_PROBE(31);
  pdl_trigger();
  pdl_wait();
  cl_wait();  // every CTA of the cluster has started
  LBX_PROBE(32);

  // ---- V: this CTA's z rows
  if (ntl > 0) {
    if (vp.prologue == LBX_PRO_SILU_MUL)
      vstage_stage<PM_SILU>(vp, sg.v2, nullptr, nullptr, 0, act, sh, [] {});
    else if (vp.prologue == LBX_PRO_MUL)
      vstage_stage<PM_MUL>(vp, sg.v2, nullptr, nullptr, 0, act, sh, [] {});
    else
      vstage_stage<PM_X>(vp, sg.v2, nullptr, nullptr, 0, act, sh, [] {});
    __syncthreads();
    LBX_PROBE(33);
#pragma unroll
    for (int tl = 0; tl < SL_VT; ++tl) {
      if (tl < ntl) {
        int acc[NCB][4];
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) acc[cb][0] = acc[cb][1] = acc[cb][2] = acc[cb][3] = 0;
        if (vblk) {
          mma_group<NCB>(acc, vw[tl][0][0], vw[tl][0][1], act + (BLK_WORDS * warp + q) * ws, ncols, lane);
          if (BLK_WORDS * warp + 4 < Wv)
            mma_group<NCB>(acc, vw[tl][1][0], vw[tl][1][1], act + (BLK_WORDS * warp + 4 + q) * ws, ncols,
                           lane);
        }
        float *rw = red + (tl * VWARPS + warp) * 16 * k;
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
          const int t = cb * 4 + q;
          if (t < k) {
            float v0 = 0.f, v1 = 0.f;
            if (vblk) {  // (a single pass: the V-stage's running sum starts from this value)
              const int sq = sh.v_sq[warp][t];
              const float inv = sh.v_inv[warp][t];
              v0 += __fmul_rn(__int2float_rn(sq + 2 * (256 * acc[cb][0] + acc[cb][1])), inv);
              v1 += __fmul_rn(__int2float_rn(sq + 2 * (256 * acc[cb][2] + acc[cb][3])), inv);
            }
            rw[g * k + t] = v0;
            rw[(g + 8) * k + t] = v1;
          }
        }
      }
    }
    LBX_PROBE(40);
    __syncthreads();
    LBX_PROBE(41);
    const bool rms = vp.prologue == LBX_PRO_RMSNORM;
    for (int i = tid; i < myrows * k; i += VTHREADS) {
      const int rr = i / k, t = i - rr * k;
      const int tl = rr >> 4, r16 = rr & 15;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < VWARPS; ++w) v += red[((tl * VWARPS + w) * 16 + r16) * k + t];
      if (rms) {
        float s2 = 0.f;
#pragma unroll
        for (int w = 0; w < VWARPS; ++w) s2 += sh.v_ssq[w][t];
        v *= rsqrtf(s2 / (float)vp.K + vp.eps);
      }
      // into the gathered z of every CTA of the cluster (this CTA's rows
      // start at cluster row t0 * 16)
      const float z0 = smid[rr] * v;
      const float z1 = sg.mid1 ? smid[SL_ZR + rr] * v : 0.f;
      float *d0 = zall + t * p.zcap + t0 * 16 + rr;
      float *d1 = zall + (k + t) * p.zcap + t0 * 16 + rr;
#pragma unroll 4
      for (int s2 = 0; s2 < SL_S; ++s2) {
        *cl_map_w(d0, s2) = z0;
        if (sg.mid1) *cl_map_w(d1, s2) = z1;
      }
    }
  }
  LBX_PROBE(42);
  __syncthreads();
  LBX_PROBE(34);
  cl_arrive();  // this CTA's z rows are in every CTA of the cluster
  cl_wait();
  LBX_PROBE(35);

  LBX_PROBE(36);

  // ---- group exponents (warp per (group, token)) and digits
  for (int it = warp; it < nug * k; it += VWARPS) {
    const int ug = it / k, t = it - ug * k;
    const int pl = ug / ngc, gl = ug - pl * ngc;
    const float *zp = zall + (pl * k + t) * p.zcap + gl * UGRP;
    const int lim = min(UGRP, C.rows - gl * UGRP);
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = lane + 32 * e;
      if (r < lim) m = fmaxf(m, fabsf(zp[r]));
    }
    m = __int_as_float(__reduce_max_sync(0xffffffffu, __float_as_int(m)));
    const int ex = m > 0.f ? u_group_exp(m) : UE_NONE;
    const float sc = ex == UE_NONE ? 0.f : pow2f(ex);
    // item (Wd, slot) of the group: the U-stage's digit layout
    const int Wd = lane >> 3, slot = lane & 7, hh = slot >> 2, jj = slot & 3;
    int hi[4], lo[4], sq = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int pos = 32 * Wd + 16 * hh + jj + 4 * e;
      const float z = pos < lim ? zp[pos] : 0.f;
      const int qv = __float2int_rn(z * sc);
      sq += qv;
      split_digits(qv, hi[e], lo[e]);
    }
    uint32_t *aw = act + (ug * 4 + Wd) * ws + 2 * t;
    aw[slot * ncols] = pack4(hi[0], hi[1], hi[2], hi[3]);
    aw[slot * ncols + 1] = pack4(lo[0], lo[1], lo[2], lo[3]);
    sq = __reduce_add_sync(0xffffffffu, sq);
    if (lane == 0) {
      sue[ug * k + t] = ex;
      ssq[ug * k + t] = sq;
      P.gexp[sl_gexp_index(C.br[pl], C.row0 / UGRP + gl, t)] = ex;  // (every CTA of the cluster: same value)
    }
  }
  __syncthreads();
  LBX_PROBE(37);

  // ---- U contraction: exact group sums of this CTA's output rows
#pragma unroll
  for (int pi = 0; pi < SL_UP; ++pi) {
    const int pair = warp + pi * VWARPS;
    if (pair < npair) {
      const int rt = pair / nug, ug = pair - rt * nug;
      const int pl = ug / ngc, gl = ug - pl * ngc;
      int acc[NCB][4];
#pragma unroll
      for (int cb = 0; cb < NCB; ++cb) acc[cb][0] = acc[cb][1] = acc[cb][2] = acc[cb][3] = 0;
      const uint2 u = suw[(pi * VWARPS + warp) * 32 + lane];
      mma_group<NCB>(acc, u.x, u.y, act + (ug * 4 + q) * ws, ncols, lane);
      const int n = (rt0 + rt) * 16 + g;
#pragma unroll
      for (int cb = 0; cb < NCB; ++cb) {
        const int t = cb * 4 + q;
        if (t < k) {
          const int sq = ssq[ug * k + t];
          int *pp = P.part + sl_part_index(P, C.br[pl], C.row0 / UGRP + gl, t, k, n);
          pp[0] = sq + 2 * (256 * acc[cb][0] + acc[cb][1]);
          pp[8] = sq + 2 * (256 * acc[cb][2] + acc[cb][3]);
        }
      }
    }
  }
  __syncthreads();
  LBX_PROBE(38);

  // ---- the last CTA of this output range combines the clusters' group sums
  if (tid == 0) {  // release this CTA's sums, acquire the other clusters' (CTA barrier above)
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(old) : "l"(p.ticket + C.proj * SL_S + j) : "memory");
    s_last = old == (unsigned)P.ncl - 1u;
  }
  __syncthreads();
  if (s_last) {
    int *fe = reinterpret_cast<int *>(smem + p.o_fin);  // [2][ZGMAX][k] exponents
    const int ng0 = P.ngrp[0], ng1 = P.nbr > 1 ? P.ngrp[1] : 0;
    // exponents: loaded together with the first chunk's sums below
    int fe_at = -1, fe_v = 0;
    {
      const int i = VTHREADS - 1 - tid;
      if (i < (ng0 + ng1) * k) {
        const int b = i < ng0 * k ? 0 : 1;
        const int r = b ? i - ng0 * k : i;
        const int grp = r / k, t = r - grp * k;
        fe_at = (b * ZGMAX + grp) * k + t;
        fe_v = __ldcg(P.gexp + sl_gexp_index(b, grp, t));
      }
    }
    // group sums of the range through shared memory in chunks (all loads of
    // a chunk in flight together)
    int *fs = fe + 2 * ZGMAX * k;  // [group][k][fin_rows]
    const int R = nrt * 16;  // (0 for a range past the last output tile)
    for (int c0 = 0; c0 < R; c0 += p.fin_rows) {
      const int cr = min(p.fin_rows, R - c0);
      const int tot = (ng0 + ng1) * k * cr;
      for (int i0 = tid; i0 < tot; i0 += 12 * VTHREADS) {  // 12 loads in flight per thread
        int v[12];
#pragma unroll
        for (int u = 0; u < 12; ++u) {
          const int i = i0 + u * VTHREADS;
          v[u] = 0;
          if (i < tot) {
            const int gt = i / cr, r = i - gt * cr;
            v[u] = __ldcg(P.part + gt * P.out + rt0 * 16 + c0 + r);
          }
        }
#pragma unroll
        for (int u = 0; u < 12; ++u)
          if (i0 + u * VTHREADS < tot) fs[i0 + u * VTHREADS] = v[u];
      }
      if (c0 == 0 && fe_at >= 0) fe[fe_at] = fe_v;
      __syncthreads();
      if (c0 == 0) {  // the coarsest exponent per (branch, token)
        if (tid < 2 * k) {
          const int b = tid / k, t = tid - b * k;
          const int ng = b ? ng1 : ng0;
          int ec = UE_NONE;
          for (int grp = 0; grp < ng; ++grp) ec = min(ec, fe[(b * ZGMAX + grp) * k + t]);
          s_ec[b][t] = ec == UE_NONE ? 0 : ec;
        }
        __syncthreads();
      }
      for (int i = tid; i < cr * k; i += VTHREADS) {
        const int t = i / cr, r = i - t * cr;
        int I0 = 0, I1 = 0;
        for (int grp = 0; grp < ng0; ++grp) {
          const int ex = fe[grp * k + t];
          if (ex != UE_NONE) I0 += rshr(fs[(grp * k + t) * cr + r], ex - s_ec[0][t]);
        }
        for (int grp = 0; grp < ng1; ++grp) {
          const int ex = fe[(ZGMAX + grp) * k + t];
          if (ex != UE_NONE) I1 += rshr(fs[((ng0 + grp) * k + t) * cr + r], ex - s_ec[1][t]);
        }
        const int rr = c0 + r;
        const int n = rt0 * 16 + rr;
        float v = u_result(su1[rr], I0, s_ec[0][t], P.nbr > 1, su1[p.rmax + rr], I1, s_ec[1][t],
                           P.bias != nullptr, su1[2 * p.rmax + rr]);
        if (p.epi == LBX_EPI_SILU0 && C.proj == 0) v = v / (1.0f + expf(-v));
        const int64_t off = (int64_t)t * P.y_ld + n;
        if (p.ydt == LBX_F32) {
          float *y = reinterpret_cast<float *>(P.y) + off;
          if (p.epi == LBX_EPI_ADD) v += *y;
          *y = v;
        } else {
          reinterpret_cast<uint16_t *>(P.y)[off] = f32_to_bf16(v);
        }
      }
      __syncthreads();
    }
    if (tid == 0) p.ticket[C.proj * SL_S + j] = 0u;
  }
  LBX_PROBE(39);
  // (no shared memory of another CTA is touched after the cluster barrier)
}
