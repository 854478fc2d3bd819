// Decode / verify attention over a bf16 KV cache for sm_100a.
//
// Replaces fused_attention (patches/littlebit_cpu_optimized.cpp:1172-1301) and
// the causal loop of full_forward_batch (cpp:1963-2021), adding what the CPU
// path lacks: rotary embedding (HF Llama rotate_half form), a bf16 cache,
// and tree masks for tree verification (tree_utils.py:72-175 masks).
//
// Split over the key sequence in fixed 64-key chunks (flash-decoding): unit
// (chunk c, kv head h, row group g) scores up to 64 query rows of the GQA
// group against its chunk and writes an unnormalised partial (max, sum,
// Σ p·v).  The last live chunk of each (h, g) to finish -- a self-resetting
// ticket -- merges the partials in chunk order, so the whole op is one launch
// (or one phase of a persistent program).
//
// Keys are ordered by their RANK in each query's visible sequence: the cached
// prefix by slot, then the visible new tokens in index order.  Chunk
// membership, lane placement in the reductions and the p·v order all follow
// the rank, so a query's output is the same bit pattern whether it is decoded
// alone, inside a causal verify batch, or as a node of a tree whose ancestors
// sit at scattered slots.
//
// New tokens' keys are rotated, rounded to bf16 and written to the cache by
// the CTA whose slot range holds their slot; every CTA that needs them uses
// the rounded values it computed itself, so no CTA reads a cache slot written
// in the same launch.

#include <type_traits>

#include "common.cuh"

namespace lbx {

constexpr int ACH = 64;        // keys per chunk
constexpr int ATHREADS = 128;
constexpr int AMAX_ROWS = 64;  // query rows (tokens x GQA group) per CTA at most; more rows -> more CTAs
constexpr int ATK_GROUPS = 64; // ticket slots per kv head (row groups of one launch)
constexpr int ARB = 8;         // query rows of one token sharing each key / value load

struct AttnParams {
  int n, heads, kvh, d, max_seq, prefix, rep, R, nchunk, ngroups;
  int rows;  // query rows per unit (row group), <= AMAX_ROWS
  const int32_t *prefix_dev;  // actual cached-slot count (prefix is then a bound)
  float scale, theta;
  const float *q; int64_t q_ld;
  const float *k_new; const float *v_new; int64_t kv_ld;
  const int32_t *pos;
  const uint64_t *tree;
  const float2 *rope;  // [n][d/2] (cos, sin) of each new token's position, or nullptr
  uint16_t *kc; uint16_t *vc;
  float *out;
  float *part_o;     // [kvh][nchunk][R][d]
  float2 *part_ml;   // [kvh][nchunk][R]
  unsigned *ticket;  // [kvh][ATK_GROUPS], zero between launches
  // independent sequences of one launch (nseq > 1): sequence s owns token rows
  // [s*n, (s+1)*n), its caches start seq_stride elements after sequence s-1's,
  // its cached-slot count is prefix_seq[s], and it has its own partials and
  // tickets (part_seq / ml_seq elements and kvh * ATK_GROUPS words apart)
  int nseq;
  int64_t seq_stride, part_seq, ml_seq;
  const int32_t *prefix_seq;
};

// cos/sin of pos * theta^(-2i/d) in double precision, rounded to float (HF
// Llama's LlamaRotaryEmbedding evaluates the same angle in fp32).
LBX_DEV float2 rope_cs_d(int pos, int i, int d, float theta) {
  if (!(theta > 0.f)) return make_float2(1.f, 0.f);  // theta <= 0: no rotation (the reference CPU runtime)
  const double inv = pow((double)theta, -2.0 * (double)i / (double)d);
  double sd, cd;
  sincos((double)pos * inv, &sd, &cd);
  return make_float2((float)cd, (float)sd);
}

LBX_DEV float2 rope_at(const AttnParams &p, int i, int j) {
  return p.rope ? __ldcg(p.rope + i * (p.d >> 1) + j) : rope_cs_d(__ldcg(p.pos + i), j, p.d, p.theta);
}

// table of rope_cs_d for n positions (one launch per decoder step, shared by all layers)
__global__ void rope_table_kernel(const int32_t *__restrict__ pos, int n, int d, float theta,
                                  float2 *__restrict__ out) {
  const int half = d >> 1;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e < n * half) out[e] = rope_cs_d(pos[e / half], e % half, d, theta);
}

// bf16 element counts rounded up to 16 bytes
__host__ __device__ inline int attn_al8(int n) { return (n + 7) & ~7; }

// one unit = (chunk c, kv head h, row group g); S holds its staging buffers.
// B16: keys and values are staged as bf16 (half the shared memory: more units
// per SM, for launches of many sequences); otherwise as fp32 (no conversion
// at use: the lower latency of a single sequence's decode).  Both give the
// same values, so the same bits.
// Chunks at or past the live length do nothing; the last live chunk of (h, g)
// to finish merges the partials.  Runs with any multiple of 32 threads.
template <bool B16>
LBX_DEV void attn_unit(const AttnParams &p, int unit, float *sm) {
  const int d = p.d, half = d / 2, KP = d + 4;  // query row pitch (float4-aligned)
  const int KPB = d + 4;  // key row pitch in bf16 (66 words at d = 128: conflict-free 8-byte loads)
  const int c = unit % p.nchunk;
  const int h = (unit / p.nchunk) % p.kvh;
  const int g = unit / (p.nchunk * p.kvh);
  const int rlo = g * p.rows;                   // this unit's query rows: rlo .. rlo+Rg-1
  const int Rg = min(p.rows, p.R - rlo);
  const int Rcap = p.rows;
  const int tid = threadIdx.x, nthr = blockDim.x;
  // keys (ACH + n rows: cached ranks 0..63, new tokens 64..) and values
  uint16_t *Kb = reinterpret_cast<uint16_t *>(sm);  // B16: (ACH + n) x KPB bf16
  uint16_t *Vb = Kb + attn_al8((ACH + p.n) * KPB);  // B16: (ACH + n) x d bf16
  float *Ka = sm;                                   // fp32: (ACH + n) x KP
  float *Va = Ka + (ACH + p.n) * KP;                // fp32: (ACH + n) x d
  float *Qs = B16 ? reinterpret_cast<float *>(Vb + attn_al8((ACH + p.n) * d)) : Va + (ACH + p.n) * d;  // Rcap x KP
  float *Pm = Qs + Rcap * KP;                   // Rcap x ACH
  int16_t *map = reinterpret_cast<int16_t *>(Pm + Rcap * ACH);  // Rcap x ACH: row of Ka/Va, -1 = none
  uint8_t *sel = reinterpret_cast<uint8_t *>(map + Rcap * ACH);  // n x 64: t-th visible new token
  __shared__ int s_cnt[64];
  __shared__ int s_last;
  __shared__ int s_bstart[AMAX_ROWS + 1];  // row blocks: rows of one token, at most ARB each
  __shared__ int s_nb;

  const int prefix = p.prefix_dev ? __ldcg(p.prefix_dev) : p.prefix;
  const int total = prefix + p.n;
  const int nlive = (total + ACH - 1) / ACH;
  if (c >= nlive) return;  // past the live sequence: no partial, no ticket
  const int64_t pbase = ((int64_t)h * p.nchunk + c) * p.R;
  const int r0 = c * ACH;  // first rank of this chunk
  const bool has_new = r0 + ACH > prefix;  // ranks >= prefix name new tokens

  // visible new tokens of each query in index order (tree: the set bits of
  // its mask, which for generate_tree_buffers trees is root-to-node depth
  // order; causal: 0..i), so rank prefix+t of query i is new token sel[i][t]
  if (has_new && tid < p.n) {
    const int i = tid;
    int cnt = 0;
    if (p.tree) {
      uint64_t m = p.tree[i];
      if (p.n < 64) m &= (1ull << p.n) - 1ull;
      while (m) {
        sel[i * 64 + cnt++] = (uint8_t)(__ffsll((long long)m) - 1);
        m &= m - 1ull;
      }
    } else {
      for (int j = 0; j <= i; ++j) sel[i * 64 + cnt++] = (uint8_t)j;
    }
    s_cnt[i] = cnt;
  }
  // row blocks (the rows of one token share the key / value row of every
  // rank, so one load serves the block's rows)
  if (tid == 0) {
    int nbk = 0;
    for (int r = 0; r < Rg;) {
      s_bstart[nbk++] = r;
      const int i = (rlo + r) / p.rep;
      r = min(min(Rg, (i + 1) * p.rep - rlo), r + ARB);
    }
    s_bstart[nbk] = Rg;
    s_nb = nbk;
  }
  // queries of this row group, rotated
  for (int e = tid; e < Rg * half; e += nthr) {
    const int r = e / half, j = e - r * half;
    const int gr = rlo + r;
    const int i = gr / p.rep, qh = h * p.rep + (gr - i * p.rep);
    const float *qr = p.q + (int64_t)i * p.q_ld + (int64_t)qh * d;
    const float2 cs = rope_at(p, i, j);
    const float x1 = __ldcg(qr + j), x2 = __ldcg(qr + j + half);
    Qs[r * KP + j] = x1 * cs.x - x2 * cs.y;
    Qs[r * KP + j + half] = x2 * cs.x + x1 * cs.y;
  }
  // cached keys / values of ranks r0.. (rank == slot below the prefix): four
  // bf16 per 8-byte load (head_dim % 4 == 0); a batch of KB loads of each is
  // issued before any is stored (one memory round trip for the whole chunk
  // at head_dim 128 and 128 threads)
  const int64_t cache_base = (int64_t)h * p.max_seq * d;
  const int d4 = d / 4;
  constexpr int KB = 16;
  for (int e0 = tid; e0 < ACH * d4; e0 += KB * nthr) {
    uint2 kq[KB], vq[KB];
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const int e = e0 + u * nthr;
      const int jj = e / d4, j4 = e - jj * d4;
      const int slot = r0 + jj;
      kq[u] = vq[u] = make_uint2(0u, 0u);
      if (e < ACH * d4 && slot < prefix) {
        kq[u] = __ldg(reinterpret_cast<const uint2 *>(p.kc + cache_base + (int64_t)slot * d + 4 * j4));
        vq[u] = __ldg(reinterpret_cast<const uint2 *>(p.vc + cache_base + (int64_t)slot * d + 4 * j4));
      }
    }
#pragma unroll
    for (int u = 0; u < KB; ++u) {
      const int e = e0 + u * nthr;
      if (e >= ACH * d4) break;
      const int jj = e / d4, j4 = e - jj * d4;
      if constexpr (B16) {
        *reinterpret_cast<uint2 *>(Kb + jj * KPB + 4 * j4) = kq[u];
        *reinterpret_cast<uint2 *>(Vb + jj * d + 4 * j4) = vq[u];
      } else {
        *reinterpret_cast<float4 *>(Ka + jj * KP + 4 * j4) =
            make_float4(__uint_as_float(kq[u].x << 16), __uint_as_float(kq[u].x & 0xFFFF0000u),
                        __uint_as_float(kq[u].y << 16), __uint_as_float(kq[u].y & 0xFFFF0000u));
        *reinterpret_cast<float4 *>(Va + jj * d + 4 * j4) =
            make_float4(__uint_as_float(vq[u].x << 16), __uint_as_float(vq[u].x & 0xFFFF0000u),
                        __uint_as_float(vq[u].y << 16), __uint_as_float(vq[u].y & 0xFFFF0000u));
      }
    }
  }
  // the new tokens: rotate, round to bf16; the unit whose slot range holds
  // cache slot prefix+i writes it
  if (has_new) {
    for (int e = tid; e < p.n * half; e += nthr) {
      const int i = e / half, j = e - i * half;
      const float *kr = p.k_new + (int64_t)i * p.kv_ld + (int64_t)h * d;
      const float *vr = p.v_new + (int64_t)i * p.kv_ld + (int64_t)h * d;
      const float2 cs = rope_at(p, i, j);
      const float ka = __ldcg(kr + j), kb = __ldcg(kr + j + half);
      const uint16_t b1 = f32_to_bf16(ka * cs.x - kb * cs.y);
      const uint16_t b2 = f32_to_bf16(kb * cs.x + ka * cs.y);
      const uint16_t c1 = f32_to_bf16(__ldcg(vr + j)), c2 = f32_to_bf16(__ldcg(vr + j + half));
      const int slot = prefix + i;
      if (slot >= r0 && slot < r0 + ACH) {
        uint16_t *kw = p.kc + cache_base + (int64_t)slot * d;
        uint16_t *vw = p.vc + cache_base + (int64_t)slot * d;
        kw[j] = b1; kw[j + half] = b2; vw[j] = c1; vw[j + half] = c2;
      }
      if constexpr (B16) {
        Kb[(ACH + i) * KPB + j] = b1; Kb[(ACH + i) * KPB + j + half] = b2;
        Vb[(ACH + i) * d + j] = c1; Vb[(ACH + i) * d + j + half] = c2;
      } else {
        Ka[(ACH + i) * KP + j] = bf16_to_f32(b1); Ka[(ACH + i) * KP + j + half] = bf16_to_f32(b2);
        Va[(ACH + i) * d + j] = bf16_to_f32(c1); Va[(ACH + i) * d + j + half] = bf16_to_f32(c2);
      }
    }
  }
  __syncthreads();

  // scores by rank: every quantity below depends only on the key's rank in
  // the query's visible sequence.  A thread takes one rank for a whole row
  // block (one key row, loaded once per step); each score is the same fmaf
  // chain over the head dimension as a thread per (row, rank) would form.
  const int nbk = s_nb;
  // (the row count of a block as a compile-time bound: a one-row block, every
  // row of a multi-head-attention step, runs no predicated-off rows)
  // rows ra .. ra+nr of block bi (the block's map row is written once, by its
  // first part)
  auto score_block = [&](auto nrc, int bi, int jj, int ra, int nr) {
    constexpr int NR = decltype(nrc)::value;
    const int i = (rlo + ra) / p.rep;
    const int rank = r0 + jj;
    int row = -1;
    if (rank < prefix) {
      row = jj;
    } else {
      const int t = rank - prefix;
      if (has_new && t < s_cnt[i]) row = ACH + sel[i * 64 + t];
    }
    if (ra == s_bstart[bi]) map[bi * ACH + jj] = (int16_t)row;
    float a[NR];
#pragma unroll
    for (int u = 0; u < NR; ++u) a[u] = 0.f;
    if (row >= 0) {
      for (int t = 0; t < d / 4; ++t) {
        float4 kv;
        if constexpr (B16) {
          const uint2 kw = reinterpret_cast<const uint2 *>(Kb + row * KPB)[t];
          kv = make_float4(__uint_as_float(kw.x << 16), __uint_as_float(kw.x & 0xFFFF0000u),
                           __uint_as_float(kw.y << 16), __uint_as_float(kw.y & 0xFFFF0000u));
        } else {
          kv = reinterpret_cast<const float4 *>(Ka + row * KP)[t];
        }
#pragma unroll
        for (int u = 0; u < NR; ++u) {
          if (u < nr) {
            const float4 qv = reinterpret_cast<const float4 *>(Qs + (ra + u) * KP)[t];
            float x = a[u];
            x = fmaf(qv.x, kv.x, x);
            x = fmaf(qv.y, kv.y, x);
            x = fmaf(qv.z, kv.z, x);
            x = fmaf(qv.w, kv.w, x);
            a[u] = x;
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < NR; ++u)
      if (u < nr) Pm[(ra + u) * ACH + jj] = row >= 0 ? a[u] * p.scale : -INFINITY;
  };
  // with threads to spare, each block's rows are scored in two halves (a
  // decode step's GQA block of 8 rows fills 64 of 128 threads otherwise)
  const int S = nbk * ACH * 2 <= nthr ? 2 : 1, HR = ARB / S;
  for (int e = tid; e < nbk * ACH * S; e += nthr) {
    const int bh = e / ACH, jj = e - bh * ACH;
    const int bi = bh / S, h = bh - bi * S;
    const int ra = s_bstart[bi] + h * HR, nr = min(s_bstart[bi + 1] - ra, HR);
    if (nr <= 0) continue;
    if (nr == 1) score_block(std::integral_constant<int, 1>{}, bi, jj, ra, nr);
    else if (nr <= 2) score_block(std::integral_constant<int, 2>{}, bi, jj, ra, nr);
    else if (nr <= 4) score_block(std::integral_constant<int, 4>{}, bi, jj, ra, nr);
    else score_block(std::integral_constant<int, ARB>{}, bi, jj, ra, nr);
  }
  __syncthreads();

  // chunk-local softmax numerators
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < Rg; r += nthr / 32) {
    const float s0 = Pm[r * ACH + lane], s1 = Pm[r * ACH + lane + 32];
    const float m = warp_max(fmaxf(s0, s1));
    float e0 = 0.f, e1 = 0.f;
    if (m != -INFINITY) {
      e0 = s0 == -INFINITY ? 0.f : expf(s0 - m);
      e1 = s1 == -INFINITY ? 0.f : expf(s1 - m);
    }
    Pm[r * ACH + lane] = e0;
    Pm[r * ACH + lane + 32] = e1;
    const float l = warp_sum(e0 + e1);
    if (lane == 0) p.part_ml[pbase + rlo + r] = make_float2(m, l);
  }
  __syncthreads();

  // Σ p·v in rank order (ranks without a key carry p = 0).  A thread takes
  // one head-dimension column for a whole row block (one value load per rank
  // serves the block's rows); each output is the same fmaf chain over the
  // ranks as a thread per (row, column) would form.
  auto pv_block = [&](auto nrc, int bi, int t) {
    constexpr int NR = decltype(nrc)::value;
    const int ra = s_bstart[bi], nr = s_bstart[bi + 1] - ra;
    const int16_t *mr = map + bi * ACH;
    float a[NR];
#pragma unroll
    for (int u = 0; u < NR; ++u) a[u] = 0.f;
    for (int j0 = 0; j0 < ACH; j0 += 4) {
      float v[4];
#pragma unroll
      for (int jq = 0; jq < 4; ++jq) {
        const int row = mr[j0 + jq];
        v[jq] = B16 ? bf16_to_f32(Vb[(row < 0 ? 0 : row) * d + t]) : Va[(row < 0 ? 0 : row) * d + t];
      }
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        if (u < nr) {
          const float4 pq = *reinterpret_cast<const float4 *>(Pm + (ra + u) * ACH + j0);
          float x = a[u];
          x = fmaf(pq.x, v[0], x);
          x = fmaf(pq.y, v[1], x);
          x = fmaf(pq.z, v[2], x);
          x = fmaf(pq.w, v[3], x);
          a[u] = x;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < NR; ++u)
      if (u < nr) p.part_o[(pbase + rlo + ra + u) * d + t] = a[u];
  };
  for (int e = tid; e < nbk * d; e += nthr) {
    const int bi = e / d, t = e - bi * d;
    const int nr = s_bstart[bi + 1] - s_bstart[bi];
    if (nr == 1) pv_block(std::integral_constant<int, 1>{}, bi, t);
    else if (nr <= 2) pv_block(std::integral_constant<int, 2>{}, bi, t);
    else if (nr <= 4) pv_block(std::integral_constant<int, 4>{}, bi, t);
    else pv_block(std::integral_constant<int, ARB>{}, bi, t);
  }

  // the last live chunk of (h, g) merges the partials, in chunk order
  __threadfence();
  __syncthreads();
  unsigned *tk = p.ticket + h * ATK_GROUPS + g;
  if (tid == 0) s_last = atomicAdd(tk, 1u) == (unsigned)(nlive - 1);
  __syncthreads();
  // (identical arithmetic in both forms: M = max of the chunk maxima, then
  // in chunk order over the chunks with keys w = exp(m - M), L += w*l,
  // O += w*o, out = O / L)
  // staged merge for long sequences (more than 16 chunks: the per-output
  // form below then needs 6 or more L2 round trips per output), when its
  // tables fit in the key / value buffers
  const int scratch = B16 ? (attn_al8((ACH + p.n) * KPB) + (ACH + p.n) * d) / 2 : (ACH + p.n) * (KP + d);  // floats
  const bool staged = nlive > 16 && 2 * Rg * nlive + Rg <= scratch;
  if (s_last && staged) {
    __threadfence();
    // per (row, chunk) (m, l) into shared memory, all loads in flight; per
    // row M, the weights (-1: a chunk without keys) and L; then each output
    // loads its chunks' partial sums a batch at a time
    float *wsm = reinterpret_cast<float *>(Kb);  // [Rg][nlive]: m, then w
    float *lsm = wsm + Rg * nlive;               // [Rg][nlive]: l
    float *Lsm = lsm + Rg * nlive;       // [Rg]
#pragma unroll 4
    for (int i = tid; i < Rg * nlive; i += nthr) {
      const int r = i / nlive, c = i - r * nlive;
      const float2 ml = __ldcg(p.part_ml + ((int64_t)h * p.nchunk + c) * p.R + rlo + r);
      wsm[i] = ml.x;
      lsm[i] = ml.y;
    }
    __syncthreads();
    for (int r = tid; r < Rg; r += nthr) {
      float M = -INFINITY;
      for (int c = 0; c < nlive; ++c) M = fmaxf(M, wsm[r * nlive + c]);
      float L = 0.f;
      for (int c = 0; c < nlive; ++c) {
        const float m = wsm[r * nlive + c];
        float w = -1.f;
        if (m != -INFINITY) {
          w = expf(m - M);
          L = fmaf(w, lsm[r * nlive + c], L);
        }
        wsm[r * nlive + c] = w;
      }
      Lsm[r] = L;
    }
    __syncthreads();
    constexpr int CB = 16;  // chunks whose partial sums one thread loads together
    for (int e = tid; e < Rg * d; e += nthr) {
      const int r = e / d, t = e - r * d;
      const float *wr = wsm + r * nlive;
      float O = 0.f;
      for (int c0 = 0; c0 < nlive; c0 += CB) {
        float ov[CB];
#pragma unroll
        for (int u = 0; u < CB; ++u) {
          ov[u] = 0.f;
          if (c0 + u < nlive && wr[c0 + u] >= 0.f)
            ov[u] = __ldcg(p.part_o + (((int64_t)h * p.nchunk + c0 + u) * p.R + rlo + r) * d + t);
        }
#pragma unroll
        for (int u = 0; u < CB; ++u)
          if (c0 + u < nlive && wr[c0 + u] >= 0.f) O = fmaf(wr[c0 + u], ov[u], O);
      }
      const float L = Lsm[r];
      const int gr = rlo + r;
      const int i = gr / p.rep, qh = h * p.rep + (gr - i * p.rep);
      p.out[(int64_t)i * p.heads * d + (int64_t)qh * d + t] = L > 0.f ? O / L : 0.f;
    }
    if (tid == 0) *tk = 0u;  // ready for the next launch
  } else if (s_last) {  // per output, the partials straight from L2
    __threadfence();
    constexpr int MB = 8;  // chunks whose partials are loaded together
    for (int e = tid; e < Rg * d; e += nthr) {
      const int r = e / d, t = e - r * d;
      const int gr = rlo + r;
      float M = -INFINITY;
      for (int c0 = 0; c0 < nlive; c0 += MB) {
        float mx[MB];
#pragma unroll
        for (int u = 0; u < MB; ++u)
          mx[u] = c0 + u < nlive ? __ldcg(p.part_ml + ((int64_t)h * p.nchunk + c0 + u) * p.R + gr).x
                                 : -INFINITY;
#pragma unroll
        for (int u = 0; u < MB; ++u) M = fmaxf(M, mx[u]);
      }
      float L = 0.f, O = 0.f;  // in chunk order
      for (int c0 = 0; c0 < nlive; c0 += MB) {
        float2 ml[MB];
        float ov[MB];
#pragma unroll
        for (int u = 0; u < MB; ++u) {
          ml[u] = make_float2(-INFINITY, 0.f);
          ov[u] = 0.f;
          if (c0 + u < nlive) {
            const int64_t b = ((int64_t)h * p.nchunk + c0 + u) * p.R + gr;
            ml[u] = __ldcg(p.part_ml + b);
            ov[u] = __ldcg(p.part_o + b * d + t);
          }
        }
#pragma unroll
        for (int u = 0; u < MB; ++u) {
          if (ml[u].x == -INFINITY) continue;
          const float w = expf(ml[u].x - M);
          L = fmaf(w, ml[u].y, L);
          O = fmaf(w, ov[u], O);
        }
      }
      const int i = gr / p.rep, qh = h * p.rep + (gr - i * p.rep);
      p.out[(int64_t)i * p.heads * d + (int64_t)qh * d + t] = L > 0.f ? O / L : 0.f;
    }
    if (tid == 0) *tk = 0u;  // ready for the next launch
  }
  __syncthreads();  // the unit's shared buffers are free again
}

// the parameters of sequence s of a multi-sequence launch: one sequence's
// attention exactly as a launch of its own would see it
LBX_DEV AttnParams attn_seq(const AttnParams &p, int s) {
  AttnParams q = p;
  const int64_t rows = (int64_t)s * p.n;
  q.q += rows * p.q_ld;
  q.k_new += rows * p.kv_ld;
  q.v_new += rows * p.kv_ld;
  q.pos += rows;
  if (q.tree) q.tree += rows;
  if (q.rope) q.rope += rows * (p.d >> 1);
  q.kc += s * p.seq_stride;
  q.vc += s * p.seq_stride;
  q.out += rows * p.heads * p.d;
  q.prefix_dev = p.prefix_seq + s;
  q.part_o += s * p.part_seq;
  q.part_ml += s * p.ml_seq;
  q.ticket += (int64_t)s * p.kvh * ATK_GROUPS;
  q.nseq = 1;
  return q;
}

template <bool B16>
__global__ void __launch_bounds__(ATHREADS, B16 ? 4 : 1) attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  pdl_trigger();
  pdl_wait();
  if (p.nseq > 1) {
    const int s = blockIdx.z / p.ngroups, g = blockIdx.z - s * p.ngroups;
    const AttnParams ps = attn_seq(p, s);
    attn_unit<B16>(ps, blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * g), sm);
  } else {
    attn_unit<B16>(p, blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), sm);
  }
}

static int attn_sm_count() { return device_sm_count(); }

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
  // query rows per unit: a kv head's whole GQA group (and tokens) up to
  // AMAX_ROWS, halved while the units would not cover the SMs twice (the
  // rows of one unit are scored one after another; each row's arithmetic is
  // the same whichever unit holds it)
  p.nseq = a->n_seq > 1 ? a->n_seq : 1;
  int rows = p.R < AMAX_ROWS ? p.R : AMAX_ROWS;
  while (rows > 1 && (int64_t)p.nchunk * p.kvh * p.nseq * ((p.R + rows - 1) / rows) < 2 * attn_sm_count() &&
         (p.R + (rows + 1) / 2 - 1) / ((rows + 1) / 2) <= ATK_GROUPS)
    rows = (rows + 1) / 2;
  p.rows = rows;
  p.ngroups = (p.R + rows - 1) / rows;
  p.scale = a->scale;
  p.theta = a->theta;
  p.q = a->q;
  p.q_ld = a->q_ld ? a->q_ld : (int64_t)a->heads * a->head_dim;
  p.k_new = a->k_new;
  p.v_new = a->v_new;
  p.kv_ld = a->kv_ld ? a->kv_ld : (int64_t)a->kv_heads * a->head_dim;
  p.pos = a->pos;
  p.tree = a->tree_mask;
  p.rope = reinterpret_cast<const float2 *>(a->rope_cs);
  p.kc = a->k_cache;
  p.vc = a->v_cache;
  p.out = a->out;
  p.prefix_dev = a->prefix_dev;
  p.seq_stride = a->cache_seq_stride;
  p.prefix_seq = a->prefix_seq;
}

// scratch: [tickets: fixed size and offset, whatever n is] [partials]
struct AttnWs {
  size_t tk, o, ml, total;
};

static size_t attn_ticket_bytes(int kv_heads, int n_seq = 1) {
  return ((size_t)kv_heads * ATK_GROUPS * 4 * (n_seq > 1 ? n_seq : 1) + 255) & ~(size_t)255;
}

// partials: [seq][kvh][nchunk][R][d] floats, then [seq][kvh][nchunk][R] (max, sum)
static size_t attn_partial_bytes(const lbx_attn_args *a, size_t *ml_off) {
  const int rep = a->heads / a->kv_heads;
  const int64_t R = (int64_t)a->n * rep;
  const int64_t nchunk = (a->prefix_len + a->n + ACH - 1) / ACH;
  const int64_t S = a->n_seq > 1 ? a->n_seq : 1;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const size_t o = al((size_t)S * a->kv_heads * nchunk * R * a->head_dim * 4);
  if (ml_off) *ml_off = o;
  return o + al((size_t)S * a->kv_heads * nchunk * R * 8);
}

static AttnWs attn_ws_layout(const lbx_attn_args *a) {
  AttnWs w;
  w.tk = 0;
  w.o = attn_ticket_bytes(a->kv_heads, a->n_seq);
  size_t ml = 0;
  const size_t part = attn_partial_bytes(a, &ml);
  w.ml = w.o + ml;
  w.total = w.o + part;
  return w;
}

// validated parameters of one attention op with explicit scratch pointers
// (lbx_forward keeps the tickets at a fixed offset of its own workspace)
// b16: the shared-memory size of the bf16-staged unit (attn_unit<true>)
static int attn_prep(const lbx_attn_args *a, void *partials, unsigned *tickets, AttnParams &p,
                     size_t &smem, bool b16 = false) {
  LBX_CHECK_ARG(a, "args is NULL");
  LBX_CHECK_ARG(a->n >= 1 && a->n <= 64, "n must be in [1,64]");
  LBX_CHECK_ARG(a->kv_heads >= 1 && a->heads >= a->kv_heads && a->heads % a->kv_heads == 0,
                "heads must be a multiple of kv_heads");
  LBX_CHECK_SUP(a->head_dim > 0 && a->head_dim <= 128 && a->head_dim % 4 == 0,
                "head_dim must be a multiple of 4 and <= 128");
  LBX_CHECK_ARG(a->prefix_len >= 0 && a->prefix_len + a->n <= a->max_seq,
                "prefix_len + n exceeds max_seq");
  LBX_CHECK_ARG(a->q && a->k_new && a->v_new && a->pos && a->k_cache && a->v_cache && a->out,
                "NULL pointer");
  LBX_CHECK_ARG(a->n_seq <= 1 || (a->prefix_seq && a->cache_seq_stride >= (int64_t)a->kv_heads * a->max_seq *
                                                                             a->head_dim),
                "multi-sequence attention needs prefix_seq and a cache stride of at least one sequence's cache");
  LBX_CHECK_ARG(a->n_seq >= 0 && a->n_seq <= LBX_ATTN_MAX_SEQ, "n_seq must be in [0,%d]", LBX_ATTN_MAX_SEQ);
  p = AttnParams{};
  attn_fill(a, p);
  LBX_CHECK_SUP(p.ngroups <= ATK_GROUPS, "too many query rows (n * heads/kv_heads)");
  size_t ml = 0;
  attn_partial_bytes(a, &ml);
  p.part_o = reinterpret_cast<float *>(partials);
  p.part_ml = reinterpret_cast<float2 *>(reinterpret_cast<uint8_t *>(partials) + ml);
  p.ticket = tickets;
  p.part_seq = (int64_t)p.kvh * p.nchunk * p.R * p.d;
  p.ml_seq = (int64_t)p.kvh * p.nchunk * p.R;
  const int Rcap = p.rows;
  const int KP = p.d + 4, KPB = p.d + 4;
  const size_t kv = b16 ? ((size_t)attn_al8((ACH + p.n) * KPB) + (size_t)attn_al8((ACH + p.n) * p.d)) * 2
                        : ((size_t)(ACH + p.n) * KP + (size_t)(ACH + p.n) * p.d) * 4;
  smem = kv + ((size_t)Rcap * KP + (size_t)Rcap * ACH) * 4 + (size_t)Rcap * ACH * 2 + (size_t)p.n * 64;
  return LBX_OK;
}

static int attn_launch(const lbx_attn_args *a, void *partials, unsigned *tickets, cudaStream_t stream) {
  AttnParams p;
  size_t smem = 0;
  // many sequences: bf16 staging (more units per SM); one sequence: fp32 (lower latency)
  const bool b16 = a->n_seq > 1;
  int rc = attn_prep(a, partials, tickets, p, smem, b16);
  if (rc) return rc;
  static DevCache<size_t> smax_cache;
  size_t smax = 0;
  rc = smax_cache.get(smax, [](size_t &out) {
    size_t o2 = 0;
    cudaError_t e = allow_max_smem(attn_kernel<false>, &out);
    if (e == cudaSuccess) e = allow_max_smem(attn_kernel<true>, &o2);
    out = std::min(out, o2);
    return e != cudaSuccess ? cuda_status(e, "attn smem attribute") : (int)LBX_OK;
  });
  if (rc) return rc;
  LBX_CHECK_SUP(smem <= smax, "attention needs %zu bytes of shared memory (max %zu)", smem, smax);
  const bool pdl = a->use_pdl != 0;
  const dim3 grid(p.nchunk, p.kvh, p.ngroups * p.nseq);
  const cudaError_t e = b16 ? launch(attn_kernel<true>, grid, dim3(ATHREADS), smem, stream, pdl, p)
                            : launch(attn_kernel<false>, grid, dim3(ATHREADS), smem, stream, pdl, p);
  return cuda_status(e, "attn launch");
}

}  // namespace lbx

extern "C" size_t lbx_attn_workspace_size(const lbx_attn_args *a) {
  if (!a || a->n < 1 || a->kv_heads < 1 || a->heads < a->kv_heads) return 0;
  return lbx::attn_ws_layout(a).total;
}

extern "C" int lbx_attn_decode(const lbx_attn_args *a, void *ws, size_t ws_bytes,
                               cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(a && a->n >= 1 && a->kv_heads >= 1 && a->heads >= a->kv_heads, "bad arguments");
  const AttnWs W = attn_ws_layout(a);
  LBX_CHECK_ARG(ws && ws_bytes >= W.total, "workspace too small (%zu < %zu)", ws_bytes, W.total);
  uint8_t *w = reinterpret_cast<uint8_t *>(ws);
  return attn_launch(a, w + W.o, reinterpret_cast<unsigned *>(w + W.tk), stream);
}

extern "C" int lbx_rope_table(const int32_t *pos, int32_t n, int32_t head_dim, float theta, float *out,
                              cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(pos && out && n >= 1 && head_dim >= 2 && head_dim % 2 == 0, "bad arguments");
  const int tot = n * (head_dim / 2);
  rope_table_kernel<<<(tot + 127) / 128, 128, 0, stream>>>(pos, n, head_dim, theta,
                                                            reinterpret_cast<float2 *>(out));
  return cuda_status(cudaGetLastError(), "rope table launch");
}
