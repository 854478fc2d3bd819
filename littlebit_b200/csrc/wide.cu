// Tensor-core batches of a linear call: up to 64 tokens per launch on the
// fifth-generation tensor cores (tcgen05.mma kind::i8, accumulators in TMEM).
//
// The stage grids contract the sign matrices with warp-level mma.sync over at
// most 16 tokens per launch; a call with many tokens (a batch of independent
// sequences, a long verification) then re-streams every packed weight once
// per 16 tokens and spends most of its time expanding sign bits for the
// legacy tensor path.  Here a batch of up to 64 tokens is one pass over the
// weights in three grids:
//
//   wx_stage_kernel  x -> per (V segment, 256-column block) a record holding
//                    the int8 digit pairs of every token as the MMA's B
//                    operand image (K-major, 128-byte swizzle) and the
//                    block scales; the RMSNorm factor per token
//   wv_kernel        one CTA per 128 ranks of a V segment: the sign rows are
//                    expanded to +-1 bytes in shared memory (operand A), each
//                    block is 8 tcgen05.mma (M=128, N=2*tokens, K=32) into a
//                    TMEM accumulator, read back with tcgen05.ld and scaled
//                    and summed in the stage grids' order; the tile's z is
//                    quantised with its group exponent straight into the
//                    U-stage's B operand image (a tile of 128 ranks is one
//                    U quantisation group)
//   wu_kernel        one CTA per 128 output rows: per quantisation group,
//                    4 tcgen05.mma over the group's 128 ranks; the exact int32
//                    group sums are rounded to the branch's coarsest exponent
//                    and added, then the shared epilogue (u_result)
//
// Every token's bits are those of the stage grids (the integers fed to each
// rounding are equal: sum(s*q) with s = +-1 bytes equals the stage grids'
// sum(q) + 2*sum(A*q) with A = 0/-1 bytes, and each float operation is the
// same expression in the same order), so the executor changes no result.
//
// Within every 32-column (32-rank) word the K order of both operands is the
// permutation that makes the sign expansion one byte-select per 4 bytes:
// K byte 4*j + i holds column bit (j < 4 ? j : j + 12) + 4*i.  A contraction
// does not depend on the order of its K terms, so A and B only need to agree.
#include "common.cuh"

namespace lbx {

constexpr int WD_MAXK = 64;       // tokens per tensor-core batch
constexpr int WD_NBV = 4;         // B-operand buffers of the V kernel
constexpr int WD_NBU = 8;         // B-operand buffers of the U kernel
constexpr int WD_NAU = 4;         // A-operand / TMEM accumulator buffers of the U kernel
constexpr int WD_MAXBLK = 512;    // 256-column blocks (in_features <= 131072)
constexpr int WX_THREADS = 512;
constexpr int WD_PD = 4;          // sign-word loads in flight ahead of the expansion (blocks / groups)

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
LBX_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LBX_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// (one full warp)
LBX_DEV void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
LBX_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[128 x N] (+)= A[128 x 32] . B[N x 32]^T, s8 x s8 -> s32, both K-major
LBX_DEV void umma_i8(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every tcgen05.mma issued so far by this thread completed
LBX_DEV void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
LBX_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x NC consecutive 32-bit columns: thread i gets lane (base lane + i)
template <int NC>
LBX_DEV void tmem_ld(uint32_t taddr, uint32_t *r);
template <>
LBX_DEV void tmem_ld<4>(uint32_t a, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
template <>
LBX_DEV void tmem_ld<8>(uint32_t a, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(a));
}
template <>
LBX_DEV void tmem_ld<16>(uint32_t a, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a));
}
template <>
LBX_DEV void tmem_ld<32>(uint32_t a, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a));
}
// NC columns in loads of at most 32
template <int NC>
LBX_DEV void tmem_ld_cols(uint32_t a, uint32_t *r) {
  if constexpr (NC <= 32) {
    tmem_ld<NC>(a, r);
  } else {
    tmem_ld<32>(a, r);
    tmem_ld_cols<NC - 32>(a + 32, r + 32);
  }
}

// Shared-memory matrix descriptor of a K-major operand in 128-byte swizzle
// atoms (8 rows x 128 bytes, 1024-byte aligned, stacked every 1024 bytes):
// start address >> 4 in bits 0-13, leading byte offset 16 B (unused by this
// layout), stride byte offset 1024 B, descriptor version 1 (bit 46), swizzle
// mode 2 (128 B) in bits 61-63.  Advancing the start by 32 bytes selects the
// next K=32 slice inside the atom (the swizzle applies to the full address).
LBX_DEV uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// instruction descriptor: D s32 (bits 4-5 = 2), A and B s8 (bits 7-9, 10-12
// = 1), both K-major, N >> 3 in bits 17-22, M >> 4 = 8 (M = 128) in bits 24-28
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// byte offset of (row n, K byte c < 128) in a stack of swizzled atoms
LBX_DEV uint32_t sw128_off(int n, int c) {
  return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((c >> 4) ^ n) & 7) << 4) + (c & 15));
}
// K byte position, within its 32-byte word, of column bit b (0..31)
LBX_DEV int wd_pos(int b) {
  const int h = b >> 4, bl = b & 15;
  return 4 * ((bl & 3) + 4 * h) + (bl >> 2);
}
// four sign bits (bit 0 of each selector nibble) -> +1 (bit 0) / -1 (bit 1) bytes
LBX_DEV uint32_t pm1bits4(uint32_t sel) { return negbits4(sel) | 0x01010101u; }
// one 32-bit sign word -> its 32 +-1 bytes in the permuted K order (two 16-byte chunks)
LBX_DEV void wd_expand(uint32_t w, uint4 &c0, uint4 &c1) {
  c0 = make_uint4(pm1bits4(w), pm1bits4(w >> 1), pm1bits4(w >> 2), pm1bits4(w >> 3));
  c1 = make_uint4(pm1bits4(w >> 16), pm1bits4(w >> 17), pm1bits4(w >> 18), pm1bits4(w >> 19));
}
// asynchronous global -> shared copies of this thread's own sign words (the
// thread reads them back after cp.async.wait_group; no barrier involved).
// src_bytes 0 fills zeros without reading.
LBX_DEV void cpa16(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
LBX_DEV void cpa8(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
LBX_DEV void cpa4(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
LBX_DEV void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
LBX_DEV void cpa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

LBX_DEV uint8_t *align1024(uint8_t *p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// ---------------------------------------------------------------------------
// parameters
// ---------------------------------------------------------------------------
struct WSeg {              // one V segment (a branch with its own V)
  const int32_t *v_sign;   // [rank, Wv]
  const float *v2;         // [K]
  const float *mid0, *mid1;  // mid1: the shared-V residual's mid, or nullptr
  int rank, tile0;         // first wv CTA of the segment
  uint8_t *xrec;           // [nblk] x rec_bytes: B image of x digits, then KP block scales
  float *rs;               // [KP] RMSNorm factor per token
  uint8_t *urec0, *urec1;  // U records of the branch(es) this segment feeds: [groups] x urec_bytes
};
struct WUProj {
  const int32_t *u_sign[2];
  const float *u1[2];
  const uint8_t *urec[2];  // [groups] x urec_bytes: B image of z digits, then KP group exponents
  int words[2], ng[2];
  int nbr, out, tile0;     // first wu CTA of the projection
  const float *bias;
  void *y;
  int64_t y_ld;
};
struct WParams {
  WSeg seg[2 * LBX_MAX_PROJ];
  WUProj up[LBX_MAX_PROJ];
  int nseg, nproj;
  int K, Wv, nblk, k, KP;  // KP: tokens of the records (the batch padded to 8, 16, 32 or 64)
  int vts, uts;            // token splits of the V and U grids: a CTA takes KP / splits tokens
  int xdt, prologue, ydt, epi;
  float eps;
  const void *x, *x2;
  const float *norm_w;
  int rec_bytes;   // x record: 2*KP*256 image bytes + KP floats, 16-byte multiple
  int urec_bytes;  // U record: 2*KP*128 image bytes + KP ints, 16-byte multiple
};

// ---------------------------------------------------------------------------
// x staging: CTA (token t, segment s); warp w stages blocks w, w+16, ...
// with the stage grids' per-block arithmetic (vstage_stage)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(WX_THREADS) wx_stage_kernel(const __grid_constant__ WParams p) {
  __shared__ float ssq[16];
  __shared__ __align__(16) uint8_t scr[16][512];  // per warp: [digit][atom][128 K bytes]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x;
  const WSeg &sg = p.seg[blockIdx.y];
  const int N = 2 * p.KP;
  LBX_PROBE(30);
  if (lane == 0) ssq[warp] = 0.f;
  pdl_trigger();
  pdl_wait();
  LBX_PROBE(31);
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const int pm = pm_of(p.prologue);
  uint8_t *sw = scr[warp];
  for (int b = warp; b < p.nblk; b += 16) {
    const int64_t col = (int64_t)b * 256 + 8 * lane;
    const bool valid = col < p.K;
    float xv[8], uv[8], hw[8];
    if (valid) {
      load8(p.x, p.xdt, (int64_t)t * p.K + col, xv);
      if (pm != PM_X) load8(p.x2, p.xdt, (int64_t)t * p.K + col, uv);
      load8f(sg.v2 + col, hw);
      if (rms) {
        float nw[8];
        load8f(p.norm_w + col, nw);
#pragma unroll
        for (int i = 0; i < 8; ++i) hw[i] *= nw[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = uv[i] = hw[i] = 0.f;
    }
    float a[8];
    float sq2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float xx = xv[i];
      if (pm == PM_SILU) {
        a[i] = (xx / (1.0f + expf(-xx))) * uv[i] * hw[i];
      } else if (pm == PM_MUL) {
        a[i] = xx * uv[i] * hw[i];
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
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int qv = __float2int_rn(a[i] * sc);
      int hi, lo;
      split_digits(qv, hi, lo);
      const int c = 8 * lane + i;  // column within the block
      const int off = (c >> 7) * 128 + ((c & 127) >> 5) * 32 + wd_pos(c & 31);
      sw[off] = (uint8_t)hi;
      sw[256 + off] = (uint8_t)lo;
    }
    if (rms) {
      sq2 = warp_sum(sq2);
      if (lane == 0) ssq[warp] += sq2;
    }
    __syncwarp();
    {
      const int d = lane >> 4, at = (lane >> 3) & 1, c = lane & 7;
      const int n = 2 * t + d;
      uint8_t *rec = sg.xrec + (size_t)b * p.rec_bytes;
      *reinterpret_cast<uint4 *>(rec + (size_t)at * N * 128 + sw128_off(n, 16 * c)) =
          *reinterpret_cast<const uint4 *>(sw + d * 256 + at * 128 + 16 * c);
      if (lane == 0) reinterpret_cast<float *>(rec + (size_t)N * 256)[t] = m / QMAX;
    }
    __syncwarp();
  }
  if (rms) {
    __syncthreads();
    if (tid == 0) {
      float s2 = 0.f;
      for (int w = 0; w < 16; ++w) s2 += ssq[w];
      sg.rs[t] = rsqrtf(s2 / (float)p.K + p.eps);
    }
  }
  LBX_PROBE(32);
}

// ---------------------------------------------------------------------------
// Warp roles of the tensor-core stages: warps 0-15 expand the sign rows
// (operand A) and read the accumulators back; warp 16 issues the operand-B
// copies and the MMAs.  They meet only at mbarriers:
//   afull[j]  the 512 expanding threads have written A buffer j
//   dfull[j]  the MMAs into TMEM buffer j (and their reads of A buffer j and
//             of the B buffer) completed (tcgen05.commit)
//   dfree[j]  the 512 reading threads have loaded TMEM buffer j and read what
//             they need of the step's B buffer
// Every wait gives up after 1 s or as soon as another thread gave up (the
// CTA's abort flag), so a fault anywhere ends the kernel promptly.
// ---------------------------------------------------------------------------
constexpr int WD_CW = 512;                // expanding / reading threads
constexpr int WD_TPB = WD_CW + 32;        // plus the issuing warp

// (try_wait suspends the thread in hardware until the phase completes or a
// short time limit passes, so waiting warps leave the issue slots to the
// working ones)
LBX_DEV bool wd_wait(uint64_t *bar, uint32_t parity, int code, volatile int *abort) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 7u) == 0) {
      if (*abort) return false;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (it == 0) t0 = t;
      else if (t - t0 > 1000000000ull) {
        *abort = 1;
        atomicCAS(&g_lbx_device_error, 0, code);
        return false;
      }
    }
  }
}
LBX_DEV void mbar_arrive1(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------
// V-stage on the tensor cores.  Expanding thread (row = tid % 128, quarter =
// tid / 128) expands 2 of the 8 sign words of its row's block and reads TMEM
// lane `row` (its warp's lane quarter) for tokens [quarter*KP/4, +KP/4).
// ---------------------------------------------------------------------------
template <int KP>
__global__ void __launch_bounds__(WD_TPB, 1) wv_kernel(const __grid_constant__ WParams p) {
  constexpr int N = 2 * KP, KQ = KP / 4;
  constexpr int SB = N * 256 + 1024;  // B buffer: image (two atoms of N x 128 B), then the block scales
  constexpr uint32_t IDESC = idesc_i8(N);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sA = align1024(smem_raw);  // 2 x (2 atoms x 128 rows x 128 B)
  uint8_t *sB = sA + 2 * 32768;        // WD_NBV x SB
  uint2 *sQ = reinterpret_cast<uint2 *>(sB + WD_NBV * SB);  // [WD_PD][WD_CW] sign-word ring
  __shared__ __align__(8) uint64_t bbar[WD_NBV];
  __shared__ __align__(8) uint64_t afull[2], dfull[2], dfree[2];
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  __shared__ uint16_t blist[WD_MAXBLK];
  __shared__ int gmx[2][KP];
  __shared__ int gex[KP];
  __shared__ float gsc[KP];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool cw = tid < WD_CW;
  const int row = tid & 127, qd = (tid >> 7) & 3;
  // CTA = (tile, token split): tokens t0 .. t0+KP of the batch's KPR
  const int tile = (int)blockIdx.x / p.vts, t0 = ((int)blockIdx.x - tile * p.vts) * KP;
  const int NR = 2 * p.KP;  // rows of the records' operand images
  int si = 0;
  while (si + 1 < p.nseg && tile >= p.seg[si + 1].tile0) ++si;
  const WSeg &sg = p.seg[si];
  const int grp = tile - sg.tile0;
  const int rr = grp * 128 + row;
  const bool rvalid = cw && rr < sg.rank;
  const int nb = p.nblk;
  const int k = p.k - t0;  // valid tokens from t0 on (may exceed KP)
  volatile int *abrt = &abort_flag;
  LBX_PROBE(40);

  if (tid == 0) {
    // block order: per 16-block slot w its passes in order, slots in order
    // (the stage grids' per-warp running sums, then the sum over warps)
    int i = 0;
    for (int w = 0; w < 16; ++w)
      for (int b = w; b < nb; b += 16) blist[i++] = (uint16_t)(b | (b + 16 >= nb ? 0x8000 : 0));
    for (int j = 0; j < WD_NBV; ++j) mbar_init(&bbar[j], 1);
    for (int j = 0; j < 2; ++j) {
      mbar_init(&afull[j], WD_CW);
      mbar_init(&dfull[j], 1);
      mbar_init(&dfree[j], WD_CW);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (tid < 2 * KP) (&gmx[0][0])[tid] = 0;
  if (warp == 16) tmem_alloc(&tbase, 2 * N);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;

  const int32_t *vrow = sg.v_sign + (int64_t)(rvalid ? rr : 0) * p.Wv;
  // this thread's 2 sign words of block i into ring slot i % WD_PD (one commit group per block)
  auto load_bits = [&](int i) {
    const int w0 = i < nb ? 8 * (blist[i] & 0x7fff) + 2 * qd : 0;
    const bool v = i < nb && rvalid && w0 < p.Wv;
    cpa8(&sQ[(i % WD_PD) * WD_CW + tid], vrow + (v ? w0 : 0), v ? 8u : 0u);
    cpa_commit();
  };
  if (cw) {
#pragma unroll
    for (int j = 0; j + 1 < WD_PD; ++j) load_bits(j);
  }
  LBX_PROBE(41);
  pdl_trigger();
  pdl_wait();  // x records come from the staging grid
  LBX_PROBE(42);

  float T[KQ], V[KQ];
#pragma unroll
  for (int i = 0; i < KQ; ++i) T[i] = V[i] = 0.f;

  if (warp == 16) {
    // ---- issuing warp (lane 0 acts, the warp stays converged)
    int nissued = 0, ncommit = 0;
    // this CTA's rows of each image atom, and its tokens' block scales (rows
    // 2*t0 .. are a whole number of 8-row swizzle atoms, so the copies keep the layout)
    auto issue_b = [&](int i) {
      if (lane == 0) {
        const int buf = i % WD_NBV;
        const uint8_t *rec = sg.xrec + (size_t)(blist[i] & 0x7fff) * p.rec_bytes;
        uint8_t *dst = sB + buf * SB;
        mbar_arrive_expect_tx(&bbar[buf], (uint32_t)(2 * N * 128 + KP * 4));
        bulk_g2s(dst, rec + (size_t)2 * t0 * 128, N * 128u, &bbar[buf]);
        bulk_g2s(dst + N * 128, rec + (size_t)NR * 128 + (size_t)2 * t0 * 128, N * 128u, &bbar[buf]);
        bulk_g2s(dst + N * 256, rec + (size_t)NR * 256 + (size_t)t0 * 4, KP * 4u, &bbar[buf]);
      }
      ++nissued;
    };
    for (int j = 0; j < WD_NBV && j < nb; ++j) issue_b(j);
    for (int i = 0; i < nb; ++i) {
      if (i >= 2) {  // TMEM buffer i & 1 and the B buffer of block i-2 are free again
        if (!__all_sync(0xffffffffu, wd_wait(&dfree[i & 1], (uint32_t)((i - 2) >> 1) & 1u, 0x706, abrt))) break;
        if (i + 2 < nb) issue_b(i + 2);
      }
      if (!__all_sync(0xffffffffu, wd_wait(&afull[i & 1], (uint32_t)(i >> 1) & 1u, 0x707, abrt))) break;
      if (!__all_sync(0xffffffffu, wd_wait(&bbar[i % WD_NBV], (uint32_t)(i / WD_NBV) & 1u, 0x701, abrt))) break;
      __syncwarp();
      tc_fence_after();
      if (lane == 0) {
        const uint32_t aB = smem_u32(sA + (i & 1) * 32768), bB = smem_u32(sB + (i % WD_NBV) * SB);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const int at = s >> 2, ko = 32 * (s & 3);
          umma_i8(tmem + (uint32_t)((i & 1) * N), sw128_desc(aB + at * 16384 + ko),
                  sw128_desc(bB + at * N * 128 + ko), IDESC, s > 0 ? 1u : 0u);
        }
        umma_commit(&dfull[i & 1]);
      }
      ++ncommit;
      __syncwarp();
    }
    if (*abrt && lane == 0) {  // work in flight ends before shared memory and TMEM are released
      const int nused = ncommit;
      for (int j = nused; j < nissued; ++j) mbar_poll_cta(&bbar[j % WD_NBV], (uint32_t)(j / WD_NBV) & 1u, 0x704);
      if (ncommit > 0) mbar_poll_cta(&dfull[(ncommit - 1) & 1], (uint32_t)((ncommit - 1) >> 1) & 1u, 0x705);
    }
    __syncwarp();
  } else {
    // ---- expanding / reading warps
    auto epilogue = [&](int j) {
      bool okw = wd_wait(&dfull[j & 1], (uint32_t)(j >> 1) & 1u, 0x702, abrt) &&
                 wd_wait(&bbar[j % WD_NBV], (uint32_t)(j / WD_NBV) & 1u, 0x703, abrt);
      okw = __all_sync(0xffffffffu, okw);
      tc_fence_after();
      if (!okw) return false;
      const float *inv = reinterpret_cast<const float *>(sB + (j % WD_NBV) * SB + N * 256) + qd * KQ;
      float iv[KQ];
#pragma unroll
      for (int i = 0; i < KQ; ++i) iv[i] = inv[i];
      const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)((j & 1) * N + qd * 2 * KQ);
      uint32_t r[2 * KQ];
      tmem_ld_cols<2 * KQ>(ta, r);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive1(&dfree[j & 1]);
#pragma unroll
      for (int i = 0; i < KQ; ++i) {
        const int val = 256 * (int)r[2 * i] + (int)r[2 * i + 1];
        T[i] += __fmul_rn(__int2float_rn(val), iv[i]);
      }
      if (blist[j] & 0x8000) {
#pragma unroll
        for (int i = 0; i < KQ; ++i) {
          V[i] += T[i];
          T[i] = 0.f;
        }
      }
      return true;
    };
    for (int i = 0; i < nb; ++i) {
      if (i == 10) LBX_PROBE(45);
      load_bits(i + WD_PD - 1);
      cpa_wait<WD_PD - 1>();  // block i's words have landed
      // A buffer i & 1 is free once the MMAs of block i-2 completed
      if (i >= 2 && !__all_sync(0xffffffffu, wd_wait(&dfull[i & 1], (uint32_t)((i - 2) >> 1) & 1u, 0x708, abrt)))
        break;
      if (i == 10) LBX_PROBE(46);
      {
        uint8_t *a = sA + (i & 1) * 32768 + (qd >> 1) * 16384;
        const uint2 q = sQ[(i % WD_PD) * WD_CW + tid];
        const int c0 = 64 * (qd & 1);
        uint4 e0, e1;
        wd_expand(q.x, e0, e1);
        *reinterpret_cast<uint4 *>(a + sw128_off(row, c0)) = e0;
        *reinterpret_cast<uint4 *>(a + sw128_off(row, c0 + 16)) = e1;
        wd_expand(q.y, e0, e1);
        *reinterpret_cast<uint4 *>(a + sw128_off(row, c0 + 32)) = e0;
        *reinterpret_cast<uint4 *>(a + sw128_off(row, c0 + 48)) = e1;
      }
      fence_proxy_async();
      mbar_arrive1(&afull[i & 1]);
      if (i == 10) LBX_PROBE(47);
      if (i >= 1 && !epilogue(i - 1)) break;
      if (i == 10) LBX_PROBE(49);
    }
    if (!*abrt) epilogue(nb - 1);
    cpa_wait<0>();
  }
  LBX_PROBE(43);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool ok = !*abrt;
  if (warp == 16) tmem_dealloc(tmem, 2 * N);
  if (!ok) return;

  // ---- z = mid (.) v (RMSNorm: v * rs first), the group exponent per token
  // over the tile's 128 ranks, and the digits into the U records
  const bool rms = p.prologue == LBX_PRO_RMSNORM;
  const int nside = sg.mid1 ? 2 : 1;
  const float m0 = rvalid ? sg.mid0[rr] : 0.f;
  const float m1 = rvalid && sg.mid1 ? sg.mid1[rr] : 0.f;
#pragma unroll
  for (int i = 0; i < KQ; ++i) {
    const int t = qd * KQ + i;
    float vv = V[i];
    if (rms && cw && t < k) vv *= __ldcg(sg.rs + t0 + t);
    T[i] = vv;
  }
  uint8_t *img = sA;  // staging images of the two sides (the A buffers are free)
  for (int sd = 0; sd < nside; ++sd) {
    const float mm = sd ? m1 : m0;
    if (cw) {
#pragma unroll
      for (int i = 0; i < KQ; ++i) {
        const int t = qd * KQ + i;
        const float z = rvalid && t < k ? mm * T[i] : 0.f;
        V[i] = z;
        const int mb = __reduce_max_sync(0xffffffffu, __float_as_int(fabsf(z)));
        if (lane == 0 && mb) atomicMax(&gmx[sd][t], mb);
      }
    }
    __syncthreads();
    if (tid < KP) {  // the group exponent of each token, once
      const float gm = __int_as_float(gmx[sd][tid]);
      const int ex = tid < k && gm > 0.f ? u_group_exp(gm) : UE_NONE;
      gex[tid] = ex;
      gsc[tid] = ex == UE_NONE ? 0.f : pow2f(ex);
    }
    __syncthreads();
    uint8_t *im = img + sd * 16384;
    if (cw) {
      const int pos = 32 * (row >> 5) + wd_pos(row & 31);
#pragma unroll
      for (int i = 0; i < KQ; ++i) {
        const int t = qd * KQ + i;
        const int qv = t < k ? __float2int_rn(V[i] * gsc[t]) : 0;
        int hi, lo;
        split_digits(qv, hi, lo);
        im[sw128_off(2 * t, pos)] = (uint8_t)hi;
        im[sw128_off(2 * t + 1, pos)] = (uint8_t)lo;
      }
    }
    __syncthreads();
    // (this CTA's tokens' rows of the record image: bytes 2*t0*128 on, the layout kept)
    uint8_t *rec = (sd ? sg.urec1 : sg.urec0) + (size_t)grp * p.urec_bytes;
    for (int o = 16 * tid; o < N * 128; o += 16 * WD_TPB)
      *reinterpret_cast<uint4 *>(rec + (size_t)2 * t0 * 128 + o) = *reinterpret_cast<const uint4 *>(im + o);
    if (tid < KP) reinterpret_cast<int *>(rec + (size_t)NR * 128)[t0 + tid] = gex[tid];
    __syncthreads();  // (gex / gsc are rewritten by the next side)
  }
  LBX_PROBE(44);
}

// ---------------------------------------------------------------------------
// U-stage on the tensor cores.  Expanding thread (row, quarter) as in
// wv_kernel; rows are output rows, the K dimension one quantisation group
// (128 ranks) per step, each thread expanding one of the group's 4 sign
// words of its row.
// ---------------------------------------------------------------------------
template <int KP>
__global__ void __launch_bounds__(WD_TPB, 1) wu_kernel(const __grid_constant__ WParams p) {
  constexpr int N = 2 * KP, KQ = KP / 4;
  constexpr int SBU = ((N * 128 + KP * 4) + 1023) & ~1023;  // B buffer: image, then the group exponents
  constexpr uint32_t IDESC = idesc_i8(N);
  constexpr int NA = WD_NAU, D = WD_NAU - 1;  // A / TMEM buffers; groups the read-back trails the expansion by
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sA = align1024(smem_raw);  // NA x (128 rows x 128 B)
  uint8_t *sB = sA + NA * 16384;       // WD_NBU x SBU
  uint32_t *sQ = reinterpret_cast<uint32_t *>(sB + WD_NBU * SBU);  // [WD_PD][WD_CW] sign-word ring
  __shared__ __align__(8) uint64_t bbar[WD_NBU];
  __shared__ __align__(8) uint64_t afull[NA], dfull[NA], dfree[NA];
  __shared__ uint32_t tbase;
  __shared__ int abort_flag;
  __shared__ int ec[2][KP];
  __shared__ int2 rtab[WD_CW / 32][KQ];  // per warp: (add, shift) of the group being rounded
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool cw = tid < WD_CW;
  const int row = tid & 127, qd = (tid >> 7) & 3;
  // CTA = (tile, token split): tokens t0 .. t0+KP of the batch's KPR
  const int tile = (int)blockIdx.x / p.uts, t0 = ((int)blockIdx.x - tile * p.uts) * KP;
  const int NR = 2 * p.KP;  // rows of the records' operand images
  int pi = 0;
  while (pi + 1 < p.nproj && tile >= p.up[pi + 1].tile0) ++pi;
  const WUProj &pj = p.up[pi];
  const int n = (tile - pj.tile0) * 128 + row;
  const bool nvalid = cw && n < pj.out;
  const int k = p.k - t0;  // valid tokens from t0 on (may exceed KP)
  const int ng0 = pj.ng[0], ngt = pj.ng[0] + (pj.nbr > 1 ? pj.ng[1] : 0);
  volatile int *abrt = &abort_flag;
  LBX_PROBE(50);

  if (tid == 0) {
    for (int j = 0; j < WD_NBU; ++j) mbar_init(&bbar[j], 1);
    for (int j = 0; j < NA; ++j) {
      mbar_init(&afull[j], WD_CW);
      mbar_init(&dfull[j], 1);
      mbar_init(&dfree[j], WD_CW);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 16) tmem_alloc(&tbase, NA * N);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;

  // this thread's sign word of group G (word 4g + quarter of its row) into
  // ring slot G % WD_PD (one commit group per group)
  auto load_bits = [&](int G) {
    const int b = G < ng0 ? 0 : 1, g = b ? G - ng0 : G;
    const int w0 = 4 * g + qd, W = pj.words[b];
    const bool v = G < ngt && nvalid && w0 < W;
    cpa4(&sQ[(G % WD_PD) * WD_CW + tid], v ? pj.u_sign[b] + (int64_t)n * W + w0 : pj.u_sign[0], v ? 4u : 0u);
    cpa_commit();
  };
  if (cw) {
#pragma unroll
    for (int j = 0; j + 1 < WD_PD; ++j) load_bits(j);
  }
  LBX_PROBE(51);
  pdl_trigger();
  pdl_wait();  // U records come from the V grid
  // per (branch, token) the coarsest group exponent
  if (tid < 2 * KP) {
    const int b = tid / KP, t = tid - b * KP;
    int e = UE_NONE;
    if (t < k && b < pj.nbr) {
      const int ng = pj.ng[b];
      for (int g = 0; g < ng; ++g)
        e = min(e, __ldcg(reinterpret_cast<const int *>(pj.urec[b] + (size_t)g * p.urec_bytes + (size_t)NR * 128) +
                          t0 + t));
    }
    ec[b][t] = e == UE_NONE ? 0 : e;
  }
  __syncthreads();
  LBX_PROBE(52);

  int I0[KQ], I1[KQ];
#pragma unroll
  for (int i = 0; i < KQ; ++i) I0[i] = I1[i] = 0;

  if (warp == 16) {
    // ---- issuing warp (lane 0 acts, the warp stays converged)
    int nissued = 0, ncommit = 0;
    auto issue_b = [&](int G) {
      if (lane == 0) {
        const int buf = G % WD_NBU;
        const int b = G < ng0 ? 0 : 1, g = b ? G - ng0 : G;
        // this CTA's rows of the image (whole 8-row swizzle atoms), then its tokens' exponents
        const uint8_t *rec = pj.urec[b] + (size_t)g * p.urec_bytes;
        mbar_arrive_expect_tx(&bbar[buf], (uint32_t)(N * 128 + KP * 4));
        bulk_g2s(sB + buf * SBU, rec + (size_t)2 * t0 * 128, N * 128u, &bbar[buf]);
        bulk_g2s(sB + buf * SBU + N * 128, rec + (size_t)NR * 128 + (size_t)t0 * 4, KP * 4u, &bbar[buf]);
      }
      ++nissued;
    };
    for (int j = 0; j < WD_NBU && j < ngt; ++j) issue_b(j);
    for (int G = 0; G < ngt; ++G) {
      const int a = G % NA;
      if (G >= NA) {  // TMEM buffer a and the B buffer of group G-NA are free again
        if (!__all_sync(0xffffffffu, wd_wait(&dfree[a], (uint32_t)((G - NA) / NA) & 1u, 0x716, abrt))) break;
        if (G - NA + WD_NBU < ngt) issue_b(G - NA + WD_NBU);
      }
      if (!__all_sync(0xffffffffu, wd_wait(&afull[a], (uint32_t)(G / NA) & 1u, 0x717, abrt))) break;
      if (!__all_sync(0xffffffffu, wd_wait(&bbar[G % WD_NBU], (uint32_t)(G / WD_NBU) & 1u, 0x711, abrt))) break;
      __syncwarp();
      tc_fence_after();
      if (lane == 0) {
        const uint32_t aB = smem_u32(sA + a * 16384), bB = smem_u32(sB + (G % WD_NBU) * SBU);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_i8(tmem + (uint32_t)(a * N), sw128_desc(aB + 32 * s), sw128_desc(bB + 32 * s), IDESC,
                  s > 0 ? 1u : 0u);
        umma_commit(&dfull[a]);
      }
      ++ncommit;
      __syncwarp();
    }
    if (*abrt && lane == 0) {  // work in flight ends before shared memory and TMEM are released
      for (int j = ncommit; j < nissued; ++j) mbar_poll_cta(&bbar[j % WD_NBU], (uint32_t)(j / WD_NBU) & 1u, 0x714);
      if (ncommit > 0) mbar_poll_cta(&dfull[(ncommit - 1) % NA], (uint32_t)((ncommit - 1) / NA) & 1u, 0x715);
    }
    __syncwarp();
  } else {
    // ---- expanding / reading warps
    auto epilogue = [&](int G) {
      bool okw = wd_wait(&dfull[G % NA], (uint32_t)(G / NA) & 1u, 0x712, abrt) &&
                 wd_wait(&bbar[G % WD_NBU], (uint32_t)(G / WD_NBU) & 1u, 0x713, abrt);
      okw = __all_sync(0xffffffffu, okw);
      tc_fence_after();
      if (!okw) return false;
      const int b = G < ng0 ? 0 : 1;
      // the rounding of this group for the warp's tokens: rshr(v, e - ec) as
      // (v + add) >> shift (shift 31 with add 2^30 gives 0 for every |v| < 2^30;
      // an all-zero group has v = 0)
      if (lane < KQ) {
        const int t = qd * KQ + lane;
        const int ex = reinterpret_cast<const int *>(sB + (G % WD_NBU) * SBU + N * 128)[t];
        const int s = ex == UE_NONE ? 0 : min(ex - ec[b][t], 31);
        rtab[warp][lane] = make_int2(s > 0 ? 1 << (s - 1) : 0, s);
      }
      uint32_t r[2 * KQ];
      tmem_ld_cols<2 * KQ>(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)((G % NA) * N + qd * 2 * KQ), r);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive1(&dfree[G % NA]);
      __syncwarp();
      if (b) {
#pragma unroll
        for (int i = 0; i < KQ; ++i) {
          const int2 as = rtab[warp][i];
          I1[i] += (256 * (int)r[2 * i] + (int)r[2 * i + 1] + as.x) >> as.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < KQ; ++i) {
          const int2 as = rtab[warp][i];
          I0[i] += (256 * (int)r[2 * i] + (int)r[2 * i + 1] + as.x) >> as.y;
        }
      }
      __syncwarp();  // (rtab is rewritten by the next group)
      return true;
    };
    for (int G = 0; G < ngt; ++G) {
      if (G == 20) LBX_PROBE(55);
      load_bits(G + WD_PD - 1);
      cpa_wait<WD_PD - 1>();  // group G's words have landed
      // A buffer G % NA is free once the MMAs of group G-NA completed
      if (G >= NA && !__all_sync(0xffffffffu, wd_wait(&dfull[G % NA], (uint32_t)((G - NA) / NA) & 1u, 0x718, abrt)))
        break;
      if (G == 20) LBX_PROBE(56);
      {
        uint8_t *a = sA + (G % NA) * 16384;
        uint4 e0, e1;
        wd_expand(sQ[(G % WD_PD) * WD_CW + tid], e0, e1);
        *reinterpret_cast<uint4 *>(a + sw128_off(row, 32 * qd)) = e0;
        *reinterpret_cast<uint4 *>(a + sw128_off(row, 32 * qd + 16)) = e1;
      }
      fence_proxy_async();
      mbar_arrive1(&afull[G % NA]);
      if (G == 20) LBX_PROBE(57);
      if (G >= D && !epilogue(G - D)) break;
      if (G == 20) LBX_PROBE(59);
    }
    for (int j = ngt > D ? ngt - D : 0; j < ngt && !*abrt; ++j)
      if (!epilogue(j)) break;
    cpa_wait<0>();
  }
  LBX_PROBE(53);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool ok = !*abrt;
  if (warp == 16) tmem_dealloc(tmem, NA * N);
  if (!ok || !nvalid) return;

  const float u1a = pj.u1[0][n];
  const float u1b = pj.nbr > 1 ? pj.u1[1][n] : 0.f;
  const float bias = pj.bias ? pj.bias[n] : 0.f;
#pragma unroll
  for (int i = 0; i < KQ; ++i) {
    const int t = qd * KQ + i;
    if (t >= k) break;
    float v = u_result(u1a, I0[i], ec[0][t], pj.nbr > 1, u1b, I1[i], ec[1][t], pj.bias != nullptr, bias);
    if (p.epi == LBX_EPI_SILU0 && pi == 0) v = v / (1.0f + expf(-v));
    const int64_t off = (int64_t)(t0 + t) * pj.y_ld + n;
    if (p.ydt == LBX_F32) {
      float *y = reinterpret_cast<float *>(pj.y) + off;
      if (p.epi == LBX_EPI_ADD) v += *y;
      *y = v;
    } else {
      reinterpret_cast<uint16_t *>(pj.y)[off] = f32_to_bf16(v);
    }
  }
  LBX_PROBE(54);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int wide_kp(int k) { return k <= 8 ? 8 : k <= 16 ? 16 : k <= 32 ? 32 : 64; }
static int wide_rec_bytes(int KP) { return (2 * KP * 256 + KP * 4 + 15) & ~15; }
static int wide_urec_bytes(int KP) { return (2 * KP * 128 + KP * 4 + 15) & ~15; }
static size_t wv_smem(int KP) {
  return 1024 + 2 * 32768 + (size_t)WD_NBV * (2 * KP * 256 + 1024) + (size_t)WD_PD * WD_CW * 8;
}
static size_t wu_smem(int KP) {
  return 1024 + (size_t)WD_NAU * 16384 + (size_t)WD_NBU * (((2 * KP * 128 + KP * 4) + 1023) & ~1023) +
         (size_t)WD_PD * WD_CW * 4;
}

// scratch of one tensor-core batch of k tokens (0: the call does not fit it)
static size_t wide_ws_bytes(const lbx_proj *projs, int n_proj, int k) {
  if (k < 1) return 0;
  const int KP = wide_kp(std::min(k, WD_MAXK));
  const int K = projs[0].in_features;
  const int nblk = (K + 255) / 256;
  if (nblk > WD_MAXBLK) return 0;
  size_t tot = 0;
  for (int i = 0; i < n_proj; ++i)
    for (int b = 0; b < projs[i].n_branches; ++b) {
      const lbx_branch &br = projs[i].br[b];
      if (br.v_sign) tot += al256((size_t)nblk * wide_rec_bytes(KP)) + al256((size_t)KP * 4);
      tot += al256((size_t)u_groups(br.rank) * wide_urec_bytes(KP));
    }
  return tot;
}

template <int KPS>
static int wv_launch(const WParams &wp, int vtiles, bool pdl, cudaStream_t stream) {
  static DevCache<int> attr;
  int dummy = 0;
  const int rc = attr.get(dummy, [](int &) {
    return cuda_status(cudaFuncSetAttribute(wv_kernel<KPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)wv_smem(KPS)),
                       "tensor-core V-stage attribute");
  });
  if (rc) return rc;
  return cuda_status(launch(wv_kernel<KPS>, dim3(vtiles * wp.vts), dim3(WD_TPB), wv_smem(KPS), stream, pdl, wp),
                     "tensor-core V-stage launch");
}
template <int KPS>
static int wu_launch(const WParams &wp, int utiles, bool pdl, cudaStream_t stream) {
  static DevCache<int> attr;
  int dummy = 0;
  const int rc = attr.get(dummy, [](int &) {
    return cuda_status(cudaFuncSetAttribute(wu_kernel<KPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)wu_smem(KPS)),
                       "tensor-core U-stage attribute");
  });
  if (rc) return rc;
  return cuda_status(launch(wu_kernel<KPS>, dim3(utiles * wp.uts), dim3(WD_TPB), wu_smem(KPS), stream, pdl, wp),
                     "tensor-core U-stage launch");
}

// Token splits of a grid of `tiles` CTAs: while the grid would fill at most
// half of the SMs, each tile's tokens are split over twice as many CTAs (at
// least 8 tokens each, the last split holding tokens).  Every token's
// arithmetic is the same in any split.  Measured on the 70B down projection
// at 64 tokens (50 V tiles, 64 U tiles): see the design notes.
static int wide_split(int tiles, int KPR, int k) {
  const int sms = device_sm_count();
  int ts = 1;
  while (ts < 8 && KPR / (2 * ts) >= 8 && tiles * ts * 2 <= sms && (2 * ts - 1) * (KPR / (2 * ts)) < k) ts *= 2;
  return ts;
}

// one batch of k <= WD_MAXK tokens starting at token tok0
static int wide_batch(const lbx_proj *projs, const lbx_linear_args *a, int tok0, int k, void *ws,
                      cudaStream_t stream) {
  const int n_proj = a->n_proj;
  const int KP = wide_kp(k);
  const int K = projs[0].in_features;
  const int esz_x = a->x_dtype == LBX_F32 ? 4 : 2;
  const int esz_y = a->y_dtype == LBX_F32 ? 4 : 2;
  WParams wp = {};
  wp.K = K;
  wp.Wv = K / 32;
  wp.nblk = (K + 255) / 256;
  wp.k = k;
  wp.KP = KP;
  wp.xdt = a->x_dtype;
  wp.prologue = a->prologue;
  wp.ydt = a->y_dtype;
  wp.epi = a->epilogue;
  wp.eps = a->eps;
  wp.x = reinterpret_cast<const uint8_t *>(a->x) + (size_t)tok0 * K * esz_x;
  wp.x2 = a->x2 ? reinterpret_cast<const uint8_t *>(a->x2) + (size_t)tok0 * K * esz_x : nullptr;
  wp.norm_w = a->norm_w;
  wp.rec_bytes = wide_rec_bytes(KP);
  wp.urec_bytes = wide_urec_bytes(KP);
  uint8_t *w = reinterpret_cast<uint8_t *>(ws);
  uint8_t *urec[LBX_MAX_PROJ][2] = {};
  int vtiles = 0, utiles = 0;
  for (int i = 0; i < n_proj; ++i) {
    const lbx_proj &pr = projs[i];
    for (int b = 0; b < pr.n_branches; ++b) {
      urec[i][b] = w;
      w += al256((size_t)u_groups(pr.br[b].rank) * wp.urec_bytes);
    }
    for (int b = 0; b < pr.n_branches; ++b) {
      const lbx_branch &br = pr.br[b];
      if (!br.v_sign) continue;
      WSeg &sg = wp.seg[wp.nseg++];
      sg.v_sign = br.v_sign;
      sg.v2 = br.v2;
      sg.mid0 = br.mid;
      sg.rank = br.rank;
      sg.tile0 = vtiles;
      vtiles += (br.rank + 127) / 128;
      sg.xrec = w;
      w += al256((size_t)wp.nblk * wp.rec_bytes);
      sg.rs = reinterpret_cast<float *>(w);
      w += al256((size_t)KP * 4);
      sg.urec0 = urec[i][b];
      if (b == 0 && pr.n_branches == 2 && !pr.br[1].v_sign) {
        sg.mid1 = pr.br[1].mid;
        sg.urec1 = urec[i][1];
      }
    }
    WUProj &uj = wp.up[i];
    uj.nbr = pr.n_branches;
    uj.out = pr.out_features;
    uj.bias = pr.bias;
    uj.y_ld = a->y_ld[i] ? a->y_ld[i] : pr.out_features;
    uj.y = reinterpret_cast<uint8_t *>(a->y[i]) + (size_t)tok0 * uj.y_ld * esz_y;
    for (int b = 0; b < pr.n_branches; ++b) {
      uj.u_sign[b] = pr.br[b].u_sign;
      uj.u1[b] = pr.br[b].u1;
      uj.urec[b] = urec[i][b];
      uj.words[b] = (pr.br[b].rank + 31) / 32;
      uj.ng[b] = u_groups(pr.br[b].rank);
    }
    uj.tile0 = utiles;
    utiles += (pr.out_features + 127) / 128;
  }
  wp.nproj = n_proj;
  const bool pdl = a->use_pdl != 0;
  wp.vts = wide_split(vtiles, KP, k);
  wp.uts = wide_split(utiles, KP, k);
  cudaError_t e = launch(wx_stage_kernel, dim3(wp.k, wp.nseg), dim3(WX_THREADS), 0, stream, pdl, wp);
  if (e != cudaSuccess) return cuda_status(e, "x staging launch");
  int rc;
  switch (KP / wp.vts) {
    case 8: rc = wv_launch<8>(wp, vtiles, pdl, stream); break;
    case 16: rc = wv_launch<16>(wp, vtiles, pdl, stream); break;
    case 32: rc = wv_launch<32>(wp, vtiles, pdl, stream); break;
    default: rc = wv_launch<64>(wp, vtiles, pdl, stream); break;
  }
  if (rc) return rc;
  switch (KP / wp.uts) {
    case 8: return wu_launch<8>(wp, utiles, pdl, stream);
    case 16: return wu_launch<16>(wp, utiles, pdl, stream);
    case 32: return wu_launch<32>(wp, utiles, pdl, stream);
    default: return wu_launch<64>(wp, utiles, pdl, stream);
  }
}

#ifndef LBX_WIDE_MIN_TOKENS
#define LBX_WIDE_MIN_TOKENS 32  // the tensor-core executor from this many tokens on every call
#endif
#ifndef LBX_WIDE_BIG_TOKENS
#define LBX_WIDE_BIG_TOKENS 16  // ... and from this many on calls of at least LBX_WIDE_BIG_WORK
#endif
#ifndef LBX_WIDE_BIG_WORK
#define LBX_WIDE_BIG_WORK 25000000.0  // sum over projections of (in + out features) x (sum of ranks)
#endif
// Whether AUTO / KERNELS run a call of n_tokens on the tensor-core executor.
// Its cost is nearly flat up to 32 tokens (one pass over the weights per
// batch of 64), the stage grids' grows with every 16 tokens; measured on
// B200 the executor wins from 32 tokens on every shape and from 16 on the
// 7B- and 70B-class calls (7B q/k/v 74.4 -> 41.6 us, 7B down 120.0 -> 75.2,
// 70B o 88.1 -> 70.3, 70B gate/up 415 -> 219), while a single C2-sized
// projection (4096 + 4096 features x 2048 ranks) stays faster on the stage
// grids at 16 (38.1 vs 40.5 us).
static bool wide_auto(const lbx_proj *projs, int n_proj, int n_tokens) {
  if (!projs || n_proj < 1 || n_proj > LBX_MAX_PROJ) return false;
  if (n_tokens >= LBX_WIDE_MIN_TOKENS) return true;
  if (n_tokens < LBX_WIDE_BIG_TOKENS) return false;
  double work = 0;
  for (int i = 0; i < n_proj; ++i) {
    int r = 0;
    for (int b = 0; b < projs[i].n_branches && b < 2; ++b) r += projs[i].br[b].rank;
    work += (double)(projs[i].in_features + projs[i].out_features) * r;
  }
  return work >= LBX_WIDE_BIG_WORK;
}

// The tensor-core executor for this call, if it applies: LBX_EXEC_TC always
// (LBX_EUNSUPPORTED when it cannot run the call); LBX_EXEC_AUTO / _KERNELS
// when wide_auto selects it and the workspace holds a batch.  *handled tells
// whether the call ran (or failed) here.
static int wide_try(const lbx_proj *projs, const lbx_linear_args *a, void *ws, size_t ws_bytes,
                    cudaStream_t stream, bool &handled) {
  handled = false;
  const bool forced = a->exec == LBX_EXEC_TC;
  if (!forced && !((a->exec == LBX_EXEC_AUTO || a->exec == LBX_EXEC_KERNELS) &&
                   wide_auto(projs, a->n_proj, a->n_tokens)))
    return LBX_OK;
  const size_t need = wide_ws_bytes(projs, a->n_proj, a->n_tokens);
  if (need == 0 || ws_bytes < need) {
    if (!forced) return LBX_OK;
    handled = true;
    LBX_CHECK_SUP(need != 0, "in_features above %d for the tensor-core executor", WD_MAXBLK * 256);
    LBX_CHECK_ARG(false, "workspace too small for the tensor-core executor (%zu < %zu)", ws_bytes, need);
  }
  handled = true;
  for (int t0 = 0; t0 < a->n_tokens; t0 += WD_MAXK) {
    const int k = std::min(WD_MAXK, a->n_tokens - t0);
    const int rc = wide_batch(projs, a, t0, k, ws, stream);
    if (rc) return rc;
  }
  return LBX_OK;
}

}  // namespace lbx
