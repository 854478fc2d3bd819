// Fused layer chain: the U-stage of layer i and the V-stage of layer i+1 in
// one launch.
//
// A chain of single-projection LittleBit layers, x_{i+1} = layer_i(x_i)
// (quantization/modules/littlebit.py:95-121 per layer), runs as n + 1 launches
// instead of 2n: a head launch computes layer 0's V-stage partials, then launch
// i computes layer i's U-stage and, from its own outputs, layer i+1's V-stage
// partials.  The grid is one thread-block cluster of FC_CS CTAs per 256 output
// rows.
//
//  * Placement.  A launch must not put two of its CTAs on one SM: the CTAs of
//    a cluster wait for one another, so the slowest one paces the layer.  At
//    one CTA per SM a B200 holds 15 clusters of 8 but 22 of 6, so a 4096-row
//    layer (16 clusters) takes clusters of 6.  The launches of a chain
//    alternate between two builds of the kernel: FC_SMEM_SIDE (48 registers,
//    shared memory padded past half an SM) and FC_REG_SIDE (72 registers, the
//    shared memory it needs).  Two of either do not fit on one SM, one of each
//    does (with the shared-memory carveout at its maximum), so the next
//    launch's CTAs are placed under PDL beside the running ones, one per SM.
//
//  * V partials.  The V-stage quantises a = v2 ⊙ x with one scale per token
//    per 256-column block and sums the blocks' exact integer products in block
//    order (linear.cu, vstage_run).  Cluster c owns output rows [256c, 256c+256)
//    of layer i, which are exactly block c of layer i+1's input, so it can form
//    block c's product for every rank of layer i+1 as soon as its rows exist:
//    P[c][t][r] = float(Σ_{j in block c} s_rj q_j) · (absmax / QMAX).  The CTAs
//    of the cluster split the ranks (16-rank tiles).
//  * z.  Launch i+1 adds the blocks' partials of its ranks in the V-stage's
//    order (for each of the 16 block positions of a 4096-column pass, the passes
//    in order, then the positions in order) and multiplies by mid: the V-stage's
//    own float operations on the same values, so z has the same bits.
//  * U.  Every CTA of a cluster owns some of the layer's 128-rank quantisation
//    groups.  It derives each group's power-of-two exponent from the group's max
//    |z| (as the U-stage does), quantises its groups and contracts them with the
//    cluster's 256 U rows into exact int32 sums.  The sums and the exponents go
//    to every CTA of the cluster over distributed shared memory; after one
//    cluster barrier each CTA rounds every group to its branch's coarsest
//    exponent with the U-stage's integer shift and forms y for all 256 rows with
//    the U-stage's epilogue expression (u_result).  Exact integers add the same
//    in any order, so y has the bits of the two stage grids.
//  * Each CTA stores its share of the 256 rows of y and quantises the
//    cluster's 256 values (one block of layer i+1's input) for the next
//    partials.
//
// Per layer this is one grid boundary and one cluster barrier, against two grid
// boundaries for the stage grids.  Weights are copied into shared memory from a
// prepared blob (lbx_chain_prepare) in which every CTA's share of U and V is
// contiguous; the copies are issued before griddepcontrol.wait.

#include <vector>

namespace lbx {

constexpr int FC_CS = 6;          // CTAs per cluster
constexpr int FC_ROWS = 256;      // output rows per cluster (= one 256-column V block of the next layer)
constexpr int FC_GMAX = 5;        // 128-rank groups per CTA (FC_GTOT <= 32: one warp reduces over them)
constexpr int FC_GTOT = FC_CS * FC_GMAX;
constexpr int FC_MAXK = 4;        // tokens per launch (one MMA column block)
constexpr int FC_NBLK = 32;       // 256-column input blocks of a layer (in_features <= 8192)
constexpr int FC_THREADS = 512;
constexpr int FC_VPITCH = 8;      // words per V row in the blob (rows 4-7 and 12-15 of a tile hold their
                                  // two 4-word halves swapped: conflict-free fragment loads, no padding)
constexpr int FC_UGW = FC_ROWS * 4;     // words of one U group slot (256 rows x 4 words)
constexpr int FC_VTW = 16 * FC_VPITCH;  // words of one V tile (16 ranks x 8 words)
constexpr int FC_VTC = 40;              // V tiles per CTA at most
constexpr int FC_SMEM_SIDE = 48;        // register caps of the two builds of the kernel
constexpr int FC_REG_SIDE = 72;
constexpr int FC_SMEM_PAD = 118 * 1024;  // shared memory of an FC_SMEM_SIDE CTA at least (> half an SM)

struct FcGroup {  // one 128-rank quantisation group of a branch (U side)
  int b;          // branch
  int n;          // ranks in the group (<= 128)
  int r0;         // first rank within the branch
  int pidx;       // its first rank in the partial rank space
};

struct FcParams {
  // U side of layer i (absent in the head launch)
  const uint32_t *ublob;  // [N/256][ng][256 rows][4 words]
  const float *u1[2];
  const float *mid[2];
  const float *bias;
  const float *pin;       // partials of layer i: [nblk_in][k][pin_cols]
  void *y;                // [k][N]
  FcGroup g[FC_GTOT];     // groups in slot order (the CTAs' shares contiguous)
  int gstart[FC_CS + 1];
  int ng, nbr, pin_cols, nblk_in;
  // V side of layer i+1 (absent in the last launch)
  const uint32_t *vblob;  // [N/256][nvt][16 ranks][FC_VPITCH words]
  const float *v2[2];     // [N] input scale of each V segment of layer i+1 (branch 0; branch 1
                          // when it has its own V): every segment stages its own a = v2 * x
  float *pout;            // [N/256][k][pout_cols]
  // V tiles: 16 ranks each, segment 0's ranks then segment 1's (partial rank
  // space); CTA j of a cluster takes tiles [nvt*j/8, nvt*(j+1)/8)
  int nvt, vt0;           // tiles in all, tiles of segment 0
  int vr[2], vpb[2];      // ranks and first partial rank of each segment
  int nvseg, pout_cols;
  // head launch: layer 0's input
  const void *x;          // [k][N]
  int k, adt, N;          // tokens, activation dtype, features of the rows this launch owns
  int has_u, has_v;
};

// shared-memory layout of one CTA (bytes; weights first, then scratch)
struct FcSmem {
  int uw, vw, mid, u1, bias, v2, wbytes;      // weight region
  int actu, xs, stg, ex, sa, actv, total;     // scratch
};

__host__ __device__ inline FcSmem fc_smem(int k, int ng) {
  FcSmem L;
  const int ws = act_ws(2 * k);
  int o = 0;
  L.uw = o;   o += FC_GMAX * FC_UGW * 4;
  L.vw = o;   o += FC_VTC * FC_VTW * 4;
  L.mid = o;  o += FC_GMAX * 128 * 4;
  L.u1 = o;   o += 2 * FC_ROWS * 4;
  L.bias = o; o += FC_ROWS * 4;
  L.v2 = o;   o += 2 * FC_ROWS * 4;
  L.wbytes = o;
  L.actu = o; o += FC_GMAX * 4 * ws * 4;
  L.xs = o;   o += (ng ? FC_CS : 0) * FC_ROWS * k * 8;
  L.stg = o;  o += (ng && k > 1 ? 1 : 0) * FC_ROWS * k * 8;  // the bulk build's staging buffer
  L.ex = o;   o += ((ng * k * 4 + 15) / 16) * 16;
  L.sa = o;   o += 2 * k * FC_ROWS * 4;
  L.actv = o; o += 2 * 8 * ws * 4;
  L.total = o;
  return L;
}

// barrier 1 + q (q = 0..3) of the 128 threads of warps 4q..4q+3 (constant
// barrier ids, so that the kernel reserves five barriers, not sixteen)
LBX_DEV void quad_barrier(int q) {
  switch (q) {
    case 0: asm volatile("bar.sync 1, 128;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 2, 128;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 3, 128;" ::: "memory"); break;
    default: asm volatile("bar.sync 4, 128;" ::: "memory"); break;
  }
}

// shared::cluster address of `p` (this CTA's shared memory) in CTA `rank` of the cluster
LBX_DEV uint32_t cl_addr(const void *p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// asynchronous stores into a cluster CTA's shared memory, each counted (in
// bytes) on that CTA's mbarrier
LBX_DEV void st_async_b32(uint32_t addr, int v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr), "r"(v),
               "r"(bar)
               : "memory");
}
LBX_DEV void st_async_v4(uint32_t addr, int a, int b, int c, int d, uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
      "r"(a), "r"(b), "r"(c), "r"(d), "r"(bar)
      : "memory");
}
// bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// this CTA's shared memory into a cluster CTA's, counted on that CTA's mbarrier
LBX_DEV void bulk_s2cl(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar)
               : "memory");
}
// bounded wait on a phase of an mbarrier that other CTAs of the cluster
// complete (acquire at cluster scope), polled with test_wait: the data is
// usually in flight already, and a suspending try_wait may sleep past its
// arrival.  False, with `code` in the device error word, after 1 s.
LBX_DEV bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int code) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 1023u) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (it == 0) t0 = t;
      else if (t - t0 > 1000000000ull) break;
    }
  }
  atomicCAS(&g_lbx_device_error, 0, code);
  return false;
}

// the same for an mbarrier completed by this CTA's own bulk copies
LBX_DEV bool mbar_poll_cta(uint64_t *bar, uint32_t parity, int code) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 1023u) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (it == 0) t0 = t;
      else if (t - t0 > 1000000000ull) break;
    }
  }
  atomicCAS(&g_lbx_device_error, 0, code);
  return false;
}

LBX_DEV void fc_vpart(const FcParams &p, int c, int k, int ws, int vs, int ve, const uint32_t *vw,
                      const uint32_t *actv, const int *vmax, const int *vsq, int lane);

// MAXR: the register cap of the build.  BULK: the sums exchange goes by bulk
// copies (the build for 2-4 tokens) rather than 16-byte st.async stores (the
// one-token builds).  They are separate builds so that the one-token kernels
// keep their own code: with the bulk path compiled in beside it, a one-token
// chain measured 8.1 us per C2 layer against 7.5.
template <int MAXR, bool BULK>
__global__ void __launch_bounds__(FC_THREADS, 1) __maxnreg__(MAXR) fc_kernel(const __grid_constant__ FcParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ __align__(8) uint64_t xbar[2];  // exponents, then the CTAs' rounded sums (filled by st.async)
  __shared__ int s_gmax[FC_GMAX][FC_MAXK];
  __shared__ int s_usq[FC_GMAX][FC_MAXK];
  __shared__ int s_gexp[FC_GMAX][FC_MAXK];  // exponent of each of this CTA's groups
  __shared__ int s_ec[2][FC_MAXK];
  __shared__ int s_gb[FC_GTOT];  // branch of each group (slot order)
  __shared__ int s_vmax[2 * FC_MAXK], s_vsq[2 * FC_MAXK];  // per (V segment, token)
  __shared__ int s_ok;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j = cl_rank();
  const int c = blockIdx.x / FC_CS;
  const int k = p.k;
  const int ncols = 2 * k;
  const int ws = act_ws(ncols);
  const FcSmem L = fc_smem(k, p.ng);
  uint32_t *uw = reinterpret_cast<uint32_t *>(smem + L.uw);
  uint32_t *vw = reinterpret_cast<uint32_t *>(smem + L.vw);
  float *smid = reinterpret_cast<float *>(smem + L.mid);
  float *su1 = reinterpret_cast<float *>(smem + L.u1);
  float *sbias = reinterpret_cast<float *>(smem + L.bias);
  float *sv2 = reinterpret_cast<float *>(smem + L.v2);
  uint32_t *actu = reinterpret_cast<uint32_t *>(smem + L.actu);  // [slot][4 words][ws]
  int *xs = reinterpret_cast<int *>(smem + L.xs);            // [cta][row pair][t][4] rounded sums
  int *stg = reinterpret_cast<int *>(smem + L.stg);          // (bulk build) this CTA's sums, [row pair][t][4]
  int *ex = reinterpret_cast<int *>(smem + L.ex);            // [group][t] exponents
  float *sa = reinterpret_cast<float *>(smem + L.sa);        // [seg][t][256] a = v2 * x of the block
  uint32_t *actv = reinterpret_cast<uint32_t *>(smem + L.actv);  // [segment][8 words][ws]

  LBX_PROBE(20);
  const int gs = p.gstart[j], myg = p.has_u ? p.gstart[j + 1] - gs : 0;
  const int vs = p.nvt * j / FC_CS, ve = p.has_v ? p.nvt * (j + 1) / FC_CS : vs;
  if (tid == 0) {
    mbar_init(&bar, 1);
    if (p.has_u) {
      mbar_init(&xbar[0], 1);
      mbar_init(&xbar[1], 1);
    }
    fence_mbar_init();
    if (p.has_u) {  // the bytes every CTA of the cluster will store here
      mbar_arrive_expect_tx(&xbar[0], (uint32_t)p.ng * k * 4u);
      mbar_arrive_expect_tx(&xbar[1], (uint32_t)FC_CS * FC_ROWS * k * 8u);
    }
  }
  if (tid < FC_GMAX * FC_MAXK) {
    (&s_gmax[0][0])[tid] = 0;
    (&s_usq[0][0])[tid] = 0;
  }
  if (tid < FC_GTOT) s_gb[tid] = tid < p.ng ? p.g[tid].b : 0;
  if (tid < 2 * FC_MAXK) s_vmax[tid] = s_vsq[tid] = 0;
  __syncthreads();
  // cluster barrier A: this CTA has started and set up its barriers, so the
  // others may store into its shared memory (they do so only after waiting on A)
  if (p.has_u) cl_arrive_relaxed();
  // ---- weights (independent of every activation): before the dependency wait
  if (tid == 0) {
    uint32_t bytes = 0;
    if (p.has_u) {
      bytes += (uint32_t)myg * FC_UGW * 4u + (uint32_t)p.nbr * FC_ROWS * 4u + (p.bias ? FC_ROWS * 4u : 0u);
      for (int s = 0; s < myg; ++s) bytes += (uint32_t)p.g[gs + s].n * 4u;
    }
    if (p.has_v) bytes += (uint32_t)(ve - vs) * FC_VTW * 4u + (uint32_t)p.nvseg * FC_ROWS * 4u;
    mbar_arrive_expect_tx(&bar, bytes);
  }
  __syncthreads();
  if (warp == 0 && p.has_u) {
    if (lane < myg) {
      const FcGroup G = p.g[gs + lane];
      bulk_g2s(uw + lane * FC_UGW, p.ublob + ((size_t)c * p.ng + gs + lane) * FC_UGW, FC_UGW * 4u, &bar);
      bulk_g2s(smid + lane * 128, p.mid[G.b] + G.r0, (uint32_t)G.n * 4u, &bar);
    } else if (lane == 8 || (lane == 9 && p.nbr > 1)) {
      bulk_g2s(su1 + (lane - 8) * FC_ROWS, p.u1[lane - 8] + (size_t)c * FC_ROWS, FC_ROWS * 4u, &bar);
    } else if (lane == 10 && p.bias) {
      bulk_g2s(sbias, p.bias + (size_t)c * FC_ROWS, FC_ROWS * 4u, &bar);
    }
  } else if (warp == 1 && p.has_v) {
    if (lane == 0 && ve > vs)  // this CTA's tiles are contiguous in the blob
      bulk_g2s(vw, p.vblob + ((size_t)c * p.nvt + vs) * FC_VTW, (uint32_t)(ve - vs) * FC_VTW * 4u, &bar);
    else if (lane == 8 || (lane == 9 && p.nvseg > 1))
      bulk_g2s(sv2 + (lane - 8) * FC_ROWS, p.v2[lane - 8] + (size_t)c * FC_ROWS, FC_ROWS * 4u, &bar);
  }
  pdl_trigger();
  pdl_wait();  // the previous launch's partials (and outputs) are complete
  LBX_PROBE(21);
  if (tid == 0) s_ok = mbar_poll_cta(&bar, 0, 0x131) ? 1 : 0;
  __syncthreads();
  const bool ok = s_ok != 0;
  LBX_PROBE(22);

  if (p.has_u) {
    cl_wait();  // barrier A: every CTA of the cluster has started (its barriers are set up)
    // ---- per (group, token), four warps: z of the group's 128 ranks (the
    // blocks' partials in the V-stage order: for each of the 16 block
    // positions of a 4096-column pass, 0 + the passes in order, then the
    // positions in order; a pass's 16 loads in flight together), the group
    // maximum, the exponent (to every CTA of the cluster) and the digits in
    // the U-stage's layout and rounding.  Warp wq holds word wq of the group:
    // lane (slot, e) the rank 32 wq + 16 (slot >> 2) + (slot & 3) + 4 e.
    const int nblk = p.nblk_in;
    const size_t bstride = (size_t)k * p.pin_cols;
    const int quad = warp >> 2, wq = warp & 3;
    const int slot = lane >> 2, e4 = lane & 3;
    const int pos = 32 * wq + 16 * (slot >> 2) + (slot & 3) + 4 * e4;
    for (int it0 = 0; it0 < myg * k; it0 += FC_THREADS / 128) {
      const int it = it0 + quad;  // (uniform per quad)
      if (it >= myg * k) break;
      const int sl = it / k, t = it - sl * k;
      const FcGroup G = p.g[gs + sl];
      float z = 0.f;
      if (pos < G.n) {
        const float *src = p.pin + (size_t)t * p.pin_cols + G.pidx + pos;
        float tw[16];
        {
          float pv[16];
#pragma unroll
          for (int w = 0; w < 16; ++w) pv[w] = w < nblk ? __ldcg(src + w * bstride) : 0.f;
#pragma unroll
          for (int w = 0; w < 16; ++w) tw[w] = 0.f + pv[w];
        }
        for (int b0 = 16; b0 < nblk; b0 += 16) {
          float pv[16];
#pragma unroll
          for (int w = 0; w < 16; ++w) pv[w] = b0 + w < nblk ? __ldcg(src + (b0 + w) * bstride) : 0.f;
#pragma unroll
          for (int w = 0; w < 16; ++w)
            if (b0 + w < nblk) tw[w] += pv[w];
        }
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 16; ++w) v += tw[w];
        z = smid[sl * 128 + pos] * v;
      }
      const float m = warp_max(fabsf(z));
      if (lane == 0) atomicMax(&s_gmax[sl][t], __float_as_int(m));
      quad_barrier(quad);  // the quad's four maxima are in
      const float gm = __int_as_float(s_gmax[sl][t]);
      const int e = gm > 0.f ? u_group_exp(gm) : UE_NONE;
      if (wq == 0) {
        if (lane < FC_CS) st_async_b32(cl_addr(ex + (gs + sl) * k + t, lane), e, cl_addr(&xbar[0], lane));
        if (lane == 0) s_gexp[sl][t] = e;
      }
      const float sc = e == UE_NONE ? 0.f : pow2f(e);
      const int qv = __float2int_rn(z * sc);
      int hi, lo;
      split_digits(qv, hi, lo);
      // the four digits of a slot word come from lanes (slot, 0..3)
      const int base = lane & ~3;
      const int h0 = __shfl_sync(0xffffffffu, hi, base), h1 = __shfl_sync(0xffffffffu, hi, base + 1);
      const int h2 = __shfl_sync(0xffffffffu, hi, base + 2), h3 = __shfl_sync(0xffffffffu, hi, base + 3);
      const int l0 = __shfl_sync(0xffffffffu, lo, base), l1 = __shfl_sync(0xffffffffu, lo, base + 1);
      const int l2 = __shfl_sync(0xffffffffu, lo, base + 2), l3 = __shfl_sync(0xffffffffu, lo, base + 3);
      if (e4 == 0) {
        uint32_t *aw = actu + (sl * 4 + wq) * ws + 2 * t;
        aw[slot * ncols] = pack4(h0, h1, h2, h3);
        aw[slot * ncols + 1] = pack4(l0, l1, l2, l3);
      }
      const int sq = __reduce_add_sync(0xffffffffu, qv);
      if (lane == 0) atomicAdd(&s_usq[sl][t], sq);
    }
    __syncthreads();
    LBX_PROBE(23);
    // ---- contraction: warp w = output rows 16w..16w+15 of the cluster, each
    // of this CTA's groups on its own (exact int32, kept in registers)
    const int g = lane >> 2, q = lane & 3;
    int va[FC_GMAX], vb[FC_GMAX];
#pragma unroll
    for (int sl = 0; sl < FC_GMAX; ++sl) {
      va[sl] = vb[sl] = 0;
      if (sl < myg) {
        int acc[1][4] = {{0, 0, 0, 0}};
        const int G0[1] = {0};
        const uint32_t *tile = uw + sl * FC_UGW + warp * 16 * 4;
        sign_mma1<1>(acc, tile + g * 4, tile + (g + 8) * 4, actu + sl * 4 * ws, ws, ncols, G0, lane);
        const int sq = q < k ? s_usq[sl][q] : 0;
        va[sl] = sq + 2 * (256 * acc[0][0] + acc[0][1]);
        vb[sl] = sq + 2 * (256 * acc[0][2] + acc[0][3]);
      }
    }
    LBX_PROBE(25);
    // ---- every group's exponent (from every CTA), then per branch and
    // token the coarsest one
    bool okx = mbar_wait_cluster(&xbar[0], 0, 0x132);
    if (warp == 0) {
      for (int t = 0; t < k; ++t) {
        const int e = lane < p.ng ? ex[lane * k + t] : UE_NONE;
        const int b = lane < p.ng ? s_gb[lane] : 0;
        const int e0 = __reduce_min_sync(0xffffffffu, b == 0 ? e : UE_NONE);
        const int e1 = __reduce_min_sync(0xffffffffu, b == 1 ? e : UE_NONE);
        if (lane == 0) {
          s_ec[0][t] = e0 == UE_NONE ? 0 : e0;
          s_ec[1][t] = e1 == UE_NONE ? 0 : e1;
        }
      }
    }
    okx = __syncthreads_and(okx);
    LBX_PROBE(26);
    // ---- this CTA's groups rounded to their branch's coarsest exponent (the
    // U-stage's integer shift) and added per branch, to every CTA
    int I[2][2] = {{0, 0}, {0, 0}};  // [row g / g+8][branch], token q
    if (q < k) {
#pragma unroll
      for (int sl = 0; sl < FC_GMAX; ++sl) {
        if (sl < myg) {
          const int e = s_gexp[sl][q];
          if (e != UE_NONE) {
            const int b = s_gb[gs + sl];
            const int sft = e - s_ec[b][q];
            const int ra = rshr(va[sl], sft), rb = rshr(vb[sl], sft);
            if (b) {
              I[0][1] += ra;
              I[1][1] += rb;
            } else {
              I[0][0] += ra;
              I[1][0] += rb;
            }
          }
        }
      }
    }
    if constexpr (!BULK) {
      // all four lanes of a row pair store: lane q sends every token's sums
      // (fetched from lane (g, t)) to the CTAs d = q, q + 4 of the cluster
      int A[FC_MAXK][4];
#pragma unroll
      for (int t = 0; t < FC_MAXK; ++t) {
        if (t < k) {  // (uniform)
          const int src = (lane & ~3) | t;
          A[t][0] = __shfl_sync(0xffffffffu, I[0][0], src);
          A[t][1] = __shfl_sync(0xffffffffu, I[0][1], src);
          A[t][2] = __shfl_sync(0xffffffffu, I[1][0], src);
          A[t][3] = __shfl_sync(0xffffffffu, I[1][1], src);
        }
      }
      // one 16-byte store per (destination, token): both rows of the lane's
      // row pair (warp * 16 + g and + 8), both branches; xs is laid out as
      // [source CTA][row pair][token][4]
      const int rp = warp * 8 + g;
#pragma unroll
      for (int dd = 0; dd < (FC_CS + 3) / 4; ++dd) {
        const int d = q + 4 * dd;
        if (d >= FC_CS) break;
        const uint32_t bar = cl_addr(&xbar[1], d);
#pragma unroll
        for (int t = 0; t < FC_MAXK; ++t)
          if (t < k)
            st_async_v4(cl_addr(xs + ((j * (FC_ROWS / 2) + rp) * k + t) * 4, d), A[t][0], A[t][1], A[t][2],
                        A[t][3], bar);
      }
      LBX_PROBE(24);
      // cluster barrier C (waited at the exit): no CTA leaves before every
      // CTA of the cluster has issued its stores into the others' shared
      // memory.  Relaxed: the stores a CTA receives are all counted on its
      // own barriers, which it waits for before it reaches the exit.
      cl_arrive_relaxed();
    } else {
      // the sums go into this CTA's staging buffer [row pair][token][4]
      // (lane (g, q) holds token q), then one bulk copy of the buffer into
      // every CTA of the cluster (xs [source CTA][row pair][token][4], counted
      // on the receiver's xbar[1]): six large copies instead of a 16-byte
      // store per (row pair, token, destination)
      if (q < k)
        *reinterpret_cast<int4 *>(stg + ((warp * 8 + g) * k + q) * 4) = make_int4(I[0][0], I[0][1], I[1][0], I[1][1]);
      fence_proxy_async();  // the staging writes, before the copies read them
      __syncthreads();
      if (tid < FC_CS)
        bulk_s2cl(cl_addr(xs + j * (FC_ROWS / 2) * k * 4, tid), stg, (uint32_t)FC_ROWS * k * 8u,
                  cl_addr(&xbar[1], tid));
      LBX_PROBE(24);
    }
    // ---- every CTA's sums, then y for all 256 rows
    okx = __syncthreads_and(mbar_wait_cluster(&xbar[1], 0, 0x133) && okx);
    // (bulk build) cluster barrier C, waited at the exit: every copy into this
    // CTA has landed, so a CTA that passes C has had its staging buffer read
    // and no copy still targets it
    if constexpr (BULK) cl_arrive_relaxed();
    LBX_PROBE(28);
    for (int it = tid; it < FC_ROWS * k; it += FC_THREADS) {
      const int t = it / FC_ROWS, r = it - t * FC_ROWS;
      const int rp = (r >> 4) * 8 + (r & 7), hf = (r >> 3) & 1;  // row pair, and which of its rows
      int I0 = 0, I1 = 0;
#pragma unroll
      for (int d = 0; d < FC_CS; ++d) {
        const int2 v = *reinterpret_cast<const int2 *>(xs + ((d * (FC_ROWS / 2) + rp) * k + t) * 4 + 2 * hf);
        I0 += v.x;
        I1 += v.y;
      }
      const int e0 = s_ec[0][t], e1 = s_ec[1][t];
      float v = u_result(su1[r], I0, e0, p.nbr > 1, su1[FC_ROWS + r], I1, e1, p.bias != nullptr, sbias[r]);
      if (!ok || !okx) v = __int_as_float(0x7fc00000);
      float xv = v;  // the next layer's input value: as stored
      const size_t off = (size_t)t * p.N + (size_t)c * FC_ROWS + r;
      if (p.adt == LBX_F32) {
        if (r * FC_CS / FC_ROWS == j) reinterpret_cast<float *>(p.y)[off] = v;
      } else {
        const uint16_t hb = f32_to_bf16(v);
        if (r * FC_CS / FC_ROWS == j) reinterpret_cast<uint16_t *>(p.y)[off] = hb;
        xv = bf16_to_f32(hb);
      }
      if (p.has_v)
        for (int sg = 0; sg < p.nvseg; ++sg) {  // the next layer's a = v2 * x and its block maximum
          const float a = xv * sv2[sg * FC_ROWS + r];
          sa[(sg * k + t) * FC_ROWS + r] = a;
          const float m = warp_max(fabsf(a));  // (a warp's 32 items share the token)
          if (lane == 0) atomicMax(&s_vmax[sg * k + t], __float_as_int(m));
        }
    }
  } else if (p.has_v) {
    // head launch: block c of layer 0's input
    for (int it = tid; it < FC_ROWS * k; it += FC_THREADS) {
      const int t = it / FC_ROWS, r = it - t * FC_ROWS;
      const float xx = load_act(p.x, p.adt, (int64_t)t * p.N + (int64_t)c * FC_ROWS + r);
      for (int sg = 0; sg < p.nvseg; ++sg) {
        const float a = xx * sv2[sg * FC_ROWS + r];
        sa[(sg * k + t) * FC_ROWS + r] = a;
        const float m = warp_max(fabsf(a));
        if (lane == 0) atomicMax(&s_vmax[sg * k + t], __float_as_int(m));
      }
    }
  }
  if (p.has_v) {
    __syncthreads();
    LBX_PROBE(27);
    // the block's digits, once per (segment, token, word, slot) item (the
    // block maxima were taken with a = v2 * x)
    for (int it = tid; it < p.nvseg * k * 64; it += FC_THREADS) {
      const int st = it >> 6, Wd = (it >> 3) & 7, slot = it & 7;
      const int sg = st / k, t = st - sg * k;
      const float m = __int_as_float(s_vmax[st]);
      const float sc = m > 0.f ? QMAX / m : 0.f;
      int hi[4], lo[4], sq = 0;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int pos = 32 * Wd + 16 * (slot >> 2) + (slot & 3) + 4 * q4;
        const int qv = __float2int_rn(sa[st * FC_ROWS + pos] * sc);
        sq += qv;
        split_digits(qv, hi[q4], lo[q4]);
      }
      uint32_t *aw = actv + (sg * 8 + Wd) * ws + 2 * t;
      aw[slot * ncols] = pack4(hi[0], hi[1], hi[2], hi[3]);
      aw[slot * ncols + 1] = pack4(lo[0], lo[1], lo[2], lo[3]);
      sq = __reduce_add_sync(0xffffffffu, sq);  // a warp's 32 items share (segment, token)
      if (lane == 0) atomicAdd(&s_vsq[st], sq);
    }
    __syncthreads();
    if (ok) fc_vpart(p, c, k, ws, vs, ve, vw, actv, s_vmax, s_vsq, lane);
  }
  LBX_PROBE(29);
  if (p.has_u) cl_wait();  // barrier C
}

// V-stage partials of the next layer for this CTA's rank groups, warp by warp:
// each warp quantises the block itself (its private copy of the digits), so
// the block maximum, the digits and the contraction need no CTA barrier
// V-stage partials of the next layer for this CTA's rank tiles, one tile per
// warp at a time, from the block's digits (actv [segment][8 words][ws], the
// per (segment, token) maxima and digit sums)
LBX_DEV void fc_vpart(const FcParams &p, int c, int k, int ws, int vs, int ve, const uint32_t *vw,
                      const uint32_t *actv, const int *vmax, const int *vsq, int lane) {
  const int warp = threadIdx.x >> 5, ncols = 2 * k;
  const int g = lane >> 2, q = lane & 3;
  for (int mt = vs + warp; mt < ve; mt += FC_THREADS / 32) {
    const int sg = mt < p.vt0 ? 0 : 1;
    const int r0 = 16 * (sg ? mt - p.vt0 : mt);   // first rank of the tile in its segment
    const int n = min(16, p.vr[sg] - r0);
    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    const int G01[2] = {0, 1};
    const uint32_t *tile = vw + (mt - vs) * FC_VTW;
    sign_mma1<2>(acc, tile + g * FC_VPITCH, tile + (g + 8) * FC_VPITCH, actv + sg * 8 * ws, ws, ncols, G01,
                 lane, (g & 4));
    if (q < k) {
      const int sq = vsq[sg * k + q];
      const float inv = __int_as_float(vmax[sg * k + q]) / QMAX;
      const int ia = sq + 2 * (256 * (acc[0][0] + acc[1][0]) + (acc[0][1] + acc[1][1]));
      const int ib = sq + 2 * (256 * (acc[0][2] + acc[1][2]) + (acc[0][3] + acc[1][3]));
      float *dst = p.pout + ((size_t)c * k + q) * p.pout_cols + p.vpb[sg] + r0;
      if (g < n) dst[g] = 0.f + __fmul_rn(__int2float_rn(ia), inv);
      if (g + 8 < n) dst[g + 8] = 0.f + __fmul_rn(__int2float_rn(ib), inv);
    }
  }
}

// ---------------------------------------------------------------------------
// host side: the plan of a layer (groups, their owners, blob offsets)
// ---------------------------------------------------------------------------
struct FcPlan {
  int ng, nbr, pcols;
  FcGroup g[FC_GTOT];
  int gstart[FC_CS + 1];
  int nvt, vt0, vr[2], vpb[2];  // V tiles (see FcParams)
  size_t ublob_words, vblob_words;  // per layer
};

// Deal `n` items with sizes sz[] to FC_CS owners, largest first to the least
// loaded owner (at most FC_GMAX each); order[] receives the items owner by owner.
static bool fc_deal(int n, const int *sz, int *order, int *start) {
  int owner[FC_GTOT], load[FC_CS] = {}, cnt[FC_CS] = {}, idx[FC_GTOT];
  for (int i = 0; i < n; ++i) idx[i] = i;
  std::stable_sort(idx, idx + n, [&](int a, int b) { return sz[a] > sz[b]; });
  for (int ii = 0; ii < n; ++ii) {
    const int i = idx[ii];
    int best = -1;
    for (int o = 0; o < FC_CS; ++o)
      if (cnt[o] < FC_GMAX && (best < 0 || load[o] < load[best])) best = o;
    if (best < 0) return false;
    owner[i] = best;
    load[best] += sz[i];
    ++cnt[best];
  }
  int pos = 0;
  for (int o = 0; o < FC_CS; ++o) {
    start[o] = pos;
    for (int i = 0; i < n; ++i)
      if (owner[i] == o) order[pos++] = i;
  }
  start[FC_CS] = pos;
  return true;
}

static int fc_plan(const lbx_proj &pr, FcPlan &P) {
  P = FcPlan{};
  LBX_CHECK_SUP(pr.in_features % FC_ROWS == 0 && pr.out_features % FC_ROWS == 0,
                "fused chain: in/out features must be multiples of %d", FC_ROWS);
  LBX_CHECK_SUP(pr.in_features / FC_ROWS <= FC_NBLK, "fused chain: in_features must be <= %d", FC_NBLK * FC_ROWS);
  P.nbr = pr.n_branches;
  const bool shared = pr.n_branches == 2 && !pr.br[1].v_sign;
  // partial rank space: branch 0's ranks, then branch 1's when it has its own V
  const int pbase[2] = {0, shared ? 0 : pr.br[0].rank};
  P.pcols = pr.br[0].rank + (pr.n_branches == 2 && !shared ? pr.br[1].rank : 0);
  FcGroup all[FC_GTOT];
  int ng = 0;
  for (int b = 0; b < pr.n_branches; ++b)
    for (int r0 = 0; r0 < pr.br[b].rank; r0 += 128) {
      LBX_CHECK_SUP(ng < FC_GTOT, "fused chain: more than %d quantisation groups in a layer", FC_GTOT);
      all[ng++] = FcGroup{b, std::min(128, pr.br[b].rank - r0), r0, pbase[b] + r0};
    }
  int sz[FC_GTOT], order[FC_GTOT];
  for (int i = 0; i < ng; ++i) sz[i] = all[i].n;
  LBX_CHECK_SUP(fc_deal(ng, sz, order, P.gstart), "fused chain: groups do not fit %d per CTA", FC_GMAX);
  for (int i = 0; i < ng; ++i) P.g[i] = all[order[i]];
  P.ng = ng;
  // V tiles over the partial rank space (16 ranks each, per segment)
  const int nseg = shared || pr.n_branches == 1 ? 1 : 2;
  for (int sgi = 0; sgi < nseg; ++sgi) {
    P.vr[sgi] = pr.br[sgi].rank;
    P.vpb[sgi] = pbase[sgi];
  }
  P.vt0 = (P.vr[0] + 15) / 16;
  P.nvt = P.vt0 + (nseg > 1 ? (P.vr[1] + 15) / 16 : 0);
  LBX_CHECK_SUP((P.nvt + FC_CS - 1) / FC_CS <= FC_VTC, "fused chain: more than %d ranks in a layer's V-stages",
                FC_VTC * FC_CS * 16);
  P.ublob_words = (size_t)(pr.out_features / FC_ROWS) * ng * FC_UGW;
  P.vblob_words = (size_t)(pr.in_features / FC_ROWS) * P.nvt * FC_VTW;
  return LBX_OK;
}

static int fc_validate(const lbx_proj *projs, int n_layers) {
  LBX_CHECK_ARG(projs && n_layers >= 1, "need at least one layer");
  int rc = validate(projs, 1);
  if (rc) return rc;
  for (int i = 0; i < n_layers; ++i) {
    rc = validate(projs + i, 1);
    if (rc) return rc;
    if (i) LBX_CHECK_ARG(projs[i].in_features == projs[i - 1].out_features,
                         "layer %d: in_features %d != previous out_features %d", i, projs[i].in_features,
                         projs[i - 1].out_features);
  }
  return LBX_OK;
}

// blob of every layer: its U part (consumed by the layer's own launch) then
// its V part (consumed by the launch before it)
static size_t fc_blob_words(const lbx_proj *projs, int n_layers, size_t *uoff, size_t *voff) {
  size_t tot = 0;
  for (int i = 0; i < n_layers; ++i) {
    FcPlan P;
    if (fc_plan(projs[i], P)) return 0;
    if (uoff) uoff[i] = tot;
    tot += (P.ublob_words + 63) & ~(size_t)63;
    if (voff) voff[i] = tot;
    tot += (P.vblob_words + 63) & ~(size_t)63;
  }
  return tot;
}

// U part: [N/256][slot][256 rows][4 words] (words past the branch's row are 0)
__global__ void fc_pack_u_kernel(const int32_t *u0, const int32_t *u1, int w0, int w1, FcPlan P, int nrows_blk,
                                 uint32_t *dst) {
  const size_t total = (size_t)nrows_blk * P.ng * FC_ROWS * 4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int w = (int)(i & 3);
    const size_t rr = i >> 2;
    const int row = (int)(rr % FC_ROWS);
    const size_t cs = rr / FC_ROWS;
    const int s = (int)(cs % P.ng), c = (int)(cs / P.ng);
    const FcGroup G = P.g[s];
    const int word = G.r0 / 32 + w;
    const int words = G.b ? w1 : w0;
    const int32_t *src = G.b ? u1 : u0;
    dst[i] = word < words ? (uint32_t)src[(size_t)(c * FC_ROWS + row) * words + word] : 0u;
  }
}

// V part: [K/256][tile][16 ranks][8 words], rows 4-7 and 12-15 with their two
// 4-word halves swapped (word w of row r at w ^ (r & 4)); rows past the
// segment's rank are 0
__global__ void fc_pack_v_kernel(const int32_t *v0, const int32_t *v1, int Wv, FcPlan P, int nblk, uint32_t *dst) {
  const size_t total = (size_t)nblk * P.nvt * FC_VTW;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % FC_VPITCH);
    const size_t rr = i / FC_VPITCH;
    const int r = (int)(rr % 16);
    const size_t ct = rr / 16;
    const int mt = (int)(ct % P.nvt), c = (int)(ct / P.nvt);
    const int sg = mt < P.vt0 ? 0 : 1;
    const int rank = 16 * (sg ? mt - P.vt0 : mt) + r;
    const int32_t *src = sg ? v1 : v0;
    const int wl = w ^ (r & 4);  // the logical word stored at this position
    uint32_t v = 0u;
    if (rank < P.vr[sg]) v = (uint32_t)src[(size_t)rank * Wv + c * 8 + wl];
    dst[i] = v;
  }
}

static size_t fc_ws_bytes(const lbx_proj *projs, int n_layers, int k) {
  size_t mx = 0;
  for (int i = 0; i < n_layers; ++i) {
    FcPlan P;
    if (fc_plan(projs[i], P)) return 0;
    mx = std::max(mx, (size_t)(projs[i].in_features / FC_ROWS) * k * P.pcols * 4);
  }
  return 2 * al256(mx);
}

}  // namespace lbx

extern "C" size_t lbx_chain_prepare_size(const lbx_proj *projs, int32_t n_layers) {
  using namespace lbx;
  if (fc_validate(projs, n_layers)) return 0;
  return fc_blob_words(projs, n_layers, nullptr, nullptr) * 4;
}

extern "C" int lbx_chain_prepare(const lbx_proj *projs, int32_t n_layers, void *blob, size_t blob_bytes,
                                 cudaStream_t stream) {
  using namespace lbx;
  int rc = fc_validate(projs, n_layers);
  if (rc) return rc;
  std::vector<size_t> uo(n_layers), vo(n_layers);
  const size_t words = fc_blob_words(projs, n_layers, uo.data(), vo.data());
  if (!words) return LBX_EUNSUPPORTED;  // (the reason is in lbx_last_error)
  LBX_CHECK_ARG(blob && aligned16(blob) && blob_bytes >= words * 4, "blob too small (%zu < %zu) or unaligned",
                blob_bytes, words * 4);
  uint32_t *b = reinterpret_cast<uint32_t *>(blob);
  for (int i = 0; i < n_layers; ++i) {
    const lbx_proj &pr = projs[i];
    FcPlan P;
    rc = fc_plan(pr, P);
    if (rc) return rc;
    const int w0 = (pr.br[0].rank + 31) / 32, w1 = pr.n_branches > 1 ? (pr.br[1].rank + 31) / 32 : 0;
    fc_pack_u_kernel<<<296, 256, 0, stream>>>(pr.br[0].u_sign, pr.n_branches > 1 ? pr.br[1].u_sign : nullptr, w0,
                                              w1, P, pr.out_features / FC_ROWS, b + uo[i]);
    const bool own1 = pr.n_branches > 1 && pr.br[1].v_sign;
    fc_pack_v_kernel<<<296, 256, 0, stream>>>(pr.br[0].v_sign, own1 ? pr.br[1].v_sign : nullptr,
                                              pr.in_features / 32, P, pr.in_features / FC_ROWS, b + vo[i]);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "chain prepare launch");
  }
  return LBX_OK;
}

namespace lbx {

// the launches of one chain for tokens [0, k) of acts (already offset to the
// sub-batch's first token), partial sums in part[0] / part[1].  `alt` (one
// token): the launches alternate between the FC_SMEM_SIDE and FC_REG_SIDE
// builds (one CTA of a launch per SM); otherwise every launch is a 64-register
// build, two CTAs per SM (for two chains that run at once).
static int fc_run(const lbx_proj *projs, int n_layers, int k, int dtype, void *const *acts, const uint32_t *b,
                  const std::vector<FcPlan> &plan, const std::vector<size_t> &uo, const std::vector<size_t> &vo,
                  float *const (&part)[2], size_t smax, bool alt, cudaStream_t stream) {
  alt = alt && k == 1;  // the alternating builds are one-token builds
  for (int i = -1; i < n_layers; ++i) {
    FcParams p = {};
    p.k = k;
    p.adt = dtype;
    const int nx = i + 1;  // the layer whose V partials this launch forms
    if (i >= 0) {
      const lbx_proj &pr = projs[i];
      const FcPlan &P = plan[i];
      p.has_u = 1;
      p.ublob = b + uo[i];
      p.nbr = pr.n_branches;
      for (int bb = 0; bb < pr.n_branches; ++bb) {
        p.u1[bb] = pr.br[bb].u1;
        p.mid[bb] = pr.br[bb].mid;
      }
      p.bias = pr.bias;
      p.pin = part[i & 1];
      p.pin_cols = P.pcols;
      p.nblk_in = pr.in_features / FC_ROWS;
      p.y = acts[i + 1];
      p.ng = P.ng;
      for (int g = 0; g < P.ng; ++g) p.g[g] = P.g[g];
      for (int o = 0; o <= FC_CS; ++o) p.gstart[o] = P.gstart[o];
      p.N = pr.out_features;
      LBX_CHECK_ARG(aligned16(pr.br[0].u1) && (pr.n_branches < 2 || aligned16(pr.br[1].u1)) &&
                        (!pr.bias || aligned16(pr.bias)),
                    "u1 / bias must be 16-byte aligned");
    } else {
      p.x = acts[0];
      p.N = projs[0].in_features;
    }
    if (nx < n_layers) {
      const lbx_proj &pn = projs[nx];
      const FcPlan &Q = plan[nx];
      p.has_v = 1;
      p.vblob = b + vo[nx];
      p.nvseg = pn.n_branches == 2 && pn.br[1].v_sign ? 2 : 1;
      for (int sg = 0; sg < p.nvseg; ++sg) {
        p.v2[sg] = pn.br[sg].v2;
        LBX_CHECK_ARG(aligned16(pn.br[sg].v2), "v2 must be 16-byte aligned");
      }
      p.pout = part[nx & 1];
      p.pout_cols = Q.pcols;
      p.nvt = Q.nvt;
      p.vt0 = Q.vt0;
      for (int sg = 0; sg < 2; ++sg) {
        p.vr[sg] = Q.vr[sg];
        p.vpb[sg] = Q.vpb[sg];
      }
    }
    const int nclusters = p.N / FC_ROWS;
    const FcSmem Ls = fc_smem(k, p.ng);
    LBX_CHECK_SUP((size_t)Ls.total <= smax, "fused chain needs %d bytes of shared memory (max %zu)", Ls.total, smax);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(nclusters * FC_CS);
    cfg.blockDim = dim3(FC_THREADS);
    const bool sside = alt && ((i + 1) & 1) == 0;
    cfg.dynamicSmemBytes = sside ? std::max(Ls.total, FC_SMEM_PAD) : Ls.total;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = FC_CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    // (fc_smem has the staging buffer exactly when k > 1: the bulk build)
    void (*fn)(FcParams) = alt     ? (sside ? fc_kernel<FC_SMEM_SIDE, false> : fc_kernel<FC_REG_SIDE, false>)
                           : k > 1 ? fc_kernel<64, true>
                                   : fc_kernel<64, false>;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, p);
    if (e != cudaSuccess) return cuda_status(e, "fused chain launch");
  }
  return LBX_OK;
}

// tokens of the first of the two sub-chains a call of k tokens runs as.  A
// chain's cost grows faster than its token count (the sums exchange carries
// every token, and from 3 tokens on one CTA fits per SM), so two concurrent
// sub-chains win from 2 tokens on; measured per C2 layer: 2 tokens 14.7 us as
// one chain, 9.7 as two; 4 tokens 31.2 and 12.8.
static int fc_first(int k) { return k <= 1 ? k : (k + 1) / 2; }

// the library's helper stream of this device (a call of more than FC_MAXK
// tokens runs its second sub-chain there, forked from and joined back to the
// caller's stream through two events)
struct FcFork {
  cudaStream_t s;
  cudaEvent_t fork, join;
};
static int fc_fork(FcFork &f) {
  static DevCache<FcFork> cache;
  return cache.get(f, [](FcFork &o) {
    cudaError_t e = cudaStreamCreateWithFlags(&o.s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&o.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&o.join, cudaEventDisableTiming);
    return cuda_status(e, "fused chain helper stream");
  });
}

// Instantiated CUDA graphs of recent calls, per device.  A call outside
// stream capture with the same arguments as a cached one (the same layers,
// buffers, token count and dtype) replays the graph: one host launch instead
// of n_layers + 1 cluster launches, which cost the host more than the ~7 us a
// C2 layer takes on the device.  A miss captures the launches on a private
// stream (the caller's stream never enters capture mode), instantiates them
// and launches the graph on the caller's stream.  A graph reads its buffers
// through the pointers it was built with, so new contents in the same buffers
// need no new graph.
constexpr int FC_GRAPHS = 16;
struct FcGraph {
  std::vector<uintptr_t> key;
  cudaGraphExec_t exec = nullptr;
  uint64_t used = 0;
};
struct FcGraphs {
  cudaStream_t cap = nullptr;  // the private capture stream
  std::vector<FcGraph> g;
  uint64_t tick = 0;
};
static std::mutex &fc_graph_mu() {
  static std::mutex m;
  return m;
}
static FcGraphs g_fc_graphs[LBX_MAX_DEVICES];

// every argument that the launches depend on, field by field (not the
// descriptors' raw bytes, whose padding a caller need not keep equal)
static std::vector<uintptr_t> fc_key(const lbx_proj *projs, int n_layers, int n_tokens, int dtype,
                                     void *const *acts, const void *blob, size_t blob_bytes, void *ws,
                                     size_t ws_bytes) {
  std::vector<uintptr_t> k;
  k.reserve(8 + 16 * (size_t)n_layers);
  auto u = [&](const void *v) { k.push_back(reinterpret_cast<uintptr_t>(v)); };
  k.push_back((uintptr_t)n_layers);
  k.push_back((uintptr_t)n_tokens);
  k.push_back((uintptr_t)dtype);
  u(blob);
  k.push_back((uintptr_t)blob_bytes);
  u(ws);
  k.push_back((uintptr_t)ws_bytes);
  for (int i = 0; i <= n_layers; ++i) u(acts[i]);
  for (int i = 0; i < n_layers; ++i) {
    const lbx_proj &pr = projs[i];
    k.push_back((uintptr_t)(uint32_t)pr.in_features);
    k.push_back((uintptr_t)(uint32_t)pr.out_features);
    k.push_back((uintptr_t)(uint32_t)pr.n_branches);
    u(pr.bias);
    for (int bb = 0; bb < 2 && bb < pr.n_branches; ++bb) {  // (not yet validated)
      const lbx_branch &br = pr.br[bb];
      u(br.v_sign);
      u(br.v2);
      u(br.mid);
      u(br.u_sign);
      u(br.u1);
      k.push_back((uintptr_t)(uint32_t)br.rank);
    }
  }
  return k;
}

}  // namespace lbx

extern "C" size_t lbx_chain_fused_workspace_size(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens) {
  using namespace lbx;
  if (fc_validate(projs, n_layers) || n_tokens < 1 || n_tokens > 2 * FC_MAXK) return 0;
  const int k1 = fc_first(n_tokens);
  // a split call keeps both sub-chains' partial sums
  return n_tokens == 1 ? fc_ws_bytes(projs, n_layers, 1) : 2 * fc_ws_bytes(projs, n_layers, k1);
}

extern "C" int lbx_chain_fused(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens, int32_t dtype,
                               void *const *acts, const void *blob, size_t blob_bytes, void *ws, size_t ws_bytes,
                               cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(projs && n_layers >= 1, "need at least one layer");
  LBX_CHECK_SUP(n_tokens >= 1 && n_tokens <= 2 * FC_MAXK, "fused chain: 1..%d tokens", 2 * FC_MAXK);
  LBX_CHECK_ARG(dtype == LBX_F32 || dtype == LBX_BF16, "bad dtype");
  LBX_CHECK_ARG(acts && blob, "NULL argument");
  for (int i = 0; i <= n_layers; ++i) LBX_CHECK_ARG(acts[i], "acts[%d] is NULL", i);
  // outside the caller's stream capture, a call whose arguments equal a cached
  // graph's replays it (the arguments were checked and planned when it was
  // built); inside it, the call makes its launches itself
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  int rc = cuda_status(cudaStreamIsCapturing(stream, &cs), "fused chain capture query");
  if (rc) return rc;
  const int dev = cur_device();
  const bool use_graph = cs == cudaStreamCaptureStatusNone && dev >= 0 && dev < LBX_MAX_DEVICES;
  std::vector<uintptr_t> key;
  if (use_graph) {
    key = fc_key(projs, n_layers, n_tokens, dtype, acts, blob, blob_bytes, ws, ws_bytes);
    std::lock_guard<std::mutex> lk(fc_graph_mu());  // (held through the launch: no eviction meanwhile)
    FcGraphs &G = g_fc_graphs[dev];
    for (FcGraph &e : G.g)
      if (e.key == key) {
        e.used = ++G.tick;
        return cuda_status(cudaGraphLaunch(e.exec, stream), "fused chain graph launch");
      }
  }
  rc = fc_validate(projs, n_layers);
  if (rc) return rc;
  // every layer's plan once: blob offsets (as fc_blob_words lays them out)
  // and the partial-sum buffers (as fc_ws_bytes sizes them)
  const int k1 = fc_first(n_tokens), k2 = n_tokens - k1;
  std::vector<FcPlan> plan(n_layers);
  std::vector<size_t> uo(n_layers), vo(n_layers);
  size_t words = 0, pmax = 0;
  for (int i = 0; i < n_layers; ++i) {
    rc = fc_plan(projs[i], plan[i]);
    if (rc) return rc;
    uo[i] = words;
    words += (plan[i].ublob_words + 63) & ~(size_t)63;
    vo[i] = words;
    words += (plan[i].vblob_words + 63) & ~(size_t)63;
    pmax = std::max(pmax, (size_t)(projs[i].in_features / FC_ROWS) * k1 * plan[i].pcols * 4);
  }
  LBX_CHECK_ARG(blob_bytes >= words * 4, "blob too small (%zu < %zu)", blob_bytes, words * 4);
  const size_t one = 2 * al256(pmax);  // one sub-chain's partial sums
  const size_t need = k2 ? 2 * one : one;
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  static DevCache<size_t> smax_cache;
  size_t smax = 0;
  rc = smax_cache.get(smax, [](size_t &out) {
    // every build may take the SM's shared memory, and prefers the largest
    // carveout, so that an FC_SMEM_SIDE CTA leaves room for an FC_REG_SIDE one
    cudaError_t e = cudaSuccess;
    for (auto fn : {fc_kernel<64, false>, fc_kernel<64, true>, fc_kernel<FC_SMEM_SIDE, false>,
                    fc_kernel<FC_REG_SIDE, false>}) {
      if (e == cudaSuccess) e = allow_max_smem(fn, &out);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    }
    return e != cudaSuccess ? cuda_status(e, "fused chain smem attribute") : (int)LBX_OK;
  });
  if (rc) return rc;
  const uint32_t *b = reinterpret_cast<const uint32_t *>(blob);
  uint8_t *w = reinterpret_cast<uint8_t *>(ws);
  float *const part1[2] = {reinterpret_cast<float *>(w), reinterpret_cast<float *>(w + one / 2)};
  // 2..8 tokens: two sub-chains of k1 and k2 tokens (tokens never interact, so
  // every token gets the bits of a chain of its own), the second on the helper
  // stream so that both run at once
  FcFork f = {};
  if (k2) {
    rc = fc_fork(f);
    if (rc) return rc;
  }
  const size_t esz = dtype == LBX_F32 ? 4 : 2;
  std::vector<void *> acts2(n_layers + 1);
  for (int i = 0; i <= n_layers; ++i) {
    const size_t feat = i == 0 ? projs[0].in_features : projs[i - 1].out_features;
    acts2[i] = reinterpret_cast<uint8_t *>(acts[i]) + (size_t)k1 * feat * esz;
  }
  float *const part2[2] = {reinterpret_cast<float *>(w + one), reinterpret_cast<float *>(w + one + one / 2)};
  auto launch_all = [&](cudaStream_t st) -> int {
    if (!k2) return fc_run(projs, n_layers, k1, dtype, acts, b, plan, uo, vo, part1, smax, true, st);
    int r = cuda_status(cudaEventRecord(f.fork, st), "fused chain fork");
    if (!r) r = cuda_status(cudaStreamWaitEvent(f.s, f.fork, 0), "fused chain fork");
    // (two alternating chains would contend for the same builds' SM slots;
    // measured per C2 layer at 2 tokens: 9.7 us plain, 10.7 alternating)
    if (!r) r = fc_run(projs, n_layers, k2, dtype, acts2.data(), b, plan, uo, vo, part2, smax, false, f.s);
    if (!r) r = fc_run(projs, n_layers, k1, dtype, acts, b, plan, uo, vo, part1, smax, false, st);
    if (!r) r = cuda_status(cudaEventRecord(f.join, f.s), "fused chain join");
    if (!r) r = cuda_status(cudaStreamWaitEvent(st, f.join, 0), "fused chain join");
    return r;
  };
  if (!use_graph) return launch_all(stream);
  // this call's graph: captured now, unless another thread has just added it
  std::lock_guard<std::mutex> lk(fc_graph_mu());
  FcGraphs &G = g_fc_graphs[dev];
  cudaGraphExec_t exec = nullptr;
  for (FcGraph &e : G.g)
    if (e.key == key) {
      e.used = ++G.tick;
      exec = e.exec;
      break;
    }
  if (!exec) {
    if (!G.cap) {
      rc = cuda_status(cudaStreamCreateWithFlags(&G.cap, cudaStreamNonBlocking), "fused chain capture stream");
      if (rc) return rc;
    }
    rc = cuda_status(cudaStreamBeginCapture(G.cap, cudaStreamCaptureModeThreadLocal), "fused chain capture");
    if (rc) return rc;
    rc = launch_all(G.cap);
    cudaGraph_t graph = nullptr;
    const cudaError_t ee = cudaStreamEndCapture(G.cap, &graph);  // (always: the stream leaves capture)
    if (!rc && ee != cudaSuccess) rc = cuda_status(ee, "fused chain capture");
    if (!rc) rc = cuda_status(cudaGraphInstantiate(&exec, graph, 0), "fused chain graph");
    if (graph) cudaGraphDestroy(graph);
    if (rc) return rc;
    if ((int)G.g.size() >= FC_GRAPHS) {  // drop the least recently used graph
      size_t lru = 0;
      for (size_t i = 1; i < G.g.size(); ++i)
        if (G.g[i].used < G.g[lru].used) lru = i;
      cudaGraphExecDestroy(G.g[lru].exec);  // (freed once any launch in flight completes)
      G.g.erase(G.g.begin() + (long)lru);
    }
    G.g.push_back(FcGraph{std::move(key), exec, ++G.tick});
  }
  return cuda_status(cudaGraphLaunch(exec, stream), "fused chain graph launch");
}
