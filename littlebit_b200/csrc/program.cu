// Persistent programs: a decoder step (or a chain of LittleBit layers) as ONE
// cooperative launch on sm_100a.
//
// A program is a table of phases.  Each phase is a set of independent units of
// one kind -- V-stage row tiles, U-stage row tiles, attention chunks, lm_head
// row streams, ... -- and the units are the same device bodies the standalone
// kernels run, so a program computes exactly the bits the kernel-per-op path
// computes.  One CTA per SM walks the table: it runs its units of the phase
// (unit = blockIdx.x, blockIdx.x + gridDim.x, ...), then meets the others at a
// grid barrier.  Replacing kernel boundaries by barriers removes the launch,
// grid-completion and dependent-launch latencies of ~300 kernels per decoder
// step; the data never leaves L2 between phases.
//
// Weights do not depend on activations, so each CTA requests (cp.async.bulk)
// the weights of its next unit -- across the phase boundary too -- as soon as
// the current unit has released its shared-memory weight region: HBM latency
// overlaps the barrier and the preceding phase, as it overlaps the preceding
// kernel under programmatic dependent launch.
//
// Cross-CTA data produced inside the program is only read through L2
// (ld.global.cg), because L1 is not coherent across SMs within a launch.
//
// Every wait is bounded (1 s of %globaltimer for the grid barrier; the weight
// barriers as in the standalone kernels).  A timeout records an error code,
// raises the program's abort word -- every CTA leaves at its next barrier --
// and each CTA waits for its own copies in flight before it exits.  The
// co-residency the barrier needs is guaranteed by the cooperative launch (it
// fails rather than oversubscribe the GPU).

#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace lbx {

enum : int {
  PH_V = 1,      // V-stage tiles (ncb = MMA column blocks)
  PH_U = 2,      // U-stage tiles
  PH_ATTN = 3,   // attention units
  PH_START = 4,  // embed tokens (+ positions, RoPE table, start word on unit 0)
  PH_NORM = 5,   // RMSNorm rows (final hidden states)
  PH_LM = 6,     // lm_head row streams (ncb = tokens per pass)
  PH_ARGMAX = 7, // per-unit winners -> token ids
};

// which kernel argument a phase takes at run time
enum : int { IO_NONE = 0, IO_TOKENS = 1, IO_TREE = 2, IO_HIDDEN = 3, IO_LOGITS = 4, IO_ARGMAX = 5 };

struct StartP {
  const uint16_t *table;  // embedding [vocab, hidden] bf16
  const int64_t *ids;     // kernel argument
  int hidden, vocab, n, d;
  float theta;
  float *x;               // [n, hidden]
  int32_t *pos;           // [n] rotary positions of this step
  int32_t *start_word;    // the step's first cache slot (read by attention)
  float2 *rope;           // [n][d/2]
};
struct NormP {
  const float *x, *w;
  int hidden;
  float eps;
  float *out;  // kernel argument
};
struct ArgP {
  const unsigned long long *best;
  int nblocks, n;
  int64_t *out;  // kernel argument
};

struct __align__(16) Phase {
  int kind, units, ncb, io;
  int64_t io_off;  // element offset into the kernel-argument buffer
  union {
    VParams v;
    UParams u;
    AttnParams a;
    LmParams l;
    StartP st;
    NormP nm;
    ArgP am;
  };
};
static_assert(sizeof(Phase) % 16 == 0, "phase records are copied in 16-byte pieces");

struct ProgIo {
  const int64_t *tokens;
  int start;
  const int32_t *start_dev;
  const int32_t *pos;
  const uint64_t *tree;
  float *hidden;
  float *logits;
  int64_t *argmax;
};

struct GridBar {
  unsigned long long arrivals;  // monotonic count of CTA arrivals, all launches
  int abort, pad;
};

// Phase probes: no-ops in the library build.  A profiling build may define
// LBX_PPROBE(phase, point) to timestamp each CTA's passage through a phase.
#ifndef LBX_PPROBE
#define LBX_PPROBE(ph, what) ((void)0)
#endif

constexpr int PTHREADS = 512;
constexpr uint64_t SPIN_NS = 1000000000ull;  // bound of every grid-barrier wait

LBX_DEV uint64_t gtime_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
LBX_DEV unsigned long long ld_acquire64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
LBX_DEV void red_release_add64(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
LBX_DEV int ld_relaxed_i(const int *p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// barrier over all CTAs of the launch.  The arrival counter only grows, and
// barrier i of a launch completes when it reaches base + (i+1)*G, where base
// (a multiple of G: every launch has G CTAs) is known to every CTA from the
// counter's value at launch start.  Arriving is one release-reduction (no
// round trip); waiting polls the counter.  False when the program is being
// aborted (timeout here or elsewhere).
LBX_DEV bool grid_sync(GridBar *gb, unsigned long long target) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    red_release_add64(&gb->arrivals, 1ull);
    const uint64_t t0 = gtime_ns();
    while (ld_acquire64(&gb->arrivals) < target) {
      if (ld_relaxed_i(&gb->abort)) {
        ok = 0;
        break;
      }
      if (gtime_ns() - t0 > SPIN_NS) {
        atomicCAS(&g_lbx_device_error, 0, 0x501);
        atomicExch(&gb->abort, 1);
        ok = 0;
        break;
      }
    }
    if (ok && ld_relaxed_i(&gb->abort)) ok = 0;
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// ---------------------------------------------------------------------------
// small phase bodies
// ---------------------------------------------------------------------------
LBX_DEV void start_unit(const StartP &p, const ProgIo &io, int u) {
  const int64_t id = p.ids[u];
  const bool ok = id >= 0 && id < p.vocab;
  if (!ok && threadIdx.x == 0) atomicCAS(&g_lbx_device_error, 0, 0x301);
  for (int h = threadIdx.x; h < p.hidden; h += blockDim.x)
    p.x[(int64_t)u * p.hidden + h] = ok ? bf16_to_f32(p.table[id * p.hidden + h]) : 0.f;
  if (u == 0) {
    const int start = io.start_dev ? *io.start_dev : io.start;
    const int half = p.d >> 1;
    for (int i = threadIdx.x; i < p.n; i += blockDim.x) p.pos[i] = io.pos ? io.pos[i] : start + i;
    if (threadIdx.x == 0) *p.start_word = start;
    for (int e = threadIdx.x; e < p.n * half; e += blockDim.x) {
      const int i = e / half;
      p.rope[e] = rope_cs_d(io.pos ? io.pos[i] : start + i, e - i * half, p.d, p.theta);
    }
  }
}

// RMSNorm of row u: same arithmetic as rmsnorm_kernel at 512 threads
LBX_DEV void norm_unit(const NormP &p, int u) {
  __shared__ float red[32];
  const float *xr = p.x + (int64_t)u * p.hidden;
  float ss = 0.f;
  for (int h = threadIdx.x; h < p.hidden; h += blockDim.x) {
    const float v = __ldcg(xr + h);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rs = 1.0f / sqrtf(red[0] / (float)p.hidden + p.eps);
  for (int h = threadIdx.x; h < p.hidden; h += blockDim.x)
    p.out[(int64_t)u * p.hidden + h] = __ldcg(xr + h) * rs * p.w[h];
  __syncthreads();
}

// ---------------------------------------------------------------------------
// executor
// ---------------------------------------------------------------------------
struct ArmState {
  uint32_t armed;  // barriers of LinShm with copies in flight
};

LBX_DEV void issue_unit(const Phase &P, int u, uint8_t *W, LinShm &sh, ArmState &as) {
  if (P.kind != PH_V && P.kind != PH_U) return;
  __syncthreads();  // the previous unit's reads of the weight region are complete
  if (P.kind == PH_V) {
    vstage_issue(P.v, u, W, sh);
    if (threadIdx.x == 0) as.armed |= 1u << UT_MAX;
  } else {
    ustage_issue(P.u, u, W, sh);
    if (threadIdx.x == 0) {
      const int ut = P.u.ut;
      const USeg &sg = P.u.seg[useg_of(P.u, u)];
      for (int t = 0; t < ut; ++t)
        if ((u - sg.cta0) * (16 * ut) + 16 * t < sg.out) as.armed |= 1u << t;
    }
  }
}

// the executor is specialised per program: every linear of a program has the
// same token count (NCB MMA column blocks) and every lm_head pass the same
// width (LMNT), so each instance inlines only the bodies it runs
template <int NCB, int LMNT>
LBX_DEV bool run_unit(const Phase &P, const ProgIo &io, int u, uint8_t *W, uint8_t *S, LinShm &sh) {
  switch (P.kind) {
    case PH_V:
      return P.v.prologue == LBX_PRO_SILU_MUL ? vstage_run<NCB, PM_SILU>(P.v, u, W, S, sh)
             : P.v.prologue == LBX_PRO_MUL   ? vstage_run<NCB, PM_MUL>(P.v, u, W, S, sh)
                                             : vstage_run<NCB, PM_X>(P.v, u, W, S, sh);
    case PH_U:
      return ustage_run<NCB>(P.u, u, P.units, W, S, sh);
    case PH_ATTN:
      attn_unit<false>(P.a, u, reinterpret_cast<float *>(S));
      return true;
    case PH_START:
      start_unit(P.st, io, u);
      return true;
    case PH_NORM:
      norm_unit(P.nm, u);
      return true;
    case PH_LM:
      lmhead_unit<LMNT>(P.l, u, P.units, reinterpret_cast<float *>(S));
      return true;
    case PH_ARGMAX:
      argmax_unit(P.am.best, P.am.nblocks, P.am.n, P.am.out);
      return true;
    default:
      return false;
  }
}

// request the record of a phase into shared memory (bulk copy: no registers,
// lands while the current phase runs)
LBX_DEV void fetch_phase(Phase &dst, const Phase *src, uint64_t *bar) {
  __syncthreads();  // the record this copy replaces has been read by every thread
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar, (uint32_t)sizeof(Phase));
    bulk_g2s(&dst, src, (uint32_t)sizeof(Phase), bar);
  }
}

// wait for a fetched record and attach its kernel arguments
LBX_DEV bool ready_phase(Phase &dst, uint64_t *bar, uint32_t &par, const ProgIo &io) {
  const bool ok = __syncthreads_and(mbar_wait_bounded(bar, par, 0x503));
  par ^= 1u;
  if (threadIdx.x == 0 && ok) {
    switch (dst.io) {
      case IO_TOKENS: dst.st.ids = io.tokens; break;
      case IO_TREE: dst.a.tree = io.tree; break;
      case IO_HIDDEN: dst.nm.out = io.hidden; break;
      case IO_LOGITS: dst.l.logits = io.logits ? io.logits + dst.io_off : nullptr; break;
      case IO_ARGMAX: dst.am.out = io.argmax + dst.io_off; break;
      default: break;
    }
  }
  __syncthreads();
  return ok;
}

// wait (bounded) for this CTA's own copies in flight, before it leaves
LBX_DEV void drain(LinShm &sh, const ArmState &as) {
  if (threadIdx.x == 0)
    for (int b = 0; b <= UT_MAX; ++b)
      if (as.armed & (1u << b)) {
        const uint64_t t0 = gtime_ns();
        while (!mbar_try_wait(&sh.bar[b], sh.par[b]) && gtime_ns() - t0 < SPIN_NS) {
        }
      }
  __syncthreads();
}

template <int NCB, int LMNT>
__global__ void __launch_bounds__(PTHREADS, 1)
    program_kernel(const Phase *__restrict__ prog, int nph, GridBar *gb, ProgIo io, int s_bytes) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ LinShm sh;
  __shared__ Phase sph[2];
  __shared__ ArmState as;
  __shared__ __align__(8) uint64_t pbar;
  __shared__ unsigned long long s_base;
  uint8_t *S = smem;            // scratch of the running unit
  uint8_t *W = smem + s_bytes;  // weights of the running / next unit
  linshm_init(sh);
  if (threadIdx.x == 0) {
    as.armed = 0;
    mbar_init(&pbar, 1);
    fence_mbar_init();
    // fewer than G arrivals of this launch can precede this read (the first
    // barrier needs this CTA), and earlier launches left a multiple of G
    const unsigned long long a0 = ld_acquire64(&gb->arrivals);
    s_base = a0 - a0 % gridDim.x;
  }
  __syncthreads();
  uint32_t ppar = 0;
  if (ld_relaxed_i(&gb->abort)) {  // a previous program on this workspace failed
    if (threadIdx.x == 0) atomicCAS(&g_lbx_device_error, 0, 0x502);
    return;
  }
  const int G = gridDim.x, b = blockIdx.x;
  fetch_phase(sph[0], prog, &pbar);
  if (!ready_phase(sph[0], &pbar, ppar, io)) return;
  if (b < sph[0].units) issue_unit(sph[0], b, W, sh, as);
  for (int ph = 0; ph < nph; ++ph) {
    const Phase &P = sph[ph & 1];
    Phase &N = sph[(ph + 1) & 1];
    const bool more = ph + 1 < nph;
    if (more) fetch_phase(N, prog + ph + 1, &pbar);
    LBX_PPROBE(ph, 0);
    for (int u = b; u < P.units; u += G) {
      const bool ok = run_unit<NCB, LMNT>(P, io, u, W, S, sh);
      __syncthreads();
      if (threadIdx.x == 0) {
        if (P.kind == PH_V) as.armed &= ~(1u << UT_MAX);
        if (P.kind == PH_U) as.armed &= ~((1u << UT_MAX) - 1u);
      }
      if (!ok) {
        if (threadIdx.x == 0) atomicExch(&gb->abort, 1);
        drain(sh, as);
        return;
      }
      if (u + G < P.units) issue_unit(P, u + G, W, sh, as);
    }
    LBX_PPROBE(ph, 1);
    if (!more) break;  // the kernel's completion is the last barrier
    if (!ready_phase(N, &pbar, ppar, io)) {
      if (threadIdx.x == 0) atomicExch(&gb->abort, 1);
      drain(sh, as);
      return;
    }
    LBX_PPROBE(ph, 4);
    if (b < N.units) issue_unit(N, b, W, sh, as);
    LBX_PPROBE(ph, 2);
    if (!grid_sync(gb, s_base + (unsigned long long)(ph + 1) * G)) {
      drain(sh, as);
      return;
    }
    LBX_PPROBE(ph, 3);
  }
}

// ---------------------------------------------------------------------------
// host side: building, caching and launching programs
// ---------------------------------------------------------------------------
struct Program {
  std::vector<Phase> host;
  Phase *dev = nullptr;
  size_t w_bytes = 0, s_bytes = 0;
  int nph = 0;
  int ncb = 1, lmnt = 1;  // executor instance
};

struct ProgBuilder {
  std::vector<Phase> ph;
  size_t wmax = 0, smax = 0;
  int ncb = 0, lmnt = 0;  // 0: no phase of that kind yet
  void push(const Phase &p, size_t w, size_t s) {
    ph.push_back(p);
    wmax = std::max(wmax, w);
    smax = std::max(smax, s);
  }
};

using ProgKern = void (*)(const Phase *, int, GridBar *, ProgIo, int);

// instances: k = 1, 2, 3..4 tokens (NCB 1, lm_head width 1/2/4), 5..8 (NCB 2),
// 9..16 (NCB 4); lm_head passes of up to 8 tokens
static ProgKern program_instance(int ncb, int lmnt) {
  if (ncb == 1) return lmnt == 1 ? program_kernel<1, 1> : lmnt == 2 ? program_kernel<1, 2> : program_kernel<1, 4>;
  if (ncb == 2) return program_kernel<2, 8>;
  return program_kernel<4, 8>;
}

// dynamic shared memory every executor instance may use; SM count
static int program_budget(size_t &dyn_max, int &nsm) {
  static DevCache<size_t> cache;
  nsm = device_sm_count();
  return cache.get(dyn_max, [](size_t &out) {
    size_t mn = (size_t)-1, g = 0;
    for (ProgKern k : {program_kernel<1, 1>, program_kernel<1, 2>, program_kernel<1, 4>, program_kernel<2, 8>,
                       program_kernel<4, 8>}) {
      cudaError_t e = allow_max_smem(k, &g);
      // keep the L1 share as large as each launch's shared memory allows: the
      // executor's stack lives there
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxL1);
      if (e != cudaSuccess) return cuda_status(e, "program smem attribute");
      mn = std::min(mn, g);
    }
    out = mn;
    return (int)LBX_OK;
  });
}

// the two phases of each token batch of one linear call
static int build_linear(ProgBuilder &B, const lbx_proj *projs, const lbx_linear_args &a, void *ws,
                        size_t budget) {
  int rc = check_args(projs, &a);
  if (rc) return rc;
  for (int t0 = 0; t0 < a.n_tokens; t0 += LBX_MAX_TOKENS) {
    const int k = std::min(LBX_MAX_TOKENS, a.n_tokens - t0);
    LinPrep P;
    rc = prep_linear(projs, &a, t0, k, ws, budget, budget, P, /*multi_tile=*/false);
    if (rc) return rc;
    LBX_CHECK_SUP(!B.ncb || B.ncb == P.ncb, "a program's linears must share the token count");
    B.ncb = P.ncb;
    Phase v = {};
    v.kind = PH_V;
    v.units = P.vunits;
    v.ncb = P.ncb;
    v.v = P.vp;
    B.push(v, P.v_w, P.v_s);
    Phase u = {};
    u.kind = PH_U;
    u.units = P.uunits;
    u.ncb = P.ncb;
    u.u = P.up;
    B.push(u, P.u_w, P.u_s);
  }
  return LBX_OK;
}

static std::mutex g_prog_mu;
static std::unordered_map<uint64_t, Program *> g_progs;

static uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
  return h;
}

// upload a built program (once per key; never while the stream is captured)
static int finish_program(uint64_t key, ProgBuilder &B, cudaStream_t stream, Program *&out) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cs);
  if (e != cudaSuccess) return cuda_status(e, "program capture query");
  LBX_CHECK_SUP(cs == cudaStreamCaptureStatusNone,
                "a persistent program is built on its first call, which must run outside stream capture");
  Program *P = new Program();
  P->host = std::move(B.ph);
  P->nph = (int)P->host.size();
  P->w_bytes = B.wmax;
  P->s_bytes = (B.smax + 255) & ~(size_t)255;
  P->ncb = B.ncb ? B.ncb : 1;
  P->lmnt = B.lmnt ? B.lmnt : 1;
  e = cudaMalloc(&P->dev, P->host.size() * sizeof(Phase));
  if (e == cudaSuccess)
    e = cudaMemcpy(P->dev, P->host.data(), P->host.size() * sizeof(Phase), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (P->dev) cudaFree(P->dev);
    delete P;
    return cuda_status(e, "program upload");
  }
  g_progs[key] = P;
  out = P;
  return LBX_OK;
}

static int launch_program(const Program *P, GridBar *gb, const ProgIo &io, cudaStream_t stream) {
  size_t dyn_max = 0;
  int nsm = 0;
  int rc = program_budget(dyn_max, nsm);
  if (rc) return rc;
  const size_t smem = P->w_bytes + P->s_bytes;
  LBX_CHECK_SUP(smem <= dyn_max, "program needs %zu bytes of shared memory (max %zu)", smem, dyn_max);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsm);
  cfg.blockDim = dim3(PTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, program_instance(P->ncb, P->lmnt), (const Phase *)P->dev,
                                           P->nph, gb, io, (int)P->s_bytes);
  return cuda_status(e, "program launch");
}

static GridBar *gridbar_of(void *lin_ws) {
  return reinterpret_cast<GridBar *>(reinterpret_cast<uint8_t *>(lin_ws) + WS_GRIDBAR);
}

}  // namespace lbx

// ---------------------------------------------------------------------------
// chain of LittleBit layers (x_{i+1} = layer_i(x_i)) as one program
// ---------------------------------------------------------------------------
extern "C" size_t lbx_linear_chain_workspace_size(const lbx_proj *projs, int32_t n_layers,
                                                  int32_t n_tokens) {
  size_t m = 0;
  if (!projs || n_layers < 1) return 0;
  for (int i = 0; i < n_layers; ++i) m = std::max(m, lbx_linear_workspace_size(projs + i, 1, n_tokens));
  return m;
}

extern "C" int lbx_linear_chain(const lbx_proj *projs, int32_t n_layers, int32_t n_tokens, int32_t dtype,
                                void *const *acts, void *ws, size_t ws_bytes, cudaStream_t stream) {
  using namespace lbx;
  LBX_CHECK_ARG(projs && acts && n_layers >= 1, "bad arguments");
  LBX_CHECK_ARG(dtype == LBX_F32 || dtype == LBX_BF16, "bad dtype");
  const size_t need = lbx_linear_chain_workspace_size(projs, n_layers, n_tokens);
  LBX_CHECK_ARG(ws && ws_bytes >= need, "workspace too small (%zu < %zu)", ws_bytes, need);
  uint64_t key = 0xC4A1Eull;
  key = mix(key, (uintptr_t)projs);
  key = mix(key, (uint64_t)n_layers);
  key = mix(key, (uint64_t)n_tokens);
  key = mix(key, (uint64_t)dtype);
  key = mix(key, (uintptr_t)ws);
  for (int i = 0; i <= n_layers; ++i) key = mix(key, (uintptr_t)acts[i]);
  for (int i = 0; i < n_layers; ++i)
    for (int b = 0; b < projs[i].n_branches; ++b) {
      key = mix(key, (uintptr_t)projs[i].br[b].v_sign);
      key = mix(key, (uintptr_t)projs[i].br[b].u_sign);
      key = mix(key, (uintptr_t)projs[i].br[b].u1);
    }
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
    for (int i = 0; i < n_layers; ++i) {
      lbx_linear_args a = {};
      a.n_proj = 1;
      a.n_tokens = n_tokens;
      a.x_dtype = a.y_dtype = dtype;
      a.x = acts[i];
      a.y[0] = acts[i + 1];
      rc = build_linear(B, projs + i, a, ws, budget);
      if (rc) return rc;
    }
    rc = finish_program(key, B, stream, P);
    if (rc) return rc;
  }
  ProgIo io = {};
  return launch_program(P, gridbar_of(ws), io, stream);
}
