// Shared device/host helpers for the sm_100a LittleBit kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>
#include <string>

#include "../../include/lbx.h"

#define LBX_DEV __device__ __forceinline__

namespace lbx {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

#define LBX_CHECK_ARG(cond, ...)                                                    \
  do {                                                                              \
    if (!(cond)) {                                                                  \
      ::lbx::set_error(__VA_ARGS__);                                                \
      return LBX_EINVAL;                                                            \
    }                                                                               \
  } while (0)

#define LBX_CHECK_SUP(cond, ...)                                                    \
  do {                                                                              \
    if (!(cond)) {                                                                  \
      ::lbx::set_error(__VA_ARGS__);                                                \
      return LBX_EUNSUPPORTED;                                                      \
    }                                                                               \
  } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// per-device set-up values
// ---------------------------------------------------------------------------
// Kernel attributes (cudaFuncSetAttribute) and device properties belong to one
// device.  Values established on the first call are therefore cached per
// device, so a process that drives several GPUs sets each of them up on its
// first call there.  One recursive mutex guards every cache (an initialiser
// may read another cache).  Devices beyond the table are set up on every call.
constexpr int LBX_MAX_DEVICES = 64;
inline std::recursive_mutex &dev_cache_mu() {
  static std::recursive_mutex m;
  return m;
}
inline int cur_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) d = -1;
  return d;
}
template <typename T>
struct DevCache {
  T v[LBX_MAX_DEVICES] = {};
  bool ok[LBX_MAX_DEVICES] = {};
  // init(T &) returns an LBX status; its value is kept only when it succeeds
  template <typename F>
  int get(T &out, F &&init) {
    const int d = cur_device();
    const bool slot = d >= 0 && d < LBX_MAX_DEVICES;
    std::lock_guard<std::recursive_mutex> lk(dev_cache_mu());
    if (slot && ok[d]) {
      out = v[d];
      return LBX_OK;
    }
    T t{};
    const int rc = init(t);
    if (rc) return rc;
    if (slot) {
      v[d] = t;
      ok[d] = true;
    }
    out = t;
    return LBX_OK;
  }
};

// multiprocessors of the current device (148 if the query fails)
inline int device_sm_count() {
  static DevCache<int> c;
  int n = 148;
  c.get(n, [](int &v) {
    int dev = cur_device();
    if (dev < 0 || cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    return LBX_OK;
  });
  return n;
}

// Device error word: bounded waits that run out record a code here and the
// kernel returns instead of spinning forever.  The library is one translation
// unit (lbx_all.cu), so this is the single definition.
__device__ int g_lbx_device_error = 0;

// Allow a kernel the largest dynamic shared memory the device grants a block
// (opt-in limit minus the kernel's static shared memory).  Returns that size.
template <typename Kern>
cudaError_t allow_max_smem(Kern k, size_t *granted = nullptr) {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa;
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, k);
  if (e != cudaSuccess) return e;
  const int dyn = optin - (int)fa.sharedSizeBytes;
  if (granted) *granted = (size_t)dyn;
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
}

// Phase probes: no-ops in the library build.  A profiling build may define
// LBX_PROBE(id) to record a timestamp at each phase boundary of a kernel.
#ifndef LBX_PROBE
#define LBX_PROBE(id) ((void)0)
#endif

// Launch with optional programmatic dependent launch (PDL).
template <typename Kern, typename... Args>
cudaError_t launch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
LBX_DEV uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch: wait for the preceding grid (and its memory)
// and let the following grid start its prologue early.
LBX_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LBX_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

LBX_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
LBX_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
LBX_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

LBX_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bulk (non-tensor) async copy global -> shared, completion on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16.
LBX_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

LBX_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in the
// device error word) if the phase did not complete within the limit.
LBX_DEV bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int code) {
  // try_wait suspends for a hardware-defined interval per attempt; 1<<22
  // attempts is far beyond any legitimate copy latency.
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  atomicCAS(&g_lbx_device_error, 0, code);
  return false;
}

// Four sign bits (bit j, j+4, j+8, j+12 of sel) -> four int8 lanes of
// 0 (bit 0, sign +1) or -1 (bit 1, sign -1).  prmt picks byte (nibble & 7)
// of the table {0x00,0xFF,0x00,0xFF,...}: odd selectors give 0xFF.  In the
// sign-replicate mode (nibble bit 3) the chosen byte's msb is replicated,
// which yields the same byte, so only nibble bit 0 matters.
LBX_DEV uint32_t negbits4(uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %1, %2;" : "=r"(r) : "r"(0xFF00FF00u), "r"(sel));
  return r;
}

// The same expansion with fewer shifts: a byte table indexed by the selector
// nibble's bits 2..0 can key on any one of those bits (bit 0:
// {00,FF,00,FF,..}, bit 1: {00,00,FF,FF,..}, bit 2: {00,00,00,00,FF,FF,FF,FF}),
// and prmt reads only the selector's low 16 bits, so one sign word needs only
// the shifted copies w>>1, w>>16 and w>>17.
LBX_DEV uint32_t prmt_tab(uint32_t lo, uint32_t hi, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(lo), "r"(hi), "r"(sel));
  return r;
}
// k-step R (0..3) of a 4-word group: lo holds the bytes of bits sh+4j, hi those
// of bits sh+1+4j (sh = 16*(R>>1) + 2*(R&1)), i.e. exactly negbits4(w >> sh)
// and negbits4(w >> (sh+1))
template <int R>
LBX_DEV void sign_frag(uint32_t w, uint32_t &lo, uint32_t &hi) {
  constexpr uint32_t B0 = 0xFF00FF00u, B1 = 0xFFFF0000u;
  if constexpr (R == 0) {
    lo = prmt_tab(B0, B0, w);
    hi = prmt_tab(B1, B1, w);
  } else if constexpr (R == 1) {
    lo = prmt_tab(0u, ~0u, w);
    hi = prmt_tab(0u, ~0u, w >> 1);
  } else if constexpr (R == 2) {
    lo = prmt_tab(B0, B0, w >> 16);
    hi = prmt_tab(B1, B1, w >> 16);
  } else {
    lo = prmt_tab(0u, ~0u, w >> 16);
    hi = prmt_tab(0u, ~0u, w >> 17);
  }
}

// D(16x8,s32) += A(16x32,s8) * B(32x8,s8)
LBX_DEV void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                    uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

LBX_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
LBX_DEV int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
LBX_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

LBX_DEV float bf16_to_f32(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }
LBX_DEV uint16_t f32_to_bf16(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t *>(&b);
}

LBX_DEV float load_act(const void *p, int dtype, int64_t i) {
  return dtype == LBX_F32 ? __ldg(reinterpret_cast<const float *>(p) + i)
                          : bf16_to_f32(__ldg(reinterpret_cast<const uint16_t *>(p) + i));
}

// 16-bit activation quantisation as two signed int8 digits q = 256*hi + lo,
// |q| <= QMAX so that hi stays within [-127, 127].
constexpr float QMAX = 32639.0f;

LBX_DEV void split_digits(int q, int &hi, int &lo) {
  lo = ((q + 128) & 255) - 128;
  hi = (q - lo) >> 8;
}

}  // namespace lbx
