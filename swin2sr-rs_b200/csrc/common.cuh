// Device-side building blocks shared by the sm_100a kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA, commit, loads),
// and the library-wide device error word.
//
// Every wait here is bounded. A wait that exceeds its budget records an error
// code in g_s2s_err and returns false, so a kernel can unwind (skip its work,
// free its TMEM) instead of spinning forever; the host reads the word after the
// stream synchronises and turns it into S2S_ERR_TIMEOUT.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

namespace s2s {

// ---------------------------------------------------------------- dependent launch
// Every kernel of the library is launched with programmatic stream serialization:
// it signals at its start that the next kernel of the stream may be scheduled
// (pdl_trigger), and waits for the previous kernel to complete and its writes to be
// visible (pdl_wait) after its prologue - barrier setup, TMEM allocation, tensor-map
// prefetch, constant loads - and before touching any activation in global memory.
// So each kernel's prologue overlaps the tail of the one before it. S2S_PDL=0 turns
// the attribute off (plain stream order).
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("S2S_PDL");
    return !(v && strcmp(v, "0") == 0);
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Launch set-up of one kernel, per device: its dynamic shared-memory limit is raised
// and the CTAs that fit on the device at once are counted the first time the kernel
// is launched on that device (with it current); later launches read the count.
// Thread-safe: handles on several devices may launch from several host threads.
constexpr int kMaxDevices = 64;
struct LaunchSetup {
  std::mutex mu;
  std::atomic<int> ctas[kMaxDevices] = {};
};

template <typename Kern>
cudaError_t resident_ctas(LaunchSetup& ls, Kern kernel, int threads, size_t smem, int* ctas) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int n = ls.ctas[dev].load(std::memory_order_acquire);
  if (n == 0) {
    std::lock_guard<std::mutex> lock(ls.mu);
    n = ls.ctas[dev].load(std::memory_order_relaxed);
    if (n == 0) {
      err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      int sms = 0, occ = 0;
      err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (err != cudaSuccess) return err;
      err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem);
      if (err != cudaSuccess) return err;
      if (occ < 1) return cudaErrorInvalidConfiguration;
      n = sms * occ;
      ls.ctas[dev].store(n, std::memory_order_release);
    }
  }
  *ctas = n;
  return cudaSuccess;
}

// Error codes recorded on the device (first error wins).
enum : unsigned { DEV_OK = 0, DEV_TIMEOUT_FULL = 1, DEV_TIMEOUT_EMPTY = 2, DEV_TIMEOUT_ACC = 3,
                  DEV_BAD_SHAPE = 4, DEV_TIMEOUT_HALO = 5 };

// Defined once: the library is a single translation unit (s2s.cu).
__device__ unsigned int g_s2s_err = 0;

__device__ __forceinline__ void record_error(unsigned code) { atomicCAS(&g_s2s_err, 0u, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}

// Non-blocking test: has the phase with parity `phase` completed? (Only meaningful
// when the caller knows the barrier is at most one phase ahead of that one.)
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Wait for the barrier's phase `phase` to complete, for at most ~2 s of wall time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, unsigned code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, phase)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(a, phase)) return true;
    if ((it & 255u) == 255u) {
      if (global_timer_ns() - t0 > 2000000000ull) {
        record_error(code);
        return false;
      }
      // Another block already gave up: do not wait out a full budget of our own.
      if (*(volatile unsigned*)&g_s2s_err != 0u) return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// Bulk tensor stores (shared -> global) tracked by per-thread bulk async-groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N committed groups are still in flight (writes performed).
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later async-proxy
// (TMA / tensor core) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- attention helpers
// 2^x by the SFU: PTX ex2.approx (the attention logits are pre-scaled by log2 e).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shift-mask region of rolled-plane coordinate a along an axis of p pixels
// (src/plan.rs:80-108): 0 before the last window, 1 in it before the shift, 2 after.
__device__ __forceinline__ int region_of(int a, int p, int win, int shift) {
  return (a + win < p) ? 0 : (a + shift < p) ? 1 : 2;
}

// One bulk copy global -> shared (16-byte aligned, a multiple of 16 bytes),
// completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- GELU
// erf-form GELU, 0.5 x (1 + erf(x / sqrt 2)) (nn.GELU's default; the reference's
// src/cpu.rs:1125-1132), with erf from Abramowitz & Stegun (1964), formula 7.1.28:
//   erf(t) = 1 - (1 + a1 t + ... + a6 t^6)^-16,  t >= 0,  |error| <= 3e-7,
// odd-extended. Branch-free: GELU = x - 0.5 x r for x >= 0 and 0.5 x r otherwise,
// r = (1 + ...)^-16 = erfc(|x| / sqrt 2). Against the exact function it is within
// 7e-7 absolute on [-12, 12] in fp32 (tests/test_host.py), well below the fp16
// rounding of the hidden activations it feeds.
__device__ __forceinline__ float gelu_erf(float x) {
  const float t = fabsf(x) * 0.70710678118654752440f;
  float p = 0.0000430638f;
  p = fmaf(p, t, 0.0002765672f);
  p = fmaf(p, t, 0.0001520143f);
  p = fmaf(p, t, 0.0092705272f);
  p = fmaf(p, t, 0.0422820123f);
  p = fmaf(p, t, 0.0705230784f);
  p = fmaf(p, t, 1.0f);
  p = p * p;
  p = p * p;
  p = p * p;
  p = p * p;
  float r;  // hardware reciprocal (about 1 ulp); inf -> 0 for large |x|
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(p));
  const float h = 0.5f * x * r;
  return x >= 0.0f ? x - h : h;
}

// Packed two-lane fp32 arithmetic of sm_100 (add/mul/fma .f32x2): the same IEEE
// operations as the scalar forms, one instruction for two values.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// gelu_erf of (x0 + b0, x1 + b1): the bias add and the polynomial in packed form,
// each operation and its order as in gelu_erf, the tail in gelu_erf's own scalar
// expression.
__device__ __forceinline__ float2 gelu_erf2(float x0, float x1, float b0, float b1) {
  const float2 xs = f2_unpack(f2_add(f2_pack(x0, x1), f2_pack(b0, b1)));
  const unsigned long long t =
      f2_mul(f2_pack(fabsf(xs.x), fabsf(xs.y)),
             f2_pack(0.70710678118654752440f, 0.70710678118654752440f));
  unsigned long long p = f2_pack(0.0000430638f, 0.0000430638f);
  p = f2_fma(p, t, f2_pack(0.0002765672f, 0.0002765672f));
  p = f2_fma(p, t, f2_pack(0.0001520143f, 0.0001520143f));
  p = f2_fma(p, t, f2_pack(0.0092705272f, 0.0092705272f));
  p = f2_fma(p, t, f2_pack(0.0422820123f, 0.0422820123f));
  p = f2_fma(p, t, f2_pack(0.0705230784f, 0.0705230784f));
  p = f2_fma(p, t, f2_pack(1.0f, 1.0f));
  p = f2_mul(p, p);
  p = f2_mul(p, p);
  p = f2_mul(p, p);
  p = f2_mul(p, p);
  const float2 pp = f2_unpack(p);
  float r0, r1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(pp.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(pp.y));
  const float h0 = 0.5f * xs.x * r0, h1 = 0.5f * xs.y * r1;
  return make_float2(xs.x >= 0.0f ? xs.x - h0 : h0, xs.y >= 0.0f ? xs.y - h1 : h1);
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives row
// (lane base + i), columns col..col+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// The same load without the wait: issue several, then tc_wait_ld() once.
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major tile in the 128-byte swizzle
// layout: rows of 64 fp16 (128 B), 8-row groups 1024 B apart. The tile base must
// be 1024-byte aligned; advancing along K inside the 128-byte row is done by
// adding the byte offset to the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1u << 16;                  // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;        // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1u << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                  // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: kind::f16, A = B = fp16, D = fp32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace s2s
