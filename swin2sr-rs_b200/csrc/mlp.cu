// Fused MLP sublayer of a Swin2SR block (src/cpu.rs:1562-1573):
//     X <- X + LN2( fc2( GELU( fc1(X) ) ) )
// one persistent tcgen05 kernel. Per 128-token tile:
//   fc1   D1[128 x HP] = X16 * W1^T, in NP1 column parts of N1 (TMEM cols p*N1);
//   epi-1 bias + erf-GELU on each part, fp16, written straight into shared memory in
//         the 128-byte-swizzled K-major layout, where it is fc2's A operand: the
//         hidden activation never leaves the SM;
//   fc2   D2[128 x CP] = H * W2^T, on the LAST fc1 part's TMEM columns, so the next
//         tile's first fc1 parts can run while this tile's epilogue-2 drains D2;
//   epi-2 bias + LayerNorm over the real C columns + residual, fp32 X and fp16 X16
//         rewritten in place (image-order rows).
// The hidden tile's last K-chunks reuse the X16 tile's buffer (dead once fc1 has run),
// which is what makes a 180-wide model's tile fit: X16 48 KB, hidden 96 KB.
// Roles as in gemm_tc.cu: warp 0 TMA, warp 1 MMA + TMEM, warps 2..9 epilogue (two
// per TMEM lane quarter). All waits are bounded.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace s2s {
namespace {

constexpr int kMlpThreads = 320;
constexpr int kMlpEpiWarps = 8;
// Epilogue-2 tiles per warp: two fp32 32x32 tiles (residual in, result out, 128-byte
// swizzle) in a dedicated region, and two fp16 tiles (64-byte swizzle) placed in the
// hidden-head buffer, which is dead between fc2 and the next tile's epilogue 1.
constexpr int kMlpF32Buf = 2 * 4096;

template <int CP, int HP, int N1, int STAGES>
struct MlpCfg {
  static constexpr int KC1 = CP / 64;                 // K chunks of fc1 (= X16 tile chunks)
  static constexpr int KC2 = HP / 64;                 // K chunks of fc2 (= hidden chunks)
  static constexpr int NP1 = HP / N1;                 // fc1 column parts
  static constexpr int NH0 = KC2 - KC1;               // hidden chunks in the dedicated buffer
  static constexpr int D2OFF = (NP1 - 1) * N1;         // TMEM column of D2
  static constexpr int SLOT_ROWS = N1 > CP ? N1 : CP;
  static constexpr int SLOT = SLOT_ROWS * 128;        // ring slot bytes
  static constexpr uint32_t TCOLS = HP <= 32 ? 32 : HP <= 64 ? 64 : HP <= 128 ? 128 : HP <= 256 ? 256 : 512;
  static constexpr int H0B = NH0 * 16384 > kMlpEpiWarps * 4096 ? NH0 * 16384 : kMlpEpiWarps * 4096;
  static constexpr size_t SMEM = 1024 + (size_t)KC1 * 16384 + (size_t)H0B + (size_t)STAGES * SLOT +
                                 kMlpEpiWarps * kMlpF32Buf + (HP + 3 * CP) * 4 +
                                 (2 * STAGES + 2 * NP1 + 9 + 2 * kMlpEpiWarps) * 8 + 16;
};

template <int CP, int HP, int N1, int STAGES>
__global__ void __launch_bounds__(kMlpThreads, 1)
    k_mlp(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW1,
          const __grid_constant__ CUtensorMap mapW2, const __grid_constant__ CUtensorMap mapX32,
          const __grid_constant__ CUtensorMap mapX16o, const MlpArgs a) {
  using Cfg = MlpCfg<CP, HP, N1, STAGES>;
  constexpr int KC1 = Cfg::KC1, KC2 = Cfg::KC2, NP1 = Cfg::NP1, NH0 = Cfg::NH0;
  static_assert(NH0 >= 0, "hidden must be at least as wide as the embedding");
  static_assert((NH0 * 64) % N1 == 0 || NP1 == 1,
                "the hidden chunks placed in the X16 buffer must belong to the last fc1 part");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem;                           // KC1 chunks: X16 tile, then hidden tail
  uint8_t* sH0 = sX + KC1 * 16384;              // NH0 chunks: hidden head / epilogue-2 fp16 tiles
  uint8_t* ring = sH0 + Cfg::H0B;
  uint8_t* f32buf = ring + STAGES * Cfg::SLOT;  // [kMlpEpiWarps][2][4096]
  float* s_vec = reinterpret_cast<float*>(f32buf + kMlpEpiWarps * kMlpF32Buf);  // b1, b2, g2, beta2
  uint64_t* full = reinterpret_cast<uint64_t*>(s_vec + HP + 3 * CP);
  uint64_t* empty = full + STAGES;
  uint64_t* acc1 = empty + STAGES;   // [NP1] fc1 part ready
  uint64_t* hfull = acc1 + NP1;      // [NP1] hidden part written (8 warp arrivals)
  uint64_t* xfull = hfull + NP1;     // X16 tile landed
  uint64_t* xfree = xfull + 1;       // fc2 of the tile retired: X16 buffer reusable
  uint64_t* acc2 = xfree + 1;        // fc2 ready
  uint64_t* d2free = acc2 + 1;       // epilogue-2 drained D2 (8 warp arrivals)
  uint64_t* fin = d2free + 1;
  uint64_t* rbar = fin + 1;          // [kMlpEpiWarps][2] residual tile landed
  uint64_t* hfree = rbar + 2 * kMlpEpiWarps;  // epilogue-2 fp16 tiles read out (8 warp arrivals)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(hfree + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = (a.M + 127) / 128;
  auto hchunk = [&](int j) -> uint8_t* { return j < NH0 ? sH0 + j * 16384 : sX + (j - NH0) * 16384; };

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mapX);
    tma_prefetch_desc(&mapW1);
    tma_prefetch_desc(&mapW2);
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int p = 0; p < NP1; p++) {
      mbar_init(&acc1[p], 1);
      mbar_init(&hfull[p], kMlpEpiWarps);
    }
    mbar_init(xfull, 1);
    mbar_init(xfree, 1);
    mbar_init(acc2, 1);
    mbar_init(d2free, kMlpEpiWarps);
    mbar_init(fin, 1);
    for (int k = 0; k < 2 * kMlpEpiWarps; k++) mbar_init(&rbar[k], 1);
    mbar_init(hfree, kMlpEpiWarps);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      uint32_t kit = 0;
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
        if (i > 0 && !mbar_wait(xfree, (i - 1) & 1, DEV_TIMEOUT_EMPTY)) break;
        mbar_arrive_expect_tx(xfull, KC1 * 16384);
        for (int k = 0; k < KC1; k++) tma_load_2d(sX + k * 16384, &mapX, xfull, k * 64, t * 128);
        auto ring_load = [&](const CUtensorMap* m, int c0, int r0, int rows) -> bool {
          const int s = kit % STAGES;
          if (kit >= STAGES && !mbar_wait(&empty[s], ((kit / STAGES) - 1) & 1, DEV_TIMEOUT_EMPTY))
            return false;
          mbar_arrive_expect_tx(&full[s], rows * 128);
          tma_load_2d(ring + s * Cfg::SLOT, m, &full[s], c0, r0);
          kit++;
          return true;
        };
        for (int p = 0; p < NP1 && ok; p++)
          for (int k = 0; k < KC1 && ok; k++) ok = ring_load(&mapW1, k * 64, p * N1, N1);
        for (int k = 0; k < KC2 && ok; k++) ok = ring_load(&mapW2, k * 64, 0, CP);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t id1 = idesc_f16_f32(128, N1);
      constexpr uint32_t id2 = idesc_f16_f32(128, CP);
      uint32_t kit = 0;
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
        if (!mbar_wait(xfull, i & 1, DEV_TIMEOUT_FULL)) break;
        tc_fence_after();
        for (int p = 0; p < NP1 && ok; p++) {
          // the last part's columns hold the previous tile's D2 until epilogue-2 drains it
          if (p == NP1 - 1 && i > 0 && !mbar_wait(d2free, (i - 1) & 1, DEV_TIMEOUT_ACC)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int k = 0; k < KC1; k++, kit++) {
            const int s = kit % STAGES;
            if (!mbar_wait(&full[s], (kit / STAGES) & 1, DEV_TIMEOUT_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = sw128_desc(smem_u32(sX + k * 16384));
            const uint64_t bd = sw128_desc(smem_u32(ring + s * Cfg::SLOT));
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              tc_mma_f16(tmem + (uint32_t)(p * N1), ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2),
                         id1, (k | kk) != 0 ? 1u : 0u);
            tc_commit(&empty[s]);
          }
          tc_commit(&acc1[p]);
        }
        if (!ok) break;
        for (int p = 0; p < NP1 && ok; p++)
          if (!mbar_wait(&hfull[p], i & 1, DEV_TIMEOUT_ACC)) ok = false;
        if (!ok) break;
        tc_fence_after();
        for (int k = 0; k < KC2; k++, kit++) {
          const int s = kit % STAGES;
          if (!mbar_wait(&full[s], (kit / STAGES) & 1, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(hchunk(k)));
          const uint64_t bd = sw128_desc(smem_u32(ring + s * Cfg::SLOT));
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            tc_mma_f16(tmem + (uint32_t)Cfg::D2OFF, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2),
                       id2, (k | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        tc_commit(acc2);
        tc_commit(xfree);
      }
      tc_commit(fin);
      mbar_wait(fin, 0, DEV_TIMEOUT_ACC);
    }
  } else {
    // ---------------------------------------------------------------- epilogues
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int et = threadIdx.x - 64;
    const int r = q * 32 + lane;  // tile row of this thread in the thread-per-row phases
    for (int c = et; c < HP; c += 32 * kMlpEpiWarps) s_vec[c] = a.b1[c];
    for (int c = et; c < CP; c += 32 * kMlpEpiWarps) {
      s_vec[HP + c] = a.b2[c];
      s_vec[HP + CP + c] = a.g2[c];
      s_vec[HP + 2 * CP + c] = a.beta2[c];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(32 * kMlpEpiWarps) : "memory");
    const int wq = warp - 2;
    uint8_t* wf32 = f32buf + wq * kMlpF32Buf;
    uint8_t* wf16 = sH0 + wq * 4096;
    uint64_t* wrb = rbar + 2 * wq;
    uint32_t jcnt = 0;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
      const int row0 = t * 128 + q * 32;  // this warp's 32 rows as a TMA box origin
      // ---- epilogue 1: hidden = GELU(D1 + b1) -> fp16 -> shared (fc2's A operand)
      // the hidden-head buffer held the previous tile's epilogue-2 fp16 tiles
      if (i > 0 && !mbar_wait(hfree, (i - 1) & 1, DEV_TIMEOUT_ACC)) break;
      for (int p = 0; p < NP1; p++) {
        if (!mbar_wait(&acc1[p], i & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = half; c < N1 / 32; c += 2) {
          float v[32];
          tmem_ld32(tq + (uint32_t)(p * N1 + c * 32), v);
          const int col0 = p * N1 + c * 32;  // hidden column of v[0]
          uint32_t hv[16];
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const float4 bb = *reinterpret_cast<const float4*>(s_vec + col0 + 4 * j);
            const __half2 h0 = __floats2half2_rn(gelu_erf(v[4 * j] + bb.x), gelu_erf(v[4 * j + 1] + bb.y));
            const __half2 h1 = __floats2half2_rn(gelu_erf(v[4 * j + 2] + bb.z), gelu_erf(v[4 * j + 3] + bb.w));
            hv[2 * j] = *reinterpret_cast<const uint32_t*>(&h0);
            hv[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&h1);
          }
          uint8_t* chunk = hchunk(col0 >> 6);
          const int u0 = (col0 & 63) >> 3;  // first 16-byte unit in the 128-byte row
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int uu = (u0 + u) ^ (r & 7);
            *reinterpret_cast<uint4*>(chunk + r * 128 + uu * 16) =
                make_uint4(hv[4 * u], hv[4 * u + 1], hv[4 * u + 2], hv[4 * u + 3]);
          }
        }
        // generic-proxy writes -> visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&hfull[p]);
      }
      if (!ok) break;
      // ---- epilogue 2: X <- X + LN2(D2 + b2), X16 <- fp16(X), through TMA
      // the first residual tile is requested before waiting for fc2
      if (lane == 0 && half < CP / 32) {
        bulk_wait_read<0>();
        mbar_arrive_expect_tx(&wrb[jcnt & 1], 4096);
        tma_load_2d(wf32 + (jcnt & 1) * 4096, &mapX32, &wrb[jcnt & 1], half * 32, row0);
      }
      if (!mbar_wait(acc2, i & 1, DEV_TIMEOUT_ACC)) break;
      tc_fence_after();
      float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
      for (int c = 0; c < CP / 32; c++) {
        float v[32];
        tmem_ld32(tq + (uint32_t)(Cfg::D2OFF + c * 32), v);
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const float x = v[j] + s_vec[HP + c * 32 + j];
          s1 += x;
          s2 += x * x;
        }
      }
      const float nf = (float)a.ln_n;
      const float mean = s1 / nf;
      const float rstd = 1.0f / sqrtf(fmaxf(s2 / nf - mean * mean, 0.0f) + a.ln_eps);
      const float nmr = -mean * rstd;
      const int sw128 = lane & 7, sw64 = (lane >> 1) & 3;
#pragma unroll 1
      for (int c = half; c < CP / 32; c += 2, jcnt++) {
        const int jb = jcnt & 1;
        float* f32 = reinterpret_cast<float*>(wf32 + jb * 4096);
        uint8_t* f16 = wf16 + jb * 2048;
        float v[32];
        tmem_ld32(tq + (uint32_t)(Cfg::D2OFF + c * 32), v);
        if (lane == 0 && c + 2 < CP / 32) {
          bulk_wait_read<0>();
          mbar_arrive_expect_tx(&wrb[jb ^ 1], 4096);
          tma_load_2d(wf32 + (jb ^ 1) * 4096, &mapX32, &wrb[jb ^ 1], (c + 2) * 32, row0);
        }
        if (!mbar_wait(&wrb[jb], (jcnt >> 1) & 1, DEV_TIMEOUT_FULL)) {
          ok = false;
          break;
        }
        const int cl0 = c * 32;
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const float4 bb = *reinterpret_cast<const float4*>(s_vec + HP + cl0 + 4 * u);
          const float4 gg = *reinterpret_cast<const float4*>(s_vec + HP + CP + cl0 + 4 * u);
          const float4 be = *reinterpret_cast<const float4*>(s_vec + HP + 2 * CP + cl0 + 4 * u);
          float4* slot = reinterpret_cast<float4*>(f32 + lane * 32 + ((u ^ sw128) << 2));
          const float4 rr = *slot;
          float4 o;
          o.x = fmaf(fmaf(v[4 * u] + bb.x, rstd, nmr), gg.x, be.x) + rr.x;
          o.y = fmaf(fmaf(v[4 * u + 1] + bb.y, rstd, nmr), gg.y, be.y) + rr.y;
          o.z = fmaf(fmaf(v[4 * u + 2] + bb.z, rstd, nmr), gg.z, be.z) + rr.z;
          o.w = fmaf(fmaf(v[4 * u + 3] + bb.w, rstd, nmr), gg.w, be.w) + rr.w;
          *slot = o;
          v[4 * u] = o.x;
          v[4 * u + 1] = o.y;
          v[4 * u + 2] = o.z;
          v[4 * u + 3] = o.w;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
          __half2 h0 = __floats2half2_rn(v[8 * u], v[8 * u + 1]);
          __half2 h1 = __floats2half2_rn(v[8 * u + 2], v[8 * u + 3]);
          __half2 h2 = __floats2half2_rn(v[8 * u + 4], v[8 * u + 5]);
          __half2 h3 = __floats2half2_rn(v[8 * u + 6], v[8 * u + 7]);
          *reinterpret_cast<uint4*>(f16 + lane * 64 + ((u ^ sw64) << 4)) =
              make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                         *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&mapX32, f32, cl0, row0);
          tma_store_2d(&mapX16o, f16, cl0, row0);
          bulk_commit();
        }
      }
      if (!ok) break;
      // the fp16 tiles live in the hidden-head buffer: every warp's stores must have
      // read them before the next tile's epilogue 1 writes there
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(d2free);
        mbar_arrive(hfree);
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TCOLS);
  }
}

template <int CP, int HP, int N1, int STAGES>
cudaError_t launch_mlp_t(const CUtensorMap& mX, const CUtensorMap& mW1, const CUtensorMap& mW2,
                         const CUtensorMap& mX32, const CUtensorMap& mX16o, const MlpArgs& a,
                         cudaStream_t st) {
  using Cfg = MlpCfg<CP, HP, N1, STAGES>;
  static int ctas = 0;
  if (ctas == 0) {
    cudaError_t err = cudaFuncSetAttribute(k_mlp<CP, HP, N1, STAGES>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)Cfg::SMEM);
    if (err != cudaSuccess) return err;
    int dev = 0, sms = 0, occ = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_mlp<CP, HP, N1, STAGES>,
                                                        kMlpThreads, Cfg::SMEM);
    if (err != cudaSuccess) return err;
    if (occ < 1) return cudaErrorInvalidConfiguration;
    ctas = sms * occ;
  }
  const int tiles = (a.M + 127) / 128;
  const int G = tiles < ctas ? tiles : ctas;
  k_mlp<CP, HP, N1, STAGES><<<G, kMlpThreads, Cfg::SMEM, st>>>(mX, mW1, mW2, mX32, mX16o, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_mlp(const CUtensorMap& mX, const CUtensorMap& mW1, const CUtensorMap& mW2,
                       const CUtensorMap& mX32, const CUtensorMap& mX16o, const MlpArgs& a, int cp,
                       int hp, cudaStream_t st) {
  if (cp == 192 && hp == 384)
    return launch_mlp_t<192, 384, 192, 2>(mX, mW1, mW2, mX32, mX16o, a, st);
  if (cp == 64 && hp == 128)
    return launch_mlp_t<64, 128, 128, 4>(mX, mW1, mW2, mX32, mX16o, a, st);
  return cudaErrorNotSupported;
}

}  // namespace s2s
