// Fused MLP sublayer of a Swin2SR block (src/cpu.rs:1562-1573):
//     X <- X + LN2( fc2( GELU( fc1(X) ) ) )
// one persistent tcgen05 kernel over 128-token tiles. The hidden dimension is
// walked in 64-column parts j = 0 .. NP-1:
//   fc1 part j   D1[j % 2] (64 TMEM columns) = X16 tile * W1[64j : 64j+64]^T
//   epi-1 part j bias + erf-GELU, fp16, back into D1[j % 2] in TMEM over the columns
//                each warp has read (two fp16 per 32-bit column: fc2's A operand)
//   fc2 chunk j  D2[tile % 2] += hidden chunk j (A from TMEM) * W2[:, 64j : 64j+64]^T
// and once all parts are in, epilogue 2 applies bias, LayerNorm over the real C
// columns and the residual, and rewrites fp32 X and fp16 X16 in place by TMA stores.
// The MMA warp issues fc1 part j+2 right after fc2 chunk j, so the tensor core always
// has the next part queued while the epilogue warps run GELU, and with two D2
// accumulators the next tile's parts start while this tile's epilogue 2 drains.
// The hidden activation never leaves the SM. Warp roles: warp 0 TMA, warp 1 MMA +
// TMEM, warps 2..9 epilogue 1 (GELU), warps 10..17 epilogue 2 (LayerNorm +
// residual) - the two epilogue groups work on consecutive tiles at the same time,
// two warps per TMEM lane quarter each. All waits are bounded.
//
// PROJ: the attention sublayer's proj, norm1 and residual run first in the same
// kernel (src/cpu.rs:1549-1559): the tile loaded is the attention output AO,
//   proj         D2[tile % 2] = AO tile * Wproj^T
//   epilogue P   x1 = X + LN1(D2 + bp): fp32 to X (TMA store, read back as epilogue
//                2's residual), fp16 into the tile buffer in shared memory, where it
//                is fc1's A operand
// so the block's residual stream crosses HBM once fewer each way and the proj kernel
// disappears. The LayerNorm group runs epilogue P of tile i before epilogue 2 of
// tile i - 1; the two use different D2 buffers.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace s2s {
namespace {

constexpr int kMlpThreads = 576;
constexpr int kMlpEpiWarps = 8;  // per epilogue group
constexpr int kMlpPart = 64;  // hidden columns per part

// D(tmem) (+)= A(tmem) * B(smem desc)^T, fp16 inputs, fp32 accumulate. A (M = 128 rows,
// K-major) sits in TMEM as the rows' lanes, two fp16 K elements per 32-bit column.
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from this warp's registers into TMEM, and
// the wait for the store to complete.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

template <int CP, int HP, int STAGES>
struct MlpCfg {
  static constexpr int KC1 = CP / 64;                  // K chunks of fc1 (= X16 tile chunks)
  static constexpr int NP = HP / kMlpPart;             // hidden parts (= fc2 K chunks)
  static constexpr int D2OFF = 2 * kMlpPart;           // D2 buffers after the two D1 buffers
  static constexpr int TUSED = D2OFF + 2 * CP;
  static constexpr uint32_t TCOLS = TUSED <= 128 ? 128 : TUSED <= 256 ? 256 : 512;
  // a ring slot holds one fc1 part's weights (KC1 boxes of 64 x 64), one fc2 chunk or
  // one proj K-chunk (CP rows x 64)
  static constexpr int SLOT = KC1 * 8192 > CP * 128 ? KC1 * 8192 : CP * 128;
  // epilogue 2 per warp: two fp32 32x32 tiles (residual in / result out, 128-byte
  // swizzle) and one fp16 tile (64-byte swizzle)
  static constexpr int STG = 2 * 4096 + 2048;
  static constexpr size_t SMEM = 1024 + (size_t)KC1 * 16384 +
                                 (size_t)STAGES * SLOT + (size_t)kMlpEpiWarps * STG +
                                 (HP + 6 * CP) * 4 + (2 * STAGES + 16 + 2 * kMlpEpiWarps) * 8 +
                                 16;
};

template <int CP, int HP, int STAGES, bool PROJ>
__global__ void __launch_bounds__(kMlpThreads, 1)
    k_mlp(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW1,
          const __grid_constant__ CUtensorMap mapW2, const __grid_constant__ CUtensorMap mapX32,
          const __grid_constant__ CUtensorMap mapX16o, const __grid_constant__ CUtensorMap mapWp,
          const MlpArgs a) {
  using Cfg = MlpCfg<CP, HP, STAGES>;
  constexpr int KC1 = Cfg::KC1, NP = Cfg::NP;
  static_assert(HP % kMlpPart == 0 && CP % 64 == 0 && NP % 2 == 0, "tile shapes");
  static_assert(Cfg::TUSED <= 512, "TMEM columns");
  static_assert(Cfg::SMEM <= 232448, "shared memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem;                           // KC1 chunks: the X16 (PROJ: AO, then x1) tile
  uint8_t* ring = sX + KC1 * 16384;
  uint8_t* stgbuf = ring + STAGES * Cfg::SLOT;  // [kMlpEpiWarps][STG] epilogue staging
  // b1, b2, g2, beta2, bp, g1, beta1
  float* s_vec = reinterpret_cast<float*>(stgbuf + kMlpEpiWarps * Cfg::STG);
  uint64_t* full = reinterpret_cast<uint64_t*>(s_vec + HP + 6 * CP);
  uint64_t* empty = full + STAGES;
  uint64_t* acc1 = empty + STAGES;   // [2] fc1 part in D1 buffer b
  uint64_t* hfull = acc1 + 2;        // [2] fp16 hidden chunk in D1 buffer b (8 warp arrivals)
  uint64_t* acc2 = hfull + 2;        // [2] D2 buffer d complete
  uint64_t* d2free = acc2 + 2;       // [2] D2 buffer d drained (8 warp arrivals)
  uint64_t* xfull = d2free + 2;      // X16 (AO) tile landed
  uint64_t* xfree = xfull + 1;       // fc1 of the tile retired: tile buffer reusable
  uint64_t* fin = xfree + 2;
  uint64_t* accp = fin + 1;          // [2] PROJ: proj result in D2 buffer d
  uint64_t* x1ready = accp + 2;      // PROJ: x1 (fp16) in the tile buffer (8 warp arrivals)
  uint64_t* rbar = x1ready + 1;      // [kMlpEpiWarps][2] residual tile landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(rbar + 2 * kMlpEpiWarps);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = (a.M + 127) / 128;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mapX);
    tma_prefetch_desc(&mapW1);
    tma_prefetch_desc(&mapW2);
    tma_prefetch_desc(&mapX32);
    tma_prefetch_desc(&mapX16o);
    if (PROJ) tma_prefetch_desc(&mapWp);
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc1[b], 1);
      mbar_init(&hfull[b], kMlpEpiWarps);
      mbar_init(&acc2[b], 1);
      mbar_init(&d2free[b], kMlpEpiWarps);
      mbar_init(&accp[b], 1);
    }
    mbar_init(xfull, 1);
    mbar_init(xfree, 1);
    mbar_init(fin, 1);
    mbar_init(x1ready, kMlpEpiWarps);
    for (int k = 0; k < 2 * kMlpEpiWarps; k++) mbar_init(&rbar[k], 1);
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
  pdl_trigger();
  pdl_wait();  // the previous kernel's outputs (X, X16 or AO) are complete

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      // Ring order = MMA order: (PROJ: Wproj chunks 0..KC1-1,) W1 part 0, W1 part 1,
      // then per part j: W2 chunk j and (j + 2 < NP) W1 part j+2. The next tile's
      // X16 / AO follows its xfree.
      uint32_t kit = 0;
      bool ok = true;
      auto slot_wait = [&]() -> int {
        const int s = kit % STAGES;
        if (kit >= STAGES && !mbar_wait(&empty[s], ((kit / STAGES) - 1) & 1, DEV_TIMEOUT_EMPTY))
          return -1;
        return s;
      };
      auto load_wp = [&](int c) -> bool {
        const int s = slot_wait();
        if (s < 0) return false;
        mbar_arrive_expect_tx(&full[s], CP * 128);
        tma_load_2d(ring + s * Cfg::SLOT, &mapWp, &full[s], c * 64, 0);
        kit++;
        return true;
      };
      auto load_w1 = [&](int j) -> bool {
        const int s = slot_wait();
        if (s < 0) return false;
        mbar_arrive_expect_tx(&full[s], KC1 * 8192);
        for (int k = 0; k < KC1; k++)
          tma_load_2d(ring + s * Cfg::SLOT + k * 8192, &mapW1, &full[s], k * 64, j * kMlpPart);
        kit++;
        return true;
      };
      auto load_w2 = [&](int j) -> bool {
        const int s = slot_wait();
        if (s < 0) return false;
        mbar_arrive_expect_tx(&full[s], CP * 128);
        tma_load_2d(ring + s * Cfg::SLOT, &mapW2, &full[s], j * kMlpPart, 0);
        kit++;
        return true;
      };
      auto load_x = [&](int t) {
        mbar_arrive_expect_tx(xfull, KC1 * 16384);
        for (int k = 0; k < KC1; k++) tma_load_2d(sX + k * 16384, &mapX, xfull, k * 64, t * 128);
      };
      if ((int)blockIdx.x < num_tiles) load_x(blockIdx.x);
      int i = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
        if constexpr (PROJ) {
          for (int c = 0; c < KC1 && ok; c++) ok = load_wp(c);
        }
        ok = ok && load_w1(0) && load_w1(1);
        for (int j = 0; j < NP && ok; j++) {
          ok = load_w2(j);
          if (ok && j + 2 < NP) ok = load_w1(j + 2);
        }
        if (!ok) break;
        if (t + (int)gridDim.x < num_tiles) {
          if (!mbar_wait(xfree, i & 1, DEV_TIMEOUT_EMPTY)) break;
          load_x(t + gridDim.x);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t id1 = idesc_f16_f32(128, kMlpPart);
      constexpr uint32_t id2 = idesc_f16_f32(128, CP);
      uint32_t kit = 0;
      int i = 0;
      bool ok = true;
      auto slot_full = [&]() -> int {
        const int s = kit % STAGES;
        if (!mbar_wait(&full[s], (kit / STAGES) & 1, DEV_TIMEOUT_FULL)) return -1;
        tc_fence_after();
        return s;
      };
      auto fc1 = [&](int j) -> bool {
        const int s = slot_full();
        if (s < 0) return false;
        const uint32_t d = tmem + (uint32_t)((j & 1) * kMlpPart);
#pragma unroll
        for (int k = 0; k < KC1; k++) {
          const uint64_t ad = sw128_desc(smem_u32(sX + k * 16384));
          const uint64_t bd = sw128_desc(smem_u32(ring + s * Cfg::SLOT + k * 8192));
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            tc_mma_f16(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), id1,
                       (k | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
        tc_commit(&acc1[j & 1]);
        if (j == NP - 1) tc_commit(xfree);
        kit++;
        return true;
      };
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
        if (!mbar_wait(xfull, i & 1, DEV_TIMEOUT_FULL)) break;
        tc_fence_after();
        const int db = i & 1;
        const uint32_t d2 = tmem + (uint32_t)(Cfg::D2OFF + db * CP);
        if constexpr (PROJ) {
          // D2 buffer db held tile i-2 until its epilogue 2 drained it
          if (i >= 2 && !mbar_wait(&d2free[db], (uint32_t)(((i >> 1) - 1) & 1), DEV_TIMEOUT_ACC))
            break;
          tc_fence_after();
          for (int c = 0; c < KC1 && ok; c++) {
            const int s = slot_full();
            if (s < 0) {
              ok = false;
              break;
            }
            const uint64_t ad = sw128_desc(smem_u32(sX + c * 16384));
            const uint64_t bd = sw128_desc(smem_u32(ring + s * Cfg::SLOT));
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              tc_mma_f16(d2, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), id2,
                         (c | kk) != 0 ? 1u : 0u);
            tc_commit(&empty[s]);
            kit++;
          }
          if (!ok) break;
          tc_commit(&accp[db]);
          // x1 (fp16) replaced AO in the tile buffer, and D2 buffer db is drained
          if (!mbar_wait(x1ready, i & 1, DEV_TIMEOUT_ACC)) break;
          tc_fence_after();
        }
        ok = fc1(0) && fc1(1);
        for (int j = 0; j < NP && ok; j++) {
          // hidden chunk j (fp16, in D1 buffer j % 2) written by epilogue 1
          if (!mbar_wait(&hfull[j & 1], (uint32_t)((i * (NP / 2) + (j >> 1)) & 1), DEV_TIMEOUT_ACC)) {
            ok = false;
            break;
          }
          // D2 buffer db held tile i-2 until its epilogue 2 drained it
          if (!PROJ && j == 0 && i >= 2 &&
              !mbar_wait(&d2free[db], (uint32_t)(((i >> 1) - 1) & 1), DEV_TIMEOUT_ACC)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int s = slot_full();
          if (s < 0) {
            ok = false;
            break;
          }
          // hidden chunk j: K 0-31 at D1 columns 0-15, K 32-63 at columns 32-47 of
          // buffer j % 2; a K = 16 step takes 8 columns
          const uint32_t ha = tmem + (uint32_t)((j & 1) * kMlpPart);
          const uint64_t bd = sw128_desc(smem_u32(ring + s * Cfg::SLOT));
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            tc_mma_f16_ta(d2, ha + (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8),
                          bd + (uint64_t)(kk * 2), id2, (j | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
          kit++;
          if (j + 2 < NP) ok = fc1(j + 2);
        }
        if (!ok) break;
        tc_commit(&acc2[db]);
      }
      tc_commit(fin);
      mbar_wait(fin, 0, DEV_TIMEOUT_ACC);
    }
  } else {
    // ---------------------------------------------------------------- epilogues
    const bool gelu_group = warp < 2 + kMlpEpiWarps;
    const int gw = gelu_group ? warp - 2 : warp - 2 - kMlpEpiWarps;  // warp within its group
    const int q = warp & 3;            // TMEM lane quarter
    const int half = gw >> 2;          // which half of the columns
    const int et = threadIdx.x - 64;
    const int r = q * 32 + lane;       // tile row of this thread
    for (int c = et; c < HP; c += 64 * kMlpEpiWarps) s_vec[c] = a.b1[c];
    for (int c = et; c < CP; c += 64 * kMlpEpiWarps) {
      s_vec[HP + c] = a.b2[c];
      s_vec[HP + CP + c] = a.g2[c];
      s_vec[HP + 2 * CP + c] = a.beta2[c];
      if (PROJ) {
        s_vec[HP + 3 * CP + c] = a.bp[c];
        s_vec[HP + 4 * CP + c] = a.g1[c];
        s_vec[HP + 5 * CP + c] = a.beta1[c];
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(64 * kMlpEpiWarps) : "memory");
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    if (gelu_group) {
      // ---- epilogue 1: hidden chunk j = GELU(D1 + b1) -> fp16 -> back into D1 (TMEM)
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
        for (int j = 0; j < NP; j++) {
          const uint32_t ph = (uint32_t)((i * (NP / 2) + (j >> 1)) & 1);
          if (!mbar_wait(&acc1[j & 1], ph, DEV_TIMEOUT_ACC)) {
            ok = false;
            break;
          }
          tc_fence_after();
          float v[32];
          tmem_ld32(tq + (uint32_t)((j & 1) * kMlpPart + half * 32), v);
          const int col0 = j * kMlpPart + half * 32;  // hidden column of v[0]
          uint32_t hv[16];
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const float4 bb = *reinterpret_cast<const float4*>(s_vec + col0 + 4 * u);
            const float2 g0 = gelu_erf2(v[4 * u], v[4 * u + 1], bb.x, bb.y);
            const float2 g1 = gelu_erf2(v[4 * u + 2], v[4 * u + 3], bb.z, bb.w);
            const __half2 h0 = __floats2half2_rn(g0.x, g0.y);
            const __half2 h1 = __floats2half2_rn(g1.x, g1.y);
            hv[2 * u] = *reinterpret_cast<const uint32_t*>(&h0);
            hv[2 * u + 1] = *reinterpret_cast<const uint32_t*>(&h1);
          }
          // the fp16 hidden values go back into TMEM over this warp's own (already read)
          // fp32 columns: hidden column 32 * half + 2c + e at D1 column 32 * half + c,
          // half e - fc2's A operand
          tmem_st16(tq + (uint32_t)((j & 1) * kMlpPart + half * 32), hv);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&hfull[j & 1]);
        }
      }
    } else {
      // ---- the LayerNorm group: epilogue P (PROJ) and epilogue 2
      uint8_t* wf32 = stgbuf + gw * Cfg::STG;
      uint8_t* f16 = wf32 + 2 * 4096;
      uint64_t* wrb = rbar + 2 * gw;
      const int sw128 = lane & 7, sw64 = (lane >> 1) & 3;  // this row's swizzle phases
      uint32_t jcnt = 0;
      // request residual chunk c of this warp's 32 rows into staging buffer jb
      auto res_load = [&](int jb, int c, int row0) {
        mbar_arrive_expect_tx(&wrb[jb], 4096);
        tma_load_2d(wf32 + jb * 4096, &mapX32, &wrb[jb], c * 32, row0);
      };
      // ---- epilogue P: x1 = X + LN1(D2 + bp) -> X (fp32), tile buffer (fp16)
      auto epi_p = [&](int t, int i) -> bool {
        const int row0 = t * 128 + q * 32;
        const int db = i & 1;
        const uint32_t td2 = tq + (uint32_t)(Cfg::D2OFF + db * CP);
        if (lane == 0 && half < CP / 32) {
          bulk_wait_read<0>();
          res_load(jcnt & 1, half, row0);
        }
        if (!mbar_wait(&accp[db], (uint32_t)((i >> 1) & 1), DEV_TIMEOUT_ACC)) return false;
        tc_fence_after();
        // row sums of x and x^2 in column order, as the GEMM LayerNorm epilogue
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < CP / 32; c++) {
          float v[32];
          tmem_ld32(td2 + (uint32_t)(c * 32), v);
#pragma unroll
          for (int u = 0; u < 32; u++) {
            const float x = v[u] + s_vec[HP + 3 * CP + c * 32 + u];
            s1 += x;
            s2 += x * x;
          }
        }
        const float nf = (float)a.ln_n;
        const float mean = s1 / nf;
        const float rstd = 1.0f / sqrtf(fmaxf(s2 / nf - mean * mean, 0.0f) + a.ln_eps);
        const float nmr = -mean * rstd;
#pragma unroll 1
        for (int c = half; c < CP / 32; c += 2, jcnt++) {
          const int jb = jcnt & 1;
          float* f32 = reinterpret_cast<float*>(wf32 + jb * 4096);
          float v[32];
          tmem_ld32(td2 + (uint32_t)(c * 32), v);
          if (lane == 0) {
            bulk_wait_read<0>();
            if (c + 2 < CP / 32) res_load(jb ^ 1, c + 2, row0);
          }
          if (!mbar_wait(&wrb[jb], (jcnt >> 1) & 1, DEV_TIMEOUT_FULL)) return false;
          const int cl0 = c * 32;
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const float4 bb = *reinterpret_cast<const float4*>(s_vec + HP + 3 * CP + cl0 + 4 * u);
            const float4 gg = *reinterpret_cast<const float4*>(s_vec + HP + 4 * CP + cl0 + 4 * u);
            const float4 be = *reinterpret_cast<const float4*>(s_vec + HP + 5 * CP + cl0 + 4 * u);
            float4* slot = reinterpret_cast<float4*>(f32 + lane * 32 + ((u ^ sw128) << 2));
            const float4 rr = *slot;
            float x[4] = {v[4 * u] + bb.x, v[4 * u + 1] + bb.y, v[4 * u + 2] + bb.z,
                          v[4 * u + 3] + bb.w};
            x[0] = fmaf(fmaf(x[0], rstd, nmr), gg.x, be.x) + rr.x;
            x[1] = fmaf(fmaf(x[1], rstd, nmr), gg.y, be.y) + rr.y;
            x[2] = fmaf(fmaf(x[2], rstd, nmr), gg.z, be.z) + rr.z;
            x[3] = fmaf(fmaf(x[3], rstd, nmr), gg.w, be.w) + rr.w;
            *slot = make_float4(x[0], x[1], x[2], x[3]);
            v[4 * u] = x[0];
            v[4 * u + 1] = x[1];
            v[4 * u + 2] = x[2];
            v[4 * u + 3] = x[3];
          }
          // fp16 x1 into the tile buffer: K-chunk c / 2, 16-byte pieces (c % 2) * 4 + m
          uint8_t* xrow = sX + (c >> 1) * 16384 + r * 128;
#pragma unroll
          for (int m = 0; m < 4; m++) {
            const __half2 h0 = __floats2half2_rn(v[8 * m], v[8 * m + 1]);
            const __half2 h1 = __floats2half2_rn(v[8 * m + 2], v[8 * m + 3]);
            const __half2 h2 = __floats2half2_rn(v[8 * m + 4], v[8 * m + 5]);
            const __half2 h3 = __floats2half2_rn(v[8 * m + 6], v[8 * m + 7]);
            *reinterpret_cast<uint4*>(xrow + ((((c & 1) * 4 + m) ^ (r & 7)) << 4)) =
                make_uint4(*reinterpret_cast<const uint32_t*>(&h0),
                           *reinterpret_cast<const uint32_t*>(&h1),
                           *reinterpret_cast<const uint32_t*>(&h2),
                           *reinterpret_cast<const uint32_t*>(&h3));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&mapX32, f32, cl0, row0);
            bulk_commit();
          }
        }
        // x1 is fc1's operand now; D2 buffer db is drained
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(x1ready);
        return true;
      };
      // ---- epilogue 2: X <- X + LN2(D2 + b2), X16 <- fp16(X), through TMA
      auto epi_2 = [&](int t, int i) -> bool {
        const int row0 = t * 128 + q * 32;  // this warp's 32 rows as a TMA box origin
        const int db = i & 1;
        const uint32_t td2 = tq + (uint32_t)(Cfg::D2OFF + db * CP);
        // the first residual tile is requested before waiting for fc2 (with PROJ it is
        // epilogue P's x1: its stores must have landed first)
        if (lane == 0 && half < CP / 32) {
          if (PROJ) {
            bulk_wait<0>();
            asm volatile("fence.proxy.async.global;" ::: "memory");
          }
          bulk_wait_read<0>();
          res_load(jcnt & 1, half, row0);
        }
        if (!mbar_wait(&acc2[db], (uint32_t)((i >> 1) & 1), DEV_TIMEOUT_ACC)) return false;
        tc_fence_after();
        // row sums of x and x^2 in column order (the bias add two lanes at a time)
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < CP / 32; c++) {
          float v[32];
          tmem_ld32(td2 + (uint32_t)(c * 32), v);
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const float4 bb = *reinterpret_cast<const float4*>(s_vec + HP + c * 32 + 4 * u);
            const float2 x0 = f2_unpack(f2_add(f2_pack(v[4 * u], v[4 * u + 1]), f2_pack(bb.x, bb.y)));
            const float2 x1 =
                f2_unpack(f2_add(f2_pack(v[4 * u + 2], v[4 * u + 3]), f2_pack(bb.z, bb.w)));
            s1 += x0.x;
            s2 += x0.x * x0.x;
            s1 += x0.y;
            s2 += x0.y * x0.y;
            s1 += x1.x;
            s2 += x1.x * x1.x;
            s1 += x1.y;
            s2 += x1.y * x1.y;
          }
        }
        const float nf = (float)a.ln_n;
        const float mean = s1 / nf;
        const float rstd = 1.0f / sqrtf(fmaxf(s2 / nf - mean * mean, 0.0f) + a.ln_eps);
        const float nmr = -mean * rstd;
        const unsigned long long RS = f2_pack(rstd, rstd), NM = f2_pack(nmr, nmr);
#pragma unroll 1
        for (int c = half; c < CP / 32; c += 2, jcnt++) {
          const int jb = jcnt & 1;
          float* f32 = reinterpret_cast<float*>(wf32 + jb * 4096);
          float v[32];
          tmem_ld32(td2 + (uint32_t)(c * 32), v);
          if (c + 2 >= CP / 32) {  // this warp is done reading D2 buffer db
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d2free[db]);
          }
          if (lane == 0) {
            // the fp16 tile and the other fp32 buffer are free once every earlier
            // store has read them; then the next chunk's residual goes there
            bulk_wait_read<0>();
            if (c + 2 < CP / 32) res_load(jb ^ 1, c + 2, row0);
          }
          if (!mbar_wait(&wrb[jb], (jcnt >> 1) & 1, DEV_TIMEOUT_FULL)) return false;
          const int cl0 = c * 32;
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const float4 bb = *reinterpret_cast<const float4*>(s_vec + HP + cl0 + 4 * u);
            const float4 gg = *reinterpret_cast<const float4*>(s_vec + HP + CP + cl0 + 4 * u);
            const float4 be = *reinterpret_cast<const float4*>(s_vec + HP + 2 * CP + cl0 + 4 * u);
            float4* slot = reinterpret_cast<float4*>(f32 + lane * 32 + ((u ^ sw128) << 2));
            const float4 rr = *slot;
            // fma(fma(v + b, rstd, -mean * rstd), gamma, beta) + residual, two lanes at a time
            unsigned long long lo = f2_add(f2_pack(v[4 * u], v[4 * u + 1]), f2_pack(bb.x, bb.y));
            unsigned long long hi =
                f2_add(f2_pack(v[4 * u + 2], v[4 * u + 3]), f2_pack(bb.z, bb.w));
            lo = f2_add(f2_fma(f2_fma(lo, RS, NM), f2_pack(gg.x, gg.y), f2_pack(be.x, be.y)),
                        f2_pack(rr.x, rr.y));
            hi = f2_add(f2_fma(f2_fma(hi, RS, NM), f2_pack(gg.z, gg.w), f2_pack(be.z, be.w)),
                        f2_pack(rr.z, rr.w));
            const float2 ol = f2_unpack(lo), oh = f2_unpack(hi);
            const float4 o = make_float4(ol.x, ol.y, oh.x, oh.y);
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
        return true;
      };
      int i = 0;
      int tprev = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, i++) {
        if constexpr (PROJ) {
          // epilogue P of this tile first (fc1 waits for it), then epilogue 2 of the
          // previous one (its fc2 ran meanwhile)
          ok = epi_p(t, i);
          if (ok && tprev >= 0) ok = epi_2(tprev, i - 1);
          tprev = t;
        } else {
          ok = epi_2(t, i);
        }
      }
      if (PROJ && ok && tprev >= 0) epi_2(tprev, i - 1);
      if (lane == 0) bulk_wait<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TCOLS);
  }
}

template <int CP, int HP, int STAGES, bool PROJ>
cudaError_t launch_mlp_t(const CUtensorMap& mX, const CUtensorMap& mW1, const CUtensorMap& mW2,
                         const CUtensorMap& mX32, const CUtensorMap& mX16o,
                         const CUtensorMap& mWp, const MlpArgs& a, cudaStream_t st) {
  using Cfg = MlpCfg<CP, HP, STAGES>;
  static LaunchSetup setup;
  int ctas = 0;
  const cudaError_t err =
      resident_ctas(setup, k_mlp<CP, HP, STAGES, PROJ>, kMlpThreads, Cfg::SMEM, &ctas);
  if (err != cudaSuccess) return err;
  const int tiles = (a.M + 127) / 128;
  const int G = tiles < ctas ? tiles : ctas;
  return launch_pdl(k_mlp<CP, HP, STAGES, PROJ>, dim3(G), dim3(kMlpThreads), Cfg::SMEM, st, mX,
                    mW1, mW2, mX32, mX16o, mWp, a);
}

}  // namespace

cudaError_t launch_mlp(const CUtensorMap& mX, const CUtensorMap& mW1, const CUtensorMap& mW2,
                       const CUtensorMap& mX32, const CUtensorMap& mX16o, const MlpArgs& a, int cp,
                       int hp, cudaStream_t st, const CUtensorMap* mWp) {
  if (mWp) {
    if (cp == 192 && hp == 384 && a.bp && a.g1 && a.beta1)
      return launch_mlp_t<192, 384, 3, true>(mX, mW1, mW2, mX32, mX16o, *mWp, a, st);
    return cudaErrorNotSupported;
  }
  if (cp == 192 && hp == 384)
    return launch_mlp_t<192, 384, 3, false>(mX, mW1, mW2, mX32, mX16o, mX, a, st);
  if (cp == 64 && hp == 128)
    return launch_mlp_t<64, 128, 4, false>(mX, mW1, mW2, mX32, mX16o, mX, a, st);
  return cudaErrorNotSupported;
}

}  // namespace s2s
