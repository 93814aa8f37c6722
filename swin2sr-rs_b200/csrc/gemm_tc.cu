// tcgen05 GEMM and implicit-GEMM 3x3 convolution for sm_100a.
//
// A persistent kernel: each CTA owns one N tile and walks M tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... computing 128 x BN tiles of D = A * B^T in TMEM (fp16
// operands, fp32 accumulation) with a fused epilogue:
//   warp 0       TMA producer: A and B K-slices (64 fp16 = one 128-byte swizzle row)
//                into a STAGES-deep shared-memory ring that runs across tiles (with
//                B resident, variants may give A its own AR-deep ring: two tiles of
//                A in flight, so a tile's loads do not wait for the previous tile's
//                MMAs to free their slots);
//   warp 1       allocates TMEM, issues tcgen05.mma (K = 16 per instruction), frees
//                ring slots with tcgen05.commit, and alternates between two TMEM
//                accumulators so the next tile's MMAs overlap this tile's epilogue;
//   warps 2..9   epilogue, two warps per TMEM lane quarter splitting the columns:
//                tcgen05.ld of the accumulator (thread = tile row),
//                bias / activation / LayerNorm / residual in fp32, then a
//                shared-memory transpose so that every global access of a warp is
//                four 128-byte row segments (float4 per lane).
//
// In conv mode the A tile is a boxh x boxw patch of output pixels and each K-slice
// is one (tap, 64-channel chunk) of the NHWC input, fetched by a 4-D TMA box at
// the tap's offset: TMA's zero fill outside the plane IS the conv's zero padding,
// so no im2col buffer exists. With PATCH (64 input channels), a slot instead holds
// one (boxh + 2)-row patch per kx and the weights of its three ky taps: tap (ky, kx)
// is the patch from row ky * boxw on, so the input is fetched three times per tile
// instead of nine.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace s2s {

namespace {

// producer warp, MMA warp and kEpiWarps epilogue warps (a launch may take 12)
constexpr int kEpiWarps = 8;
constexpr int kStageFloats = 32 * 36;  // STORE_SHUFFLE2 staging: 32 rows x 32 cols, 16-B rows
// Per epilogue warp: two fp32 32x32 tiles (residual in, result out; 128-byte swizzle)
// and two fp16 32x32 tiles (64-byte swizzle), double-buffered across chunks. Variants
// whose epilogue writes fp16 only keep just the two fp16 tiles (kWarpBufF16).
constexpr int kWarpBuf = 2 * 4096 + 2 * 2048;
constexpr int kWarpBufF16 = 2 * 2048;

template <int BN>
struct TmemCols {
  static constexpr uint32_t value = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

template <int BN, int STAGES, int ACT, bool LN, int RES, int STORE, int AR = 0,
          int WB = kWarpBuf, bool PATCH = false, int EW = kEpiWarps>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
    k_gemm(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
           const __grid_constant__ OutMaps om, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = BN * 128;
  constexpr int NA = AR > 0 ? AR : STAGES;  // A ring slots (= the ring's barriers)
  // a slot's A and B bytes: one K-slice, or with PATCH a (boxh + 2) x boxw patch (at
  // most 24 KB for boxw <= 32) and three taps' weights
  constexpr int A_SLOT = PATCH ? 24576 : A_BYTES;
  constexpr int B_SLOT = PATCH ? 3 * B_BYTES : B_BYTES;
  static_assert(!PATCH || (AR == 0 && (STORE == STORE_PLANES ||
                                         (STORE == STORE_ROWS && WB == kWarpBufF16))),
                "patch mode: the plane store, or fp16-only row stores");
  constexpr int F16OFF = WB >= kWarpBuf ? 8192 : 0;  // fp16 tiles within a warp's staging
  static_assert(WB == kWarpBuf || (WB == kWarpBufF16 && STORE == STORE_ROWS && RES != 2) ||
                    (WB == kStageFloats * 4 && STORE == STORE_SHUFFLE2) ||
                    (WB == 0 && STORE == STORE_PLANES),
                "fp16-only staging, the pixel-shuffle transpose tile alone, or none for the "
                "plane store (registers to global)");
  uint8_t* sA = smem;
  uint8_t* sB = smem + NA * A_SLOT;
  uint8_t* obuf = sB + STAGES * B_SLOT;                     // [EW][WB], 1 KB aligned
  float* s_vec = reinterpret_cast<float*>(obuf + EW * WB);  // bias, gamma, beta [3][BN]
  int* s_rows = reinterpret_cast<int*>(s_vec + 3 * BN);     // shuffle store: per warp, per row
  uint64_t* full = reinterpret_cast<uint64_t*>(s_rows + EW * 32 * 4);
  uint64_t* empty = full + NA;
  uint64_t* accf = empty + NA;       // [2] accumulator ready
  uint64_t* acce = accf + 2;         // [2] accumulator drained
  uint64_t* fin = acce + 2;          // all MMAs of this CTA retired
  uint64_t* bfull = fin + 1;         // resident B (all K-slices) landed
  uint64_t* rbar = bfull + 1;        // [EW][2] residual tile landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(rbar + 2 * EW);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t NCOLS = TmemCols<2 * BN>::value;

  const int NT = a.N / BN;
  const int tiles_m = a.conv ? a.B * a.tiles_x * a.tiles_y : (a.M + 127) / 128;
  const int num_tiles = tiles_m * NT;
  const int G = gridDim.x;  // a multiple of NT: the CTA's N tile is fixed
  const int n0 = (blockIdx.x % NT) * BN;
  const int num_k = PATCH ? 3 : a.conv ? 9 * a.kc : a.K / 64;  // K-slices (PATCH: kx) per tile
  auto coords = [&](int t, int& m0, int& bimg, int& y0, int& x0) {
    const int mt = t / NT;
    m0 = 0;
    bimg = 0;
    y0 = 0;
    x0 = 0;
    if (!a.conv) {
      m0 = mt * 128;
    } else {
      const int per_img = a.tiles_x * a.tiles_y;
      bimg = mt / per_img;
      const int rem = mt - bimg * per_img;
      y0 = a.y_off + (rem / a.tiles_x) * a.boxh;
      x0 = (rem % a.tiles_x) * a.boxw;
    }
  };

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapB);
    for (int s = 0; s < NA; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], EW);
    }
    mbar_init(fin, 1);
    mbar_init(bfull, 1);
    for (int k = 0; k < 2 * EW; k++) mbar_init(&rbar[k], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, NCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_trigger();
  // When all of this CTA's B (its N tile over the whole K) fits the ring's B slots -
  // a GEMM with K <= 64 * STAGES - it is loaded once and stays resident; the ring then
  // streams A only. B is a weight, never the previous kernel's output: its load is
  // issued before the dependency wait and overlaps the previous kernel's tail.
  const bool bres = !a.conv && num_k <= STAGES;  // AR > 0 launches guarantee it
  if (warp == 0 && lane == 0 && bres) {
    mbar_arrive_expect_tx(bfull, (uint32_t)(num_k * B_BYTES));
    for (int k = 0; k < num_k; k++) tma_load_2d(sB + k * B_BYTES, &mapB, bfull, k * 64, n0);
  }
  pdl_wait();  // the previous kernel's outputs (this kernel's A operand) are complete

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      uint32_t kit = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += G) {
        int m0, bimg, y0, x0;
        coords(t, m0, bimg, y0, x0);
        for (int k = 0; k < num_k; k++, kit++) {
          const int s = kit % NA;
          if (kit >= NA && !mbar_wait(&empty[s], ((kit / NA) - 1) & 1, DEV_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          if constexpr (PATCH) {
            // the patch of kx = k: rows y0 - 1 .. y0 + boxh, columns x0 + k - 1 .. ,
            // and the weights of taps (0, k), (1, k), (2, k)
            mbar_arrive_expect_tx(&full[s], (uint32_t)((a.boxh + 2) * a.boxw * 128 + B_SLOT));
            tma_load_4d(sA + s * A_SLOT, &mapA, &full[s], 0, x0 + k - 1, y0 - 1, bimg);
            for (int ky = 0; ky < 3; ky++)
              tma_load_2d(sB + s * B_SLOT + ky * B_BYTES, &mapB, &full[s], (ky * 3 + k) * 64, n0);
          } else {
            mbar_arrive_expect_tx(&full[s], bres ? A_BYTES : A_BYTES + B_BYTES);
            if (!a.conv) {
              const int ak = a.amod ? k % a.amod : k;
              tma_load_2d(sA + s * A_SLOT, &mapA, &full[s], ak * 64, m0);
            } else {
              const int tap = k / a.kc, cc = k - tap * a.kc;
              const int ky = tap / 3, kx = tap - ky * 3;
              const int ac = a.amod ? cc % a.amod : cc;
              tma_load_4d(sA + s * A_SLOT, &mapA, &full[s], ac * 64, x0 + kx - 1, y0 + ky - 1,
                          bimg);
            }
            if (!bres) tma_load_2d(sB + s * B_SLOT, &mapB, &full[s], k * 64, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      uint32_t kit = 0;
      bool ok = !bres || mbar_wait(bfull, 0, DEV_TIMEOUT_FULL);
      int i = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += G, i++) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&acce[b], ((i >> 1) - 1) & 1, DEV_TIMEOUT_ACC)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int k = 0; k < num_k; k++, kit++) {
          const int s = kit % NA;
          if (!mbar_wait(&full[s], (kit / NA) & 1, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if constexpr (PATCH) {
            // tap (ky, k): the patch from row ky * boxw on (1024-byte aligned: boxw % 8 == 0)
            for (int ky = 0; ky < 3; ky++) {
              const uint64_t ad = sw128_desc(smem_u32(sA + s * A_SLOT + ky * a.boxw * 128));
              const uint64_t bd = sw128_desc(smem_u32(sB + s * B_SLOT + ky * B_BYTES));
#pragma unroll
              for (int kk = 0; kk < 4; kk++)
                tc_mma_f16(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                           (k | ky | kk) != 0 ? 1u : 0u);
            }
          } else {
            const uint64_t ad = sw128_desc(smem_u32(sA + s * A_SLOT));
            const uint64_t bd = sw128_desc(smem_u32(sB + (bres ? k : s) * B_SLOT));
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
              tc_mma_f16(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                         (k | kk) != 0 ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);
        }
        tc_commit(&accf[b]);
      }
      // Every MMA this thread issued has retired before TMEM is released.
      tc_commit(fin);
      mbar_wait(fin, 0, DEV_TIMEOUT_ACC);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const Epi& e = a.epi;
    const int q = warp & 3;           // TMEM lane quarter this warp may read
    // which of the EW / 4 interleaved sets of column chunks this warp stores
    const int part = (warp - 2) >> 2;
    constexpr int NPART = EW / 4;
    const int et = threadIdx.x - 64;  // 0..255 among the epilogue threads
    const int r = q * 32 + lane;      // tile row owned in the thread-per-row phases
    int* s_row = s_rows + (warp - 2) * 32 * 4 - q * 32 * 4;  // indexed by tile row q*32..q*32+31
    // Column vectors of this CTA's (fixed) N tile, loaded once.
    for (int c = et; c < BN; c += 32 * EW) {
      const int col = n0 + c;
      s_vec[c] = e.bias ? e.bias[col] : 0.0f;
      s_vec[BN + c] = (e.ln_n > 0 && col < e.ln_n) ? e.ln_g[col] : 0.0f;
      s_vec[2 * BN + c] = (e.ln_n > 0 && col < e.ln_n) ? e.ln_b[col] : 0.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(32 * EW) : "memory");
    uint8_t* wbuf = obuf + (warp - 2) * WB;
    float* stg = reinterpret_cast<float*>(wbuf);  // STORE_SHUFFLE2 staging
    uint64_t* wrb = rbar + 2 * (warp - 2);        // this warp's residual barriers
    uint32_t jcnt = 0;                            // chunks this warp has processed (buffer parity)
    if (STORE == STORE_ROWS && lane == 0) {
      tma_prefetch_desc(&om.o32);
      tma_prefetch_desc(&om.o16);
    }
    int i = 0;
    for (int t = blockIdx.x; t < num_tiles; t += G, i++) {
    const int b = i & 1;
    int m0, bimg, y0, x0;
    coords(t, m0, bimg, y0, x0);
    int mlog, py = 0, px = 0;
    bool valid;
    if (!a.conv) {
      mlog = m0 + r;
      valid = mlog < a.M;
    } else {
      py = y0 + r / a.boxw;
      px = x0 + (r % a.boxw);
      valid = (py < a.y_end) && (px < a.W);
      mlog = (bimg * a.H + py) * a.W + px;
    }
    if constexpr (STORE == STORE_SHUFFLE2) {
      int* rw = s_row + r * 4;
      rw[0] = valid ? mlog : -1;
      rw[1] = (bimg * 2 * a.H + 2 * py) * (2 * a.W) + 2 * px;  // (dy, dx) = (0, 0) pixel
      __syncwarp();
    }
    // This warp's 32 rows as a TMA box origin: row m0 + 32q, or the conv sub-box.
    const int orow = q * 32;
    const int opx = a.conv ? x0 + (orow % a.boxw) : 0;
    const int opy = a.conv ? y0 + orow / a.boxw : 0;
    auto box_load_res = [&](void* dst, int col, uint64_t* bar) {
      if (a.conv)
        tma_load_4d(dst, &om.res, bar, col, opx, opy, bimg);
      else
        tma_load_2d(dst, &om.res, bar, col, m0 + orow);
    };
    auto box_store = [&](const CUtensorMap* m, const void* src, int col) {
      if (a.conv)
        tma_store_4d(m, src, col, opx, opy, bimg);
      else
        tma_store_2d(m, src, col, m0 + orow);
    };
    // Post-norm residual: the first chunk's tile is requested before the accumulator
    // is ready, so its latency hides behind the MMAs.
    if constexpr (STORE == STORE_ROWS && RES == 2) {
      if (lane == 0 && part < BN / 32) {
        bulk_wait_read<0>();
        const int jb = jcnt & 1;
        mbar_arrive_expect_tx(&wrb[jb], 4096);
        box_load_res(wbuf + jb * 4096, n0 + part * 32, &wrb[jb]);
      }
    }

    const uint32_t tbase = tmem + (uint32_t)(b * BN) + ((uint32_t)(q * 32) << 16);
    const bool acc_ok = mbar_wait(&accf[b], (i >> 1) & 1, DEV_TIMEOUT_ACC);
    tc_fence_after();
    if (!acc_ok) break;

    // The epilogue variant is compile-time: the per-element code below is straight
    // line. Padded columns need no masking: their weights, bias, residual, gamma and
    // beta are all zero, so they come out as exact zeros and add nothing to the LN
    // statistics.
    auto pre = [&](float v, int cl) {
      v += s_vec[cl];
      if constexpr (ACT == ACT_GELU) v = gelu_erf(v);
      if constexpr (ACT == ACT_LRELU) v = v < 0.0f ? v * e.slope : v;
      return v;
    };
    const float* rpre = nullptr;
    if constexpr (RES == 1) rpre = e.res_pre + (size_t)(valid ? mlog : 0) * e.ld_res_pre + n0;

    if constexpr (STORE == STORE_ROWS) {
      float mean = 0.0f, rstd = 1.0f;
      if constexpr (LN) {
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
#pragma unroll
          for (int j4 = 0; j4 < 8; j4++) {
            float4 r4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (RES == 1) r4 = reinterpret_cast<const float4*>(rpre + c * 32)[j4];
            const float rr[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const int j = 4 * j4 + k;
              float x = pre(v[j], c * 32 + j);
              if constexpr (RES == 1) x += rr[k];
              s1 += x;
              s2 += x * x;
            }
          }
        }
        const float nf = (float)e.ln_n;
        mean = s1 / nf;
        const float var = fmaxf(s2 / nf - mean * mean, 0.0f);
        rstd = 1.0f / sqrtf(var + e.ln_eps);
      }
      const float nmr = -mean * rstd;
      const int sw128 = lane & 7, sw64 = (lane >> 1) & 3;  // this row's swizzle phases
#pragma unroll 1
      for (int c = part; c < BN / 32; c += NPART, jcnt++) {
        const int jb = jcnt & 1;
        float* f32 = reinterpret_cast<float*>(wbuf + jb * 4096);
        uint8_t* f16 = wbuf + F16OFF + jb * 2048;
        float v[32];
        tmem_ld32(tbase + c * 32, v);
        if constexpr (RES == 2) {
          // request the next chunk's residual into the other buffer, then wait for ours
          if (lane == 0 && c + 2 < BN / 32) {
            bulk_wait_read<0>();
            mbar_arrive_expect_tx(&wrb[jb ^ 1], 4096);
            box_load_res(wbuf + (jb ^ 1) * 4096, n0 + (c + 2) * 32, &wrb[jb ^ 1]);
          }
          if (!mbar_wait(&wrb[jb], (jcnt >> 1) & 1, DEV_TIMEOUT_FULL)) break;
        } else {
          if (lane == 0) bulk_wait_read<1>();  // this buffer's store two chunks ago
          __syncwarp();
        }
        // two-term output: hi and lo take both fp16 tiles, free once every store read them
        if (e.lo_off) {
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        const int cl0 = c * 32;
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const float4 bb = *reinterpret_cast<const float4*>(s_vec + cl0 + 4 * u);
          float x[4] = {v[4 * u] + bb.x, v[4 * u + 1] + bb.y, v[4 * u + 2] + bb.z,
                        v[4 * u + 3] + bb.w};
          float4 r4 = make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (RES == 1) r4 = reinterpret_cast<const float4*>(rpre + cl0)[u];
          const float rr[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            if constexpr (ACT == ACT_GELU) x[k] = gelu_erf(x[k]);
            if constexpr (ACT == ACT_LRELU) x[k] = x[k] < 0.0f ? x[k] * e.slope : x[k];
            if constexpr (RES == 1) x[k] += rr[k];
          }
          if constexpr (LN) {
            const float4 gg = *reinterpret_cast<const float4*>(s_vec + BN + cl0 + 4 * u);
            const float4 be = *reinterpret_cast<const float4*>(s_vec + 2 * BN + cl0 + 4 * u);
            x[0] = fmaf(fmaf(x[0], rstd, nmr), gg.x, be.x);
            x[1] = fmaf(fmaf(x[1], rstd, nmr), gg.y, be.y);
            x[2] = fmaf(fmaf(x[2], rstd, nmr), gg.z, be.z);
            x[3] = fmaf(fmaf(x[3], rstd, nmr), gg.w, be.w);
          }
          float4* slot = reinterpret_cast<float4*>(f32 + lane * 32 + ((u ^ sw128) << 2));
          if constexpr (RES == 2) {
            const float4 rr = *slot;
            x[0] += rr.x;
            x[1] += rr.y;
            x[2] += rr.z;
            x[3] += rr.w;
          }
          v[4 * u] = x[0];
          v[4 * u + 1] = x[1];
          v[4 * u + 2] = x[2];
          v[4 * u + 3] = x[3];
          if constexpr (WB == kWarpBuf) {
            if (e.o32 || e.o32b) *slot = make_float4(x[0], x[1], x[2], x[3]);
          }
        }
        if constexpr (ACT == ACT_QKNORM) {
          // one head's q, k or v is one DP-wide group of this row's columns
          auto group_scale = [&](int grp, float ss) {
            const int part = grp % 3;
            const float r = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
            return part == 0 ? r * e.qk_scale[grp / 3] : part == 1 ? r : 1.0f;
          };
          const int gc = n0 + cl0;
          if (e.qk_dp == 32) {
            float ss = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; j++) ss = fmaf(v[j], v[j], ss);
            const float sc = group_scale(gc / 32, ss);
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] *= sc;
          } else {
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; j++) {
              s0 = fmaf(v[j], v[j], s0);
              s1 = fmaf(v[16 + j], v[16 + j], s1);
            }
            const float c0 = group_scale(gc / 16, s0), c1 = group_scale(gc / 16 + 1, s1);
#pragma unroll
            for (int j = 0; j < 16; j++) {
              v[j] *= c0;
              v[16 + j] *= c1;
            }
          }
        }
        uint8_t* const f16h = e.lo_off ? wbuf + F16OFF : f16;  // hi tile
        uint8_t* const f16l = wbuf + F16OFF + 2048;              // lo tile (two-term only)
        if (e.o16) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            __half2 h0 = __floats2half2_rn(v[8 * u], v[8 * u + 1]);
            __half2 h1 = __floats2half2_rn(v[8 * u + 2], v[8 * u + 3]);
            __half2 h2 = __floats2half2_rn(v[8 * u + 4], v[8 * u + 5]);
            __half2 h3 = __floats2half2_rn(v[8 * u + 6], v[8 * u + 7]);
            *reinterpret_cast<uint4*>(f16h + lane * 64 + ((u ^ sw64) << 4)) =
                make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                           *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
            if (e.lo_off) {
              // the remainder each fp16 value left out, itself in fp16
              const __half2 hs[4] = {h0, h1, h2, h3};
              uint32_t lw[4];
#pragma unroll
              for (int m = 0; m < 4; m++) {
                const float2 hf = __half22float2(hs[m]);
                const __half2 l = __floats2half2_rn(v[8 * u + 2 * m] - hf.x,
                                                    v[8 * u + 2 * m + 1] - hf.y);
                lw[m] = *reinterpret_cast<const uint32_t*>(&l);
              }
              *reinterpret_cast<uint4*>(f16l + lane * 64 + ((u ^ sw64) << 4)) =
                  make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (e.o32) box_store(&om.o32, f32, n0 + cl0);
          if (e.o32b) box_store(&om.o32b, f32, n0 + cl0);
          if (e.o16) box_store(&om.o16, f16h, n0 + cl0);
          if (e.o16 && e.lo_off) box_store(&om.o16, f16l, e.lo_off + n0 + cl0);
          bulk_commit();
        }
      }
    } else if constexpr (STORE == STORE_SHUFFLE2) {
      float mean = 0.0f, rstd = 1.0f;
      if constexpr (LN) {
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; j++) {
            float x = pre(v[j], c * 32 + j);
            if constexpr (RES == 1) x += rpre[c * 32 + j];
            s1 += x;
            s2 += x * x;
          }
        }
        const float nf = (float)e.ln_n;
        mean = s1 / nf;
        const float var = fmaxf(s2 / nf - mean * mean, 0.0f);
        rstd = 1.0f / sqrtf(var + e.ln_eps);
      }
      const int sub = lane >> 3, cg = lane & 7;  // coalesced phase: 4 rows x 8 lanes
      const int wrow0 = q * 32;
      const int F = a.N / 4;  // STORE_SHUFFLE2: output channels
#pragma unroll 1
      for (int c = part; c < BN / 32; c += NPART) {
        float v[32];
        tmem_ld32(tbase + c * 32, v);
        const int cl0 = c * 32;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          float x = pre(v[j], cl0 + j);
          if constexpr (RES == 1) x += rpre[cl0 + j];
          if constexpr (LN) x = (x - mean) * rstd * s_vec[BN + cl0 + j] + s_vec[2 * BN + cl0 + j];
          v[j] = x;
        }
        float4* srow = reinterpret_cast<float4*>(stg + lane * 36);
#pragma unroll
        for (int j = 0; j < 8; j++)
          srow[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        __syncwarp();
        const int col = n0 + cl0 + cg * 4;
        float4 val[8];
        int src[8];
#pragma unroll
        for (int it = 0; it < 8; it++) {
          const int rr = it * 4 + sub;
          val[it] = *reinterpret_cast<const float4*>(stg + rr * 36 + cg * 4);
          src[it] = s_row[(wrow0 + rr) * 4];
        }
        {
          const int qd = col / F, f = col - qd * F;
          const int dy = qd >> 1, dx = qd & 1;
          size_t dst[8];
#pragma unroll
          for (int it = 0; it < 8; it++)
            dst[it] = ((size_t)s_row[(wrow0 + it * 4 + sub) * 4 + 1] + (size_t)dy * (2 * a.W) + dx) *
                          F + f;
          if constexpr (RES == 2) {
            float4 rp[8];
#pragma unroll
            for (int it = 0; it < 8; it++)
              rp[it] = src[it] >= 0 ? __ldg(reinterpret_cast<const float4*>(e.res_post + dst[it]))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int it = 0; it < 8; it++) {
              val[it].x += rp[it].x;
              val[it].y += rp[it].y;
              val[it].z += rp[it].z;
              val[it].w += rp[it].w;
            }
          }
#pragma unroll
          for (int it = 0; it < 8; it++) {
            if (src[it] < 0) continue;
            __half2 h0 = __floats2half2_rn(val[it].x, val[it].y);
            __half2 h1 = __floats2half2_rn(val[it].z, val[it].w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&h0);
            u.y = *reinterpret_cast<uint32_t*>(&h1);
            *reinterpret_cast<uint2*>(e.o16 + dst[it]) = u;
          }
        }
        __syncwarp();
      }
    } else if constexpr (STORE == STORE_PLANES) {
      float v[32];
      tmem_ld32(tbase, v);
      if (valid && part == 0) {
#pragma unroll
        for (int ch = 0; ch < 3; ch++) {
          const float x = pre(v[ch], ch);
          const float mean = ch == 0 ? e.mean0 : ch == 1 ? e.mean1 : e.mean2;
          if (e.planes_raw)
            e.planes_raw[((size_t)(bimg * 3 + ch) * a.H + py) * a.W + px] = x;
          const int oy = py - e.crop_y0;
          if (e.planes && oy >= 0 && oy < e.crop_h && px < e.crop_w)
            e.planes[((size_t)(bimg * 3 + ch) * e.crop_h + oy) * e.crop_w + px] =
                x / e.img_range + mean;
        }
      }
    } else {  // STORE_DIRECT
      const int s = e.scale, s2 = s * s, nout = 3 * s2;
#pragma unroll 1
      for (int c = part; c < BN / 32; c += NPART) {
        float v[32];
        tmem_ld32(tbase + c * 32, v);
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int col = c * 32 + j;
          if (!valid || col >= nout) continue;
          const int ch = col / s2, rem = col - ch * s2, dy = rem / s, dx = rem - dy * s;
          const int Y = py * s + dy - e.crop_y0, X = px * s + dx;
          const float mean = ch == 0 ? e.mean0 : ch == 1 ? e.mean1 : e.mean2;
          if (Y >= 0 && Y < e.crop_h && X < e.crop_w)
            e.planes[((size_t)(bimg * 3 + ch) * e.crop_h + Y) * e.crop_w + X] =
                pre(v[j], col) / e.img_range + mean;
        }
      }
    }

    // Release this accumulator buffer to the MMA warp.
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acce[b]);
    }
  }

  if (warp >= 2 && lane == 0) bulk_wait<0>();  // this warp's bulk stores are performed
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, NCOLS);
  }
}

template <int BN, int STAGES, int ACT, bool LN, int RES, int STORE, int AR = 0,
          int WB = kWarpBuf, bool PATCH = false, int EW = kEpiWarps>
cudaError_t launch_t(const CUtensorMap& mapA, const CUtensorMap& mapB, const OutMaps& om,
                     const GemmArgs& a, cudaStream_t st) {
  constexpr int NA = AR > 0 ? AR : STAGES;
  constexpr size_t A_SLOT = PATCH ? 24576 : 128 * 128, B_SLOT = (PATCH ? 3 : 1) * BN * 128;
  if (PATCH && (!a.conv || a.kc != 1 || a.boxw > 32 || a.boxw % 8 || a.boxh + 2 > 256))
    return cudaErrorInvalidValue;
  if (AR > 0 && (a.conv || a.K / 64 > STAGES)) return cudaErrorInvalidValue;  // B not resident
  if (WB != kWarpBuf && (a.epi.o32 || a.epi.o32b)) return cudaErrorInvalidValue;
  constexpr int threads = 64 + 32 * EW;
  const size_t smem = 1024 + (size_t)NA * A_SLOT + (size_t)STAGES * B_SLOT + EW * WB +
                      3 * BN * 4 + EW * 32 * 4 * 4 + (2 * NA + 6 + 2 * EW) * 8 + 16;
  static LaunchSetup setup;  // resident CTAs (SMs x CTAs per SM), per device
  int ctas = 0;
  const cudaError_t err = resident_ctas(
      setup, k_gemm<BN, STAGES, ACT, LN, RES, STORE, AR, WB, PATCH, EW>, threads, smem, &ctas);
  if (err != cudaSuccess) return err;
  const int NT = a.N / BN;
  const int tiles_m = a.conv ? a.B * a.tiles_x * a.tiles_y : (a.M + 127) / 128;
  const long tiles = (long)tiles_m * NT;
  long G = tiles < ctas ? tiles : ctas;
  G = (G / NT) * NT;
  if (G < NT) G = NT;
  return launch_pdl(k_gemm<BN, STAGES, ACT, LN, RES, STORE, AR, WB, PATCH, EW>, dim3((unsigned)G), dim3(threads), smem,
                    st, mapA, mapB, om, a);
}

}  // namespace

// The epilogue variants the forward pass uses, per N tile.
#define S2S_VARIANT(BN_, ST_, ACT_, LN_, RES_, STORE_)                                 \
  if (BN == BN_ && act == ACT_ && ln == LN_ && res == RES_ && store == STORE_)        \
    return launch_t<BN_, ST_, ACT_, LN_, RES_, STORE_>(mapA, mapB, om, a, st);

cudaError_t launch_gemm(const CUtensorMap& mapA, const CUtensorMap& mapB, const OutMaps& om,
                        const GemmArgs& a, int BN, cudaStream_t st) {
  if (a.N % BN != 0 || (a.conv == 0 && a.K % 64 != 0)) return cudaErrorInvalidValue;
  const Epi& e = a.epi;
  if (e.ln_n > 0 && a.N != BN) return cudaErrorInvalidValue;
  if (e.res_pre && e.res_post) return cudaErrorInvalidValue;
  if (e.act == ACT_QKNORM && (e.o32 || e.o32b || e.ln_n || !e.qk_scale ||
                              (e.qk_dp != 16 && e.qk_dp != 32) || a.N % (3 * e.qk_dp)))
    return cudaErrorInvalidValue;
  const int act = e.act;
  const bool ln = e.ln_n > 0;
  const int res = e.res_pre ? 1 : (e.res_post ? 2 : 0);
  const int store = e.store;
  if (a.patch) {  // 64-channel convs from kx patches
    // conv_last: five slots (the plane store needs no staging)
    if (BN == 32 && act == ACT_NONE && !ln && res == 0 && store == STORE_PLANES)
      return launch_t<32, 5, ACT_NONE, false, 0, STORE_PLANES, 0, 0, true>(mapA, mapB, om, a, st);
    // the nearest+conv head's 64 -> 64 convs (fp16 rows, LeakyReLU): three slots
    if (BN == 64 && act == ACT_LRELU && !ln && res == 0 && store == STORE_ROWS && !e.o32 &&
        !e.o32b)
      return launch_t<64, 3, ACT_LRELU, false, 0, STORE_ROWS, 0, kWarpBufF16, true>(mapA, mapB, om,
                                                                                  a, st);
    return cudaErrorNotSupported;
  }
  // embed 180 (Cp 192): QKV, convs, fc1, proj/fc2, patch_embed, stage tail, body skip
  // the RSTB conv3x3 (fp16 output only): fp16-only staging leaves room for a 4th stage
  if (BN == 192 && act == ACT_NONE && !ln && res == 0 && store == STORE_ROWS && !e.o32 && !e.o32b)
    return launch_t<192, 4, ACT_NONE, false, 0, STORE_ROWS, 0, kWarpBufF16>(mapA, mapB, om, a, st);
  S2S_VARIANT(192, 3, ACT_NONE, false, 0, STORE_ROWS)
  S2S_VARIANT(192, 3, ACT_GELU, false, 0, STORE_ROWS)
  S2S_VARIANT(192, 3, ACT_NONE, true, 2, STORE_ROWS)
  S2S_VARIANT(192, 3, ACT_NONE, true, 0, STORE_ROWS)
  S2S_VARIANT(192, 3, ACT_NONE, false, 1, STORE_ROWS)
  S2S_VARIANT(192, 3, ACT_NONE, true, 1, STORE_ROWS)
  S2S_VARIANT(192, 3, ACT_NONE, false, 2, STORE_ROWS)
  // QKV (fp16 output only, B resident): A gets a six-slot ring of its own; with
  // two-term operands (K = 3 x 192) B streams through the ring
  // twelve epilogue warps: each stores 2 of the tile's 6 column chunks
  if (BN == 192 && act == ACT_QKNORM && !ln && res == 0 && store == STORE_ROWS && a.K / 64 <= 3)
    return launch_t<192, 3, ACT_QKNORM, false, 0, STORE_ROWS, 6, kWarpBufF16, false, 12>(
        mapA, mapB, om, a, st);
  if (BN == 192 && act == ACT_QKNORM && !ln && res == 0 && store == STORE_ROWS)
    return launch_t<192, 3, ACT_QKNORM, false, 0, STORE_ROWS, 0, kWarpBufF16>(mapA, mapB, om, a, st);
  S2S_VARIANT(96, 4, ACT_QKNORM, false, 0, STORE_ROWS)
  // embed 60 (Cp 64) and the 64-channel head convs
  S2S_VARIANT(64, 4, ACT_NONE, false, 0, STORE_ROWS)
  S2S_VARIANT(64, 4, ACT_NONE, true, 2, STORE_ROWS)
  S2S_VARIANT(64, 4, ACT_NONE, true, 0, STORE_ROWS)
  S2S_VARIANT(64, 4, ACT_NONE, false, 1, STORE_ROWS)
  S2S_VARIANT(64, 4, ACT_NONE, true, 1, STORE_ROWS)
  S2S_VARIANT(64, 4, ACT_NONE, false, 2, STORE_ROWS)
  S2S_VARIANT(64, 4, ACT_LRELU, false, 0, STORE_ROWS)
  S2S_VARIANT(96, 4, ACT_NONE, false, 0, STORE_ROWS)
  S2S_VARIANT(128, 3, ACT_GELU, false, 0, STORE_ROWS)
  // x2 octave convs with the pixel-shuffle store (+ the compressed head's bicubic add)
  // the pixel-shuffle store stages one 32 x 32 transpose tile per warp, so a third
  // ring stage fits
  if (BN == 256 && act == ACT_NONE && !ln && res == 0 && store == STORE_SHUFFLE2)
    return launch_t<256, 3, ACT_NONE, false, 0, STORE_SHUFFLE2, 0, kStageFloats * 4>(mapA, mapB, om,
                                                                                  a, st);
  if (BN == 256 && act == ACT_NONE && !ln && res == 2 && store == STORE_SHUFFLE2)
    return launch_t<256, 3, ACT_NONE, false, 2, STORE_SHUFFLE2, 0, kStageFloats * 4>(mapA, mapB, om,
                                                                                  a, st);
  // 3-channel outputs
  S2S_VARIANT(32, 4, ACT_NONE, false, 0, STORE_PLANES)
  S2S_VARIANT(32, 4, ACT_NONE, false, 0, STORE_DIRECT)
  S2S_VARIANT(64, 4, ACT_NONE, false, 0, STORE_DIRECT)
  return cudaErrorNotSupported;
}
#undef S2S_VARIANT

// ------------------------------------------------------------------- TMA maps
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
}  // namespace

bool make_map_rows(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_padded,
                   uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (cols_padded % 64) != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return false;
  cuuint64_t dims[2] = {cols_padded, rows};
  cuuint64_t strides[1] = {cols_padded * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_nhwc(CUtensorMap* m, const void* base, int B, int H, int W, int Cp, int boxw,
                   int boxh) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (Cp % 64) != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)Cp, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)Cp * 2, (cuuint64_t)W * Cp * 2, (cuuint64_t)H * W * Cp * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)boxw, (cuuint32_t)boxh, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_out_rows(CUtensorMap* m, const void* base, int elem_bytes, uint64_t rows,
                       uint64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (ld * elem_bytes) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return false;
  cuuint64_t dims[2] = {ld, rows};
  cuuint64_t strides[1] = {ld * elem_bytes};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  return fn(m, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
            2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            elem_bytes == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_out_nhwc(CUtensorMap* m, const void* base, int elem_bytes, int B, int H, int W,
                       int ld, int boxw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (ld * elem_bytes) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return false;
  const int bw = boxw < 32 ? boxw : 32, bh = 32 / bw;
  cuuint64_t dims[4] = {(cuuint64_t)ld, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ld * elem_bytes, (cuuint64_t)W * ld * elem_bytes,
                           (cuuint64_t)H * W * ld * elem_bytes};
  cuuint32_t box[4] = {32, (cuuint32_t)bw, (cuuint32_t)bh, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
            4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            elem_bytes == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void conv_box(int W, int* boxw, int* boxh) {
  int bw = 128;
  while (bw > 1 && (W % bw) != 0) bw >>= 1;
  if (bw < 8) bw = 8;  // planes are multiples of the 8-pixel window
  *boxw = bw;
  *boxh = 128 / bw;
}

}  // namespace s2s
