// Fused QKV projection and SwinV2 scaled-cosine window attention on tcgen05, for the
// 180-wide networks (6 heads of head_dim 30 padded to 32; embed padded to Cp = 192).
// Reference: the QKV linear (src/cpu.rs:1533-1540, tools/convert.py:122-138) and the
// attention (src/cpu.rs:1244-1402, tools/network_swin2sr.py:151-190).
//
// Persistent CTAs in head-pair triples: CTA c serves heads 2 (c % 3) and 2 (c % 3) + 1,
// keeps that pair's QKV weights resident in shared memory (72 KB) and walks tiles of two
// consecutive windows (128 tokens). The window partition and the cyclic roll are TMA
// coordinates: each window arrives as four 4 x 4-pixel boxes per 64-channel chunk of the
// NHWC X16 plane (a box never straddles the roll's wrap, since every plane side and the
// shift are multiples of 4), so the tile's rows are in "box order" (token i: box
// i / 16 = 2 by + bx, then row-major in the box) and nothing is gathered by threads.
// Per tile and head j of the pair, on the tensor core (fp16 operands, fp32
// accumulators in TMEM):
//   QKV[j] = X Wqkv[j]^T     (N = 96: the head's q, k and v)
//   S[j]   = Q[j] K[j]^T     (128 x 128: both windows' keys; a row reads its own 64)
//   O[j]   = P[j] V[j]       (P rows hold zeros for the other window's keys)
// and three epilogue warp groups, one thread per tile row (the softmax group two
// warps per row set, 32 keys each):
//   E1  q, k -> + q_bias, L2-normalised (F.normalize, eps 1e-12), q times
//       exp(min(logit_scale, ln 100)) log2 e -> fp16 -> shared (the S operands);
//   E2  S row (own window) + position bias (a compact 15 x 15 relative table per head,
//       row stride 40 floats so a warp's 32 queries hit 32 banks) - 100 log2 e across
//       shift regions (last window row / column of shifted blocks only), max-subtracted
//       exp2, normalised, fp16 -> P in shared;
//   E3  v + v_bias -> fp16, transposed into V^T in shared (the PV B operand, K = tokens);
//       O -> fp16 -> the token's image row of AO (per head 32 columns: [head][32]).
// The MMA warp runs a non-blocking scheduler over its three queues (PV first, then S,
// then the next tile's QKV in 4-MMA chunks), so the next tile's q / k / v epilogues
// overlap this tile's softmax. QKV never reaches HBM: per token the kernel reads the
// 384-byte X16 row (once from HBM; the pair's two sibling CTAs hit L2) and writes its
// pair's 128 bytes of the AO row. Every wait is bounded; the TMEM is always released.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace s2s {
namespace {

constexpr int kQaThreads = 576;  // TMA, MMA, E1 (4 warps), E2 (8), E3 (4)
constexpr int kQaHeads = 6;
constexpr int kQaGroups = 3;       // head pairs
constexpr int kBiasStride = 40;    // compact bias table: index 40 (dy + 7) + dx + 7
constexpr int kBiasPerHead = 576;  // >= 40 * 14 + 15
constexpr int kOffX = 0;           // X tile: 3 K-chunks of [128 tokens][64] fp16, SW128
constexpr int kOffW = 49152;       // the pair's Wqkv: 3 K-chunks of [192 rows][64] (resident)
constexpr int kOffQ = 122880;      // Q [128][32] fp16 in 128-byte swizzled rows
constexpr int kOffK = 139264;      // K, the same
constexpr int kOffP = 155648;      // P: 2 K-chunks (keys of window 0 / 1) of [128][64]
constexpr int kOffVt = 188416;     // V^T per head of the pair: 2 K-chunks (tokens) of [32][64]
constexpr int kOffBias = 204800;   // [2][576] fp32
constexpr int kOffVec = kOffBias + 2 * kBiasPerHead * 4;  // q bias, v bias [2][32], scale [2]
constexpr int kOffRed = kOffVec + 160 * 4;      // E2 partial max / sum [2][2][128]
constexpr int kOffBar = kOffRed + 512 * 4;
constexpr int kQaBars = 30;
constexpr size_t kQaSmem = 1024 + kOffBar + kQaBars * 8 + 16;
static_assert(kQaSmem <= 232448, "shared memory");

// In-window token i in box order -> its row / column in the 8 x 8 window.
__host__ __device__ constexpr int tok_y(int i) { return ((i >> 5) << 2) + ((i & 15) >> 2); }
__host__ __device__ constexpr int tok_x(int i) { return (((i >> 4) & 1) << 2) + (i & 3); }

__device__ __forceinline__ uint32_t h2u(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 18 warps: an SM sub-partition holds up to 5 of them, so 96 registers each
__global__ void __launch_bounds__(kQaThreads, 1)
    k_qkv_attention(const __grid_constant__ CUtensorMap mapX,
                    const __grid_constant__ CUtensorMap mapW, const QaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem + kOffX;
  uint8_t* sW = smem + kOffW;
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sP = smem + kOffP;
  uint8_t* sVt = smem + kOffVt;
  float* sBias = reinterpret_cast<float*>(smem + kOffBias);
  float* sQb = reinterpret_cast<float*>(smem + kOffVec);  // [2][32]
  float* sVb = sQb + 64;                                  // [2][32]
  float* sLs = sQb + 128;                                 // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* xfull = bars + 0;      // X tile landed
  uint64_t* xfree = bars + 1;      // the tile's QKV MMAs retired: X reusable
  uint64_t* wbar = bars + 2;       // Wqkv landed
  uint64_t* bbar = bars + 3;       // bias table landed
  uint64_t* qkv_acc = bars + 4;    // [2] QKV of head slot j accumulated
  uint64_t* qkready = bars + 6;    // [2] Q, K of slot j in shared; its q, k TMEM drained (4)
  uint64_t* s_acc = bars + 8;      // [2] S accumulated
  uint64_t* sfree = bars + 10;     // [2] S drained (4)
  uint64_t* s_done = bars + 12;    // an S retired: Q, K shared buffers reusable
  uint64_t* p_ready = bars + 13;   // P in shared (4)
  uint64_t* pv_done = bars + 14;   // a PV retired: P reusable
  uint64_t* vt_free = bars + 16;   // [2] PV of slot j retired: its V^T reusable
  uint64_t* o_acc = bars + 18;     // [2] O accumulated
  uint64_t* o_free = bars + 20;    // [2] O drained (4)
  uint64_t* fin = bars + 22;       // every MMA of the CTA retired
  uint64_t* vready = bars + 23;    // [2] V^T of slot j in shared; its v TMEM drained (4)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 25);
  float* sRed = reinterpret_cast<float*>(smem + kOffRed);  // [max|sum][half][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = (a.nwin_total + 1) / 2;
  const int grp = blockIdx.x % kQaGroups;       // head pair of this CTA
  const int t0 = blockIdx.x / kQaGroups;        // first tile
  const int tstep = gridDim.x / kQaGroups;      // host launches a multiple of 3 CTAs
  // TMEM columns: QKV [0, 192) (2 x 96), S [192, 448) (2 x 128), O [448, 512) (2 x 32)
  constexpr uint32_t kTmQKV = 0, kTmS = 192, kTmO = 448;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mapX);
    tma_prefetch_desc(&mapW);
    mbar_init(xfull, 1);
    mbar_init(xfree, 1);
    mbar_init(wbar, 1);
    mbar_init(bbar, 1);
    for (int j = 0; j < 2; j++) {
      mbar_init(&qkv_acc[j], 1);
      mbar_init(&qkready[j], 4);
      mbar_init(&s_acc[j], 1);
      mbar_init(&sfree[j], 8);
      mbar_init(&vt_free[j], 1);
      mbar_init(&o_acc[j], 1);
      mbar_init(&o_free[j], 4);
      mbar_init(&vready[j], 4);
    }
    mbar_init(s_done, 1);
    mbar_init(p_ready, 8);
    mbar_init(pv_done, 1);
    mbar_init(fin, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  // P rows keep zeros in the other window's key chunk: written once, never overwritten
  for (int i = threadIdx.x; i < 32768 / 16; i += kQaThreads)
    reinterpret_cast<uint4*>(sP)[i] = make_uint4(0u, 0u, 0u, 0u);
  // the pair's q / v biases and q scales (weights)
  if (threadIdx.x < 64) {
    sQb[threadIdx.x] = a.qb[grp * 64 + threadIdx.x];
    sVb[threadIdx.x] = a.vb[grp * 64 + threadIdx.x];
  }
  if (threadIdx.x < 2) sLs[threadIdx.x] = a.ls[2 * grp + threadIdx.x];
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_trigger();
  // weights and the bias table load while the previous kernel finishes
  if (warp == 0 && lane == 0) {
    mbar_arrive_expect_tx(wbar, 3 * 24576);
    for (int c = 0; c < 3; c++) tma_load_2d(sW + c * 24576, &mapW, wbar, c * 64, grp * 192);
    mbar_arrive_expect_tx(bbar, 2 * kBiasPerHead * 4);
    bulk_g2s(sBias, a.bias + grp * 2 * kBiasPerHead, 2 * kBiasPerHead * 4, bbar);
  }
  pdl_wait();  // X16 (the previous kernel's output) is complete

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int i = 0;
      for (int t = t0; t < num_tiles; t += tstep, i++) {
        if (i > 0 && !mbar_wait(xfree, (i - 1) & 1, DEV_TIMEOUT_EMPTY)) break;
        mbar_arrive_expect_tx(xfull, 49152);
        for (int w = 0; w < 2; w++) {
          const int W = 2 * t + w;
          int img = a.B, y0b = 0, x0b = 0;  // a missing second window: zero fill
          if (W < a.nwin_total) {
            img = W / a.nw_img;
            const int wi = W - img * a.nw_img;
            const int wh = wi / a.nww, ww = wi - wh * a.nww;
            y0b = a.y_base + wh * 8;
            x0b = ww * 8 + a.shift;
          }
          for (int b = 0; b < 4; b++) {
            int y0 = y0b + (b >> 1) * 4;
            if (y0 >= a.y_mod) y0 -= a.y_mod;
            int x0 = x0b + (b & 1) * 4;
            if (x0 >= a.wp) x0 -= a.wp;
            for (int c = 0; c < 3; c++)
              tma_load_4d(sX + c * 16384 + (w * 64 + b * 16) * 128, &mapX, xfull, c * 64, x0, y0,
                          img);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t id_qkv = idesc_f16_f32(128, 96), id_s = idesc_f16_f32(128, 128);
      constexpr uint32_t id_o = idesc_f16_f32(128, 32);
      bool ok = mbar_wait(wbar, 0, DEV_TIMEOUT_FULL);
      tc_fence_after();
      // A non-blocking scheduler over three queues, each in its own order: PV(i, j)
      // first (the softmax -> output chain waits on it), then S(i, j), then the QKV of
      // the tiles in 4-MMA chunks (an MMA issue blocks while the pipe is full, so a
      // whole tile's QKV issued at once would hold the PVs back). Every barrier is
      // tested only for its next completion, in order.
      int n_items = 0;
      for (int t = t0; t < num_tiles; t += tstep) n_items++;
      int iS = 0, jS = 0, iP = 0, jP = 0, iQ = 0, gQ = 0;  // next S, PV, QKV chunk group
      uint32_t vseen[2] = {0u, 0u}, xseen = 0u;            // completions observed
      uint64_t t_idle = 0;
      uint32_t spins = 0;
      while (ok && iP < n_items) {
        bool did = false;
        // ---- PV(iP, jP): P written, the O slot drained, V^T in shared
        if (iS > iP || (iS == iP && jS > jP)) {  // S(iP, jP) issued
          bool ready = mbar_test(p_ready, (uint32_t)(2 * iP + jP) & 1);
          if (ready && iP > 0) ready = mbar_test(&o_free[jP], (uint32_t)(iP - 1) & 1);
          if (ready && vseen[jP] == (uint32_t)iP) {
            ready = mbar_test(&vready[jP], (uint32_t)iP & 1);
            if (ready) vseen[jP]++;
          }
          if (ready && vseen[jP] > (uint32_t)iP) {
            tc_fence_after();
            const uint32_t d = tmem + kTmO + jP * 32;
#pragma unroll
            for (int c = 0; c < 2; c++) {
              const uint64_t ad = sw128_desc(smem_u32(sP + c * 16384));
              const uint64_t bd = sw128_desc(smem_u32(sVt + jP * 8192 + c * 4096));
#pragma unroll
              for (int kk = 0; kk < 4; kk++)
                tc_mma_f16(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), id_o,
                           (c | kk) != 0 ? 1u : 0u);
            }
            tc_commit(pv_done);
            tc_commit(&vt_free[jP]);
            tc_commit(&o_acc[jP]);
            if (++jP == 2) {
              jP = 0;
              iP++;
            }
            did = true;
          }
        }
        // ---- S(iS, jS): Q, K in shared (tile iS's QKV of the head issued), S slot drained
        if (!did && iS < n_items && (iQ > iS || (iQ == iS && gQ >= 3 * (jS + 1)))) {
          bool ready = mbar_test(&qkready[jS], (uint32_t)iS & 1);
          if (ready && iS > 0) ready = mbar_test(&sfree[jS], (uint32_t)(iS - 1) & 1);
          if (ready) {
            tc_fence_after();
            const uint32_t d = tmem + kTmS + jS * 128;
            const uint64_t ad = sw128_desc(smem_u32(sQ)), bd = sw128_desc(smem_u32(sK));
            tc_mma_f16(d, ad, bd, id_s, 0u);
            tc_mma_f16(d, ad + 2, bd + 2, id_s, 1u);
            tc_commit(&s_acc[jS]);
            tc_commit(s_done);
            if (++jS == 2) {
              jS = 0;
              iS++;
            }
            did = true;
          }
        }
        // ---- QKV chunk group gQ (head gQ / 3, K-chunk gQ % 3) of tile iQ: X landed;
        // the slot's previous contents drained (q, k: S(iQ - 1, j) issued, which waited
        // for qkready; v: vready)
        if (!did && iQ < n_items) {
          const int j = gQ / 3, c = gQ % 3;
          bool ready = true;
          if (gQ == 0 && xseen == (uint32_t)iQ) {
            ready = mbar_test(xfull, (uint32_t)iQ & 1);
            if (ready) xseen++;
          }
          ready = ready && xseen > (uint32_t)iQ;
          if (ready && c == 0 && iQ > 0) {
            ready = iS > iQ - 1 || (iS == iQ - 1 && jS > j);
            if (ready && vseen[j] == (uint32_t)(iQ - 1)) {
              ready = mbar_test(&vready[j], (uint32_t)(iQ - 1) & 1);
              if (ready) vseen[j]++;
            }
            ready = ready && vseen[j] >= (uint32_t)iQ;
          }
          if (ready) {
            tc_fence_after();
            const uint32_t d = tmem + kTmQKV + j * 96;
            const uint64_t ad = sw128_desc(smem_u32(sX + c * 16384));
            const uint64_t bd = sw128_desc(smem_u32(sW + c * 24576 + j * 12288));
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              tc_mma_f16(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), id_qkv,
                         (c | kk) != 0 ? 1u : 0u);
            if (c == 2) tc_commit(&qkv_acc[j]);
            if (++gQ == 6) {
              tc_commit(xfree);
              gQ = 0;
              iQ++;
            }
            did = true;
          }
        }
        if (did) {
          t_idle = 0;
          spins = 0;
        } else {
          // back off: the epilogue warps sharing this warp's sub-partition need its
          // issue slots more than an idle poll does
          __nanosleep(64);
        }
        if (!did && (++spins & 255u) == 0) {
          const uint64_t now = global_timer_ns();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > 2000000000ull) {
            record_error(DEV_TIMEOUT_ACC);
            ok = false;
          }
          if (*(volatile unsigned*)&g_s2s_err != 0u) ok = false;
        }
      }
      tc_commit(fin);
      mbar_wait(fin, 0, DEV_TIMEOUT_ACC);
    }
  } else if (warp < 6) {
    // -------------------------------------------------------------- E1: Q, K
    const int q = warp & 3;
    const int r = q * 32 + lane;  // TMEM lane = tile row (token)
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    int i = 0;
    bool ok = true;
    for (int t = t0; t < num_tiles && ok; t += tstep, i++) {
      for (int j = 0; j < 2; j++) {
        if (!mbar_wait(&qkv_acc[j], i & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // F.normalize per head (eps 1e-12), q also times the clamped logit scale log2 e;
        // the squares in four partial sums; each part packed to fp16 as soon as scaled
        uint32_t hq[16], hk[16];
#pragma unroll
        for (int part = 0; part < 2; part++) {
          uint32_t v[32];
          tmem_ld32_nw(tq + kTmQKV + j * 96 + part * 32, v);
          tc_wait_ld();
          float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int e = 0; e < 32; e++) {
            float x = __uint_as_float(v[e]);
            if (part == 0) x += sQb[j * 32 + e];
            v[e] = __float_as_uint(x);
            s4[e & 3] = fmaf(x, x, s4[e & 3]);
          }
          float rs = 1.0f / fmaxf(sqrtf((s4[0] + s4[1]) + (s4[2] + s4[3])), 1e-12f);
          if (part == 0) rs *= sLs[j];
          uint32_t* hp = part == 0 ? hq : hk;
#pragma unroll
          for (int e = 0; e < 16; e++)
            hp[e] = h2u(__uint_as_float(v[2 * e]) * rs, __uint_as_float(v[2 * e + 1]) * rs);
        }
        // Q and K shared buffers are free once the previous S retired
        const int sd = 2 * i + j;
        if (sd > 0 && !mbar_wait(s_done, (uint32_t)(sd - 1) & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        uint8_t* qrow = sQ + r * 128;
        uint8_t* krow = sK + r * 128;
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int off = (c ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(qrow + off) =
              make_uint4(hq[4 * c], hq[4 * c + 1], hq[4 * c + 2], hq[4 * c + 3]);
          *reinterpret_cast<uint4*>(krow + off) =
              make_uint4(hk[4 * c], hk[4 * c + 1], hk[4 * c + 2], hk[4 * c + 3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&qkready[j]);
      }
    }
  } else if (warp < 14) {
    // -------------------------------------------------------------- E2: softmax
    // two warps per TMEM lane quarter, each with 32 of the row's 64 keys; the row's
    // max and sum combine through shared memory (named barrier 1 + q, 64 threads)
    const int q = warp & 3;
    const int kh = (warp - 6) >> 2;        // key half
    const int r = q * 32 + lane;
    const int wsel = r >> 6, ii = r & 63;  // window of the row, its in-window token
    const int ty = tok_y(ii), tx = tok_x(ii);
    // keys kh * 32 + kk: rows 4 kh + .. of the window, so the bias base moves 160 kh
    const float* bq = sBias + kBiasStride * (ty + 7) + tx + 7 - kBiasStride * 4 * kh;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + kTmS + wsel * 64 + kh * 32;
    float* redm = sRed + r;          // [half][128] at redm + 128 * half
    float* reds = sRed + 256 + r;
    constexpr float kMask = -100.0f * 1.4426950408889634f;  // -100, in the exp2 domain
    const int nwh_g = a.ghp / 8;
    bool ok = mbar_wait(bbar, 0, DEV_TIMEOUT_FULL);
    int i = 0;
    for (int t = t0; t < num_tiles && ok; t += tstep, i++) {
      const int W = 2 * t + wsel;
      // shifted blocks: only the last window row and column mix roll regions; bit k
      // of mbits: key k lies in another region than this row's token
      bool masked = false;
      uint64_t mbits = 0;
      if (a.shift && W < a.nwin_total) {
        const int img = W / a.nw_img, wi = W - img * a.nw_img;
        const int wh = wi / a.nww;
        const int ww = wi - wh * a.nww;
        int whg = wh + a.wh_off;
        if (whg < 0) whg += nwh_g;
        masked = whg == nwh_g - 1 || ww == a.nww - 1;
        if (masked) {
          const int qreg = 3 * region_of(whg * 8 + ty, a.ghp, 8, a.shift) +
                           region_of(ww * 8 + tx, a.wp, 8, a.shift);
#pragma unroll
          for (int k = 0; k < 64; k++) {
            const int kr = 3 * region_of(whg * 8 + tok_y(k), a.ghp, 8, a.shift) +
                           region_of(ww * 8 + tok_x(k), a.wp, 8, a.shift);
            if (kr != qreg) mbits |= 1ull << k;
          }
        }
      }
      const uint32_t mb = (uint32_t)(mbits >> (32 * kh));
      for (int j = 0; j < 2; j++) {
        if (!mbar_wait(&s_acc[j], i & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[32];
        tmem_ld32_nw(tq + j * 128, sv);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[j]);
        const float* bt = bq + j * kBiasPerHead;
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int k = 0; k < 32; k++) {
          float x = __uint_as_float(sv[k]) + bt[-(kBiasStride * tok_y(k) + tok_x(k))];
          if (masked && ((mb >> k) & 1)) x += kMask;
          sv[k] = __float_as_uint(x);
          m4[k & 3] = fmaxf(m4[k & 3], x);
        }
        redm[128 * kh] = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
        const float mx = fmaxf(redm[0], redm[128]);
        float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k = 0; k < 32; k++) {
          const float e = ex2(__uint_as_float(sv[k]) - mx);
          sv[k] = __float_as_uint(e);
          s4[k & 3] += e;
        }
        reds[128 * kh] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
        asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
        const float inv = 1.0f / (reds[0] + reds[128]);
        // P is free once the previous PV retired
        const int pd = 2 * i + j;
        if (pd > 0 && !mbar_wait(pv_done, (uint32_t)(pd - 1) & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        uint8_t* prow = sP + wsel * 16384 + r * 128;
#pragma unroll
        for (int m = 0; m < 4; m++) {
          const float* f = reinterpret_cast<const float*>(sv + 8 * m);
          uint4 u;
          u.x = h2u(f[0] * inv, f[1] * inv);
          u.y = h2u(f[2] * inv, f[3] * inv);
          u.z = h2u(f[4] * inv, f[5] * inv);
          u.w = h2u(f[6] * inv, f[7] * inv);
          *reinterpret_cast<uint4*>(prow + (((kh * 4 + m) ^ (r & 7)) << 4)) = u;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
      }
    }
  } else {
    // -------------------------------------------------------------- E3: V^T, output
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int wsel = r >> 6, ii = r & 63;
    const int ty = tok_y(ii), tx = tok_x(ii);
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    // V^T element (d, r): K-chunk r / 64, row d, 16-byte piece (r % 64) / 8 swizzled by
    // d % 8, half r % 8
    const int vpiece = (r & 63) >> 3, vhalf = r & 7;
    int i = 0;
    bool ok = true;
    for (int t = t0; t < num_tiles && ok; t += tstep, i++) {
      // v + v_bias of both slots, transposed into V^T; a slot's V^T is free once its
      // previous PV retired
      for (int j = 0; j < 2; j++) {
        if (!mbar_wait(&qkv_acc[j], i & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32_nw(tq + kTmQKV + j * 96 + 64, v);
        tc_wait_ld();
        tc_fence_before();
        if (i > 0 && !mbar_wait(&vt_free[j], (i - 1) & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        __half* vt = reinterpret_cast<__half*>(sVt + j * 8192 + wsel * 4096);
#pragma unroll
        for (int d = 0; d < 32; d++)
          vt[d * 64 + ((vpiece ^ (d & 7)) << 3) + vhalf] =
              __float2half_rn(__uint_as_float(v[d]) + sVb[j * 32 + d]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&vready[j]);
      }
      if (!ok) break;
      const int W = 2 * t + wsel;
      const bool valid = W < a.nwin_total;
      size_t orow = 0;
      if (valid) {
        const int img = W / a.nw_img, wi = W - img * a.nw_img;
        const int wh = wi / a.nww, ww = wi - wh * a.nww;
        int y = a.y_base + wh * 8 + ty;
        if (y >= a.y_mod) y -= a.y_mod;
        int x = ww * 8 + tx + a.shift;
        if (x >= a.wp) x -= a.wp;
        orow = ((size_t)img * a.hp_l + y) * a.wp + x;
      }
      __half* dst = a.out + orow * a.ld_out;
      for (int j = 0; j < 2; j++) {
        if (!mbar_wait(&o_acc[j], i & 1, DEV_TIMEOUT_ACC)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t o[32];
        tmem_ld32_nw(tq + kTmO + j * 32, o);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[j]);
        if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + (2 * grp + j) * 32);
#pragma unroll
          for (int c = 0; c < 4; c++) {
            uint4 u;
            u.x = h2u(__uint_as_float(o[8 * c]), __uint_as_float(o[8 * c + 1]));
            u.y = h2u(__uint_as_float(o[8 * c + 2]), __uint_as_float(o[8 * c + 3]));
            u.z = h2u(__uint_as_float(o[8 * c + 4]), __uint_as_float(o[8 * c + 5]));
            u.w = h2u(__uint_as_float(o[8 * c + 6]), __uint_as_float(o[8 * c + 7]));
            d4[c] = u;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t launch_qkv_attention(const CUtensorMap& mapX, const CUtensorMap& mapW,
                                 const QaArgs& a, cudaStream_t st) {
  if (a.nwin_total < 1 || a.ld_out < kQaHeads * 32 || (a.ld_out % 8) ||
      (reinterpret_cast<uintptr_t>(a.out) & 15) || (reinterpret_cast<uintptr_t>(a.bias) & 15) ||
      a.nww < 1 || a.wp % 8 || a.y_mod < 8)
    return cudaErrorInvalidValue;
  static LaunchSetup setup;  // resident CTAs, per device
  int ctas = 0;
  const cudaError_t err = resident_ctas(setup, k_qkv_attention, kQaThreads, kQaSmem, &ctas);
  if (err != cudaSuccess) return err;
  // CTAs in head-pair triples; each walks tiles with its pair's weights resident
  const long tiles = (a.nwin_total + 1) / 2;
  long G = ctas / kQaGroups;
  if (G > tiles) G = tiles;
  G *= kQaGroups;
  return launch_pdl(k_qkv_attention, dim3((unsigned)G), dim3(kQaThreads), kQaSmem, st, mapX, mapW,
                    a);
}

// The compact relative-position bias table the fused kernel reads, from the expanded
// [heads][64][64] table (columns XOR-swizzled by row % 8): entry 40 (dy + 7) + dx + 7
// is the bias of any query/key pair at offset (dy, dx) = query - key. Thread per entry.
__global__ void k_cpb_compact(const float* __restrict__ full, float* __restrict__ compact,
                              int heads) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * kBiasPerHead) return;
  const int h = i / kBiasPerHead, e = i % kBiasPerHead;
  const int dy = e / kBiasStride - 7, dx = e % kBiasStride - 7;
  float v = 0.0f;
  if (dy <= 7 && dx <= 7) {
    const int qy = dy > 0 ? dy : 0, qx = dx > 0 ? dx : 0;
    const int qi = qy * 8 + qx, ki = (qy - dy) * 8 + (qx - dx);
    v = full[((size_t)h * 64 + qi) * 64 + (ki ^ ((qi & 7) << 2))];
  }
  compact[i] = v;
}

cudaError_t launch_cpb_compact(const float* full, float* compact, int heads, cudaStream_t st) {
  const int n = heads * kBiasPerHead;
  k_cpb_compact<<<(n + 255) / 256, 256, 0, st>>>(full, compact, heads);
  return cudaGetLastError();
}

}  // namespace s2s
