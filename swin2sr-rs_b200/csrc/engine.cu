// The forward pass behind the C ABI of include/s2s.h.
//
// Layout in HBM (per plan of B images, padded hp x wp, T = B*hp*wp tokens):
//   residual stream X      fp32 [T][Cp] rows in image order (row b*hp*wp + y*wp + x),
//                          updated in place by the epilogues of proj and fc2;
//   X16                    fp16 copy of X, the A operand of the next GEMM / conv;
//   window order           exists only inside the attention kernel, which gathers and
//                          scatters token rows through the shift's row table (the
//                          window partition and roll of src/cpu.rs:1148-1222);
//   conv planes            NHWC fp16 [B][H][W][Cp], read by 4-D TMA boxes.
// Cp = embed padded to 64 (pad lanes hold zeros), head_dim padded to DP = 16/32.
//
// Per block (src/cpu.rs:1516-1575): QKV GEMM -> window attention -> proj GEMM with
// norm1 + residual -> fc1 GEMM + GELU -> fc2 GEMM with norm2 + residual.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <array>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "s2s.h"

namespace s2s {
cudaError_t launch_window_attention(const __half* qkv, __half* out, const float* cpb,
                                    const float* lscale, const int* rows, int nwin_total,
                                    int heads, int hd, int dp, int ld_out, int nwh, int nww,
                                    int hp, int wp, int shift, cudaStream_t st);
cudaError_t launch_pad_reflect(const float* x, float* y, int B, int c, int h, int w, int hp,
                               int wp, cudaStream_t st);
cudaError_t launch_conv3_small(const float* in, const float* wgt, const float* bias, int B, int H,
                               int W, int co_n, int act, float slope, float* o32, int ld32,
                               __half* o16, int ld16, cudaStream_t st);
cudaError_t launch_zero_cols_f16(__half* x, size_t rows, int c0, int ld, cudaStream_t st);
cudaError_t launch_bicubic(const float* in, float* out, int BC, int h, int w, int oh, int ow,
                           cudaStream_t st);
cudaError_t launch_up2_nhwc(const __half* in, __half* out, int B, int H, int W, int C,
                            cudaStream_t st);
}  // namespace s2s

using namespace s2s;

namespace {

thread_local std::string g_create_error;

struct S2SError {
  int code;
  std::string msg;
};

[[noreturn]] void fail(int code, const std::string& m) { throw S2SError{code, m}; }

void ck(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return;
  if (e == cudaErrorMemoryAllocation)
    fail(S2S_ERR_OOM, std::string(what) + ": CUDA_ERROR_OUT_OF_MEMORY (out of memory)");
  fail(S2S_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

inline int pad_to(int x, int m) { return (x + m - 1) / m * m; }

// A tensor-core operand: fp16 [N][K] K-major weights, fp32 bias, and its TMA map.
struct TcWeight {
  __half* w = nullptr;
  float* b = nullptr;
  int N = 0, K = 0, BN = 0;
  CUtensorMap map;
};

struct Block {
  TcWeight qkv, proj, fc1, fc2;
  float *n1g, *n1b, *n2g, *n2b, *cpb, *ls;
};

struct Stage {
  std::vector<Block> blocks;
  TcWeight conv, pe;
};

// Activation workspace for one (B, h, w).
struct Plan {
  int B = 0, h = 0, w = 0, hp = 0, wp = 0;
  size_t T = 0;
  std::vector<void*> allocs;
  size_t bytes = 0;
  float *P = nullptr, *F0 = nullptr, *X = nullptr, *S = nullptr;
  __half *F0h = nullptr, *X16 = nullptr, *QKV = nullptr, *AO = nullptr, *H16 = nullptr;
  __half *HA = nullptr, *HB[3] = {nullptr, nullptr, nullptr};
  float *BIC = nullptr, *BICF = nullptr, *AUXRAW = nullptr;
  int* rows[2] = {nullptr, nullptr};  // window-major token -> image row, shift 0 / win/2
  CUtensorMap mF0h, mX16, mAO, mH16, cX16, cAO, cHA;
  CUtensorMap cHB[3][3];  // head planes at 1x, 2x, 4x resolution
  // Output / residual TMA maps, built on first use for each (buffer, geometry).
  std::map<std::array<int64_t, 8>, CUtensorMap> omaps;
};

struct ProfEntry {
  const char* name;
  cudaEvent_t a, b;
};

}  // namespace

struct s2s_handle {
  int device = 0;
  s2s_config cfg;
  int C = 0, Cp = 0, heads = 0, hd = 0, DP = 0, NQ = 0, HIDp = 0, feat = 64;
  float* cf_w = nullptr;
  float* cf_b = nullptr;
  TcWeight pe;
  float *pe_g = nullptr, *pe_b = nullptr, *nrm_g = nullptr, *nrm_b = nullptr;
  std::vector<Stage> stages;
  TcWeight cab;
  TcWeight cbu, oct[3], last, direct, aux, up1, up2, hr;
  float *cbic_w = nullptr, *cbic_b = nullptr, *caa_w = nullptr, *caa_b = nullptr;
  std::vector<void*> wallocs;
  size_t uploaded = 0;
  std::unique_ptr<Plan> plan;
  std::string err;
  cudaStream_t stream = nullptr;
  float *h_in = nullptr, *h_out = nullptr, *h_aux = nullptr;  // device staging for host calls
  size_t h_in_n = 0, h_out_n = 0, h_aux_n = 0;
  bool profiling = false;
  std::string prof_only;  // profile only kernel classes with this prefix
  std::vector<ProfEntry> prof_pending;
  std::vector<cudaEvent_t> ev_pool;
  std::map<std::string, std::pair<long, double>> prof;
  long long launches = 0;
  bool fused_mlp = false;      // (Cp, HIDp) has a fused MLP kernel
  long long stop_after = -1;   // diagnostics: launches per forward before stopping
  long long fwd_launches = 0;  // launches enqueued by the forward in flight
};

namespace {

// ------------------------------------------------------------------ weights
struct TensorTable {
  std::map<std::string, const s2s_tensor*> t;
  const float* get(const std::string& n, int64_t expect_numel = -1) const {
    auto it = t.find(n);
    if (it == t.end()) fail(S2S_ERR_INVALID, "missing tensor `" + n + "`");
    const s2s_tensor* x = it->second;
    int64_t numel = 1;
    for (int i = 0; i < x->ndim; i++) numel *= x->shape[i];
    if (expect_numel >= 0 && numel != expect_numel)
      fail(S2S_ERR_INVALID, "tensor `" + n + "` has " + std::to_string(numel) +
                                " values, the architecture implies " +
                                std::to_string(expect_numel));
    return x->data;
  }
  bool has(const std::string& n) const { return t.count(n) != 0; }
};

template <typename T>
T* upload(s2s_handle* H, const std::vector<T>& v) {
  void* p = nullptr;
  ck(cudaMalloc(&p, v.size() * sizeof(T)), "weight upload");
  H->wallocs.push_back(p);
  ck(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), "weight upload");
  H->uploaded += v.size() * sizeof(T);
  return static_cast<T*>(p);
}

void finish_tc(s2s_handle* H, TcWeight& tw, const std::vector<__half>& w, const std::vector<float>& b,
               int N, int K, int BN) {
  tw.N = N;
  tw.K = K;
  tw.BN = BN;
  tw.w = upload(H, w);
  tw.b = upload(H, b);
  if (!make_map_rows(&tw.map, tw.w, (uint64_t)N, (uint64_t)K, (uint32_t)BN))
    fail(S2S_ERR_CUDA, "cuTensorMapEncodeTiled failed for a weight operand");
}

// Linear [n_out][n_in] -> fp16 [N][K] with row remap (dst row -> src row or -1).
void pack_linear(s2s_handle* H, TcWeight& tw, const float* W, const float* bias, int n_in, int N,
                 int K, int BN, const std::vector<int>& rowmap) {
  std::vector<__half> w((size_t)N * K, __float2half(0.0f));
  std::vector<float> b(N, 0.0f);
  for (int r = 0; r < N; r++) {
    const int s = rowmap[r];
    if (s < 0) continue;
    for (int k = 0; k < n_in; k++) w[(size_t)r * K + k] = __float2half_rn(W[(size_t)s * n_in + k]);
    if (bias) b[r] = bias[s];
  }
  finish_tc(H, tw, w, b, N, K, BN);
}

// Conv3x3 [co][ci][3][3] -> fp16 [N][9*Cip], K index = (ky*3+kx)*Cip + c.
void pack_conv(s2s_handle* H, TcWeight& tw, const float* W, const float* bias, int ci, int Cip,
               int N, int BN, const std::vector<int>& rowmap) {
  const int K = 9 * Cip;
  std::vector<__half> w((size_t)N * K, __float2half(0.0f));
  std::vector<float> b(N, 0.0f);
  for (int r = 0; r < N; r++) {
    const int s = rowmap[r];
    if (s < 0) continue;
    for (int c = 0; c < ci; c++)
      for (int t = 0; t < 9; t++)
        w[(size_t)r * K + t * Cip + c] = __float2half_rn(W[((size_t)s * ci + c) * 9 + t]);
    b[r] = bias[s];
  }
  finish_tc(H, tw, w, b, N, K, BN);
}

std::vector<int> identity_rows(int N, int valid) {
  std::vector<int> m(N, -1);
  for (int i = 0; i < valid; i++) m[i] = i;
  return m;
}

std::vector<float> padded(const float* x, int n, int np) {
  std::vector<float> v(np, 0.0f);
  for (int i = 0; i < n; i++) v[i] = x[i];
  return v;
}

int n_tile_for(int N) {
  for (int bn : {256, 192, 128, 96, 64, 32})
    if (N % bn == 0 && N / bn <= 4) return bn;
  return 32;
}

void build_weights(s2s_handle* H, const TensorTable& T) {
  const s2s_config& c = H->cfg;
  const int C = c.embed, Cp = H->Cp, hd = H->hd, DP = H->DP, heads = H->heads;
  const int HID = c.mlp_ratio * C, HIDp = H->HIDp;
  const int n = c.window * c.window;
  // top
  H->cf_w = upload(H, std::vector<float>(T.get("conv_first.weight", (int64_t)C * 27),
                                         T.get("conv_first.weight") + (size_t)C * 27));
  H->cf_b = upload(H, std::vector<float>(T.get("conv_first.bias", C), T.get("conv_first.bias") + C));
  pack_linear(H, H->pe, T.get("patch_embed.proj.weight", (int64_t)C * C),
              T.get("patch_embed.proj.bias", C), C, Cp, Cp, Cp, identity_rows(Cp, C));
  H->pe_g = upload(H, padded(T.get("patch_embed.norm.weight", C), C, Cp));
  H->pe_b = upload(H, padded(T.get("patch_embed.norm.bias", C), C, Cp));
  H->nrm_g = upload(H, padded(T.get("norm.weight", C), C, Cp));
  H->nrm_b = upload(H, padded(T.get("norm.bias", C), C, Cp));
  pack_conv(H, H->cab, T.get("conv_after_body.weight", (int64_t)C * C * 9),
            T.get("conv_after_body.bias", C), C, Cp, Cp, Cp, identity_rows(Cp, C));
  // stages
  H->stages.resize(c.n_depths);
  std::vector<float> zeros(C, 0.0f);
  for (int s = 0; s < c.n_depths; s++) {
    Stage& st = H->stages[s];
    st.blocks.resize(c.depths[s]);
    for (int b = 0; b < c.depths[s]; b++) {
      Block& bl = st.blocks[b];
      char pfx[96];
      snprintf(pfx, sizeof pfx, "layers.%d.residual_group.blocks.%d.", s, b);
      const std::string p(pfx);
      // QKV: rows [heads][q|k|v][DP] <- [3C] (q, k, v), pad lanes zero, so one head's
      // q, k and v of a token are one contiguous run for the attention kernel.
      const float* wq = T.get(p + "attn.qkv.wq", (int64_t)C * C);
      const float* wk = T.get(p + "attn.qkv.wk", (int64_t)C * C);
      const float* wv = T.get(p + "attn.qkv.wv", (int64_t)C * C);
      const float* qb = T.get(p + "attn.qkv.q_bias", C);
      const float* vb = T.get(p + "attn.qkv.v_bias", C);
      std::vector<float> W3((size_t)3 * C * C), b3(3 * C, 0.0f);
      memcpy(&W3[0], wq, sizeof(float) * C * C);
      memcpy(&W3[(size_t)C * C], wk, sizeof(float) * C * C);
      memcpy(&W3[(size_t)2 * C * C], wv, sizeof(float) * C * C);
      for (int i = 0; i < C; i++) {
        b3[i] = qb[i];
        b3[2 * C + i] = vb[i];
      }
      std::vector<int> qmap(H->NQ, -1);
      for (int part = 0; part < 3; part++)
        for (int h = 0; h < heads; h++)
          for (int d = 0; d < hd; d++) qmap[(h * 3 + part) * DP + d] = part * C + h * hd + d;
      pack_linear(H, bl.qkv, W3.data(), b3.data(), C, H->NQ, Cp, n_tile_for(H->NQ), qmap);
      pack_linear(H, bl.proj, T.get(p + "attn.proj.weight", (int64_t)C * C),
                  T.get(p + "attn.proj.bias", C), C, Cp, Cp, Cp, identity_rows(Cp, C));
      pack_linear(H, bl.fc1, T.get(p + "mlp.fc1.weight", (int64_t)HID * C),
                  T.get(p + "mlp.fc1.bias", HID), C, HIDp, Cp, n_tile_for(HIDp),
                  identity_rows(HIDp, HID));
      pack_linear(H, bl.fc2, T.get(p + "mlp.fc2.weight", (int64_t)C * HID),
                  T.get(p + "mlp.fc2.bias", C), HID, Cp, HIDp, Cp, identity_rows(Cp, C));
      bl.n1g = upload(H, padded(T.get(p + "norm1.weight", C), C, Cp));
      bl.n1b = upload(H, padded(T.get(p + "norm1.bias", C), C, Cp));
      bl.n2g = upload(H, padded(T.get(p + "norm2.weight", C), C, Cp));
      bl.n2b = upload(H, padded(T.get(p + "norm2.bias", C), C, Cp));
      // cpb_pre [N*N][heads] -> [heads][N][N + 8] (rows padded so that the attention
      // kernel's shared-memory reads are free of bank conflicts); logit scale ->
      // exp(min(ls, ln 100)).
      const float* cpb = T.get(p + "attn.cpb_pre", (int64_t)n * n * heads);
      const int ns = n + 8;
      std::vector<float> cpbt((size_t)heads * n * ns, 0.0f);
      for (int q = 0; q < n; q++)
        for (int k = 0; k < n; k++)
          for (int h = 0; h < heads; h++)
            cpbt[((size_t)h * n + q) * ns + k] = cpb[((size_t)q * n + k) * heads + h];
      bl.cpb = upload(H, cpbt);
      const float* ls = T.get(p + "attn.logit_scale", heads);
      std::vector<float> lse(heads);
      for (int h = 0; h < heads; h++) lse[h] = std::exp(std::fmin(ls[h], std::log(100.0f)));
      bl.ls = upload(H, lse);
    }
    char cn[64], pn[64], cb[64], pb[64];
    snprintf(cn, sizeof cn, "layers.%d.conv.weight", s);
    snprintf(cb, sizeof cb, "layers.%d.conv.bias", s);
    snprintf(pn, sizeof pn, "layers.%d.patch_embed.proj.weight", s);
    snprintf(pb, sizeof pb, "layers.%d.patch_embed.proj.bias", s);
    pack_conv(H, st.conv, T.get(cn, (int64_t)C * C * 9), T.get(cb, C), C, Cp, Cp, Cp,
              identity_rows(Cp, C));
    pack_linear(H, st.pe, T.get(pn, (int64_t)C * C), T.get(pb, C), C, Cp, Cp, Cp,
                identity_rows(Cp, C));
  }
  // head
  const int F = H->feat;
  auto conv_plain = [&](TcWeight& tw, const std::string& name, int ci, int Cip, int co, int N) {
    pack_conv(H, tw, T.get(name + ".weight", (int64_t)co * ci * 9), T.get(name + ".bias", co), ci,
              Cip, N, n_tile_for(N), identity_rows(N, co));
  };
  auto conv_shuffle = [&](TcWeight& tw, const std::string& name) {
    // GEMM column n = (2dy+dx)*F + f  <-  conv output channel 4f + 2dy + dx.
    std::vector<int> m(4 * F);
    for (int q = 0; q < 4; q++)
      for (int f = 0; f < F; f++) m[q * F + f] = 4 * f + q;
    pack_conv(H, tw, T.get(name + ".weight", (int64_t)4 * F * F * 9), T.get(name + ".bias", 4 * F),
              F, F, 4 * F, 4 * F, m);
  };
  const int octs = (int)std::lround(std::log2((double)c.scale));
  switch (c.upsampler) {
    case S2S_PIXELSHUFFLE:
    case S2S_PIXELSHUFFLE_AUX:
      conv_plain(H->cbu, "conv_before_upsample.0", C, Cp, F, F);
      for (int o = 0; o < octs; o++) conv_shuffle(H->oct[o], "upsample." + std::to_string(2 * o));
      conv_plain(H->last, "conv_last", F, F, 3, 32);
      if (c.upsampler == S2S_PIXELSHUFFLE_AUX) {
        conv_plain(H->aux, "conv_aux", F, F, 3, 32);
        H->cbic_w = upload(H, std::vector<float>(T.get("conv_bicubic.weight", (int64_t)F * 27),
                                                 T.get("conv_bicubic.weight") + (size_t)F * 27));
        H->cbic_b = upload(H, std::vector<float>(T.get("conv_bicubic.bias", F),
                                                 T.get("conv_bicubic.bias") + F));
        H->caa_w = upload(H, std::vector<float>(T.get("conv_after_aux.0.weight", (int64_t)F * 27),
                                                T.get("conv_after_aux.0.weight") + (size_t)F * 27));
        H->caa_b = upload(H, std::vector<float>(T.get("conv_after_aux.0.bias", F),
                                                T.get("conv_after_aux.0.bias") + F));
      }
      break;
    case S2S_PIXELSHUFFLEDIRECT: {
      const int oc = 3 * c.scale * c.scale;
      conv_plain(H->direct, "upsample.0", C, Cp, oc, pad_to(oc, 32));
      break;
    }
    case S2S_NEARESTCONV:
      conv_plain(H->cbu, "conv_before_upsample.0", C, Cp, F, F);
      conv_plain(H->up1, "conv_up1", F, F, F, F);
      conv_plain(H->up2, "conv_up2", F, F, F, F);
      conv_plain(H->hr, "conv_hr", F, F, F, F);
      conv_plain(H->last, "conv_last", F, F, 3, 32);
      break;
    default:
      fail(S2S_ERR_UNSUPPORTED, "unknown upsampler");
  }
}

// ------------------------------------------------------------------ plans
void* dalloc(Plan& P, size_t bytes) {
  void* p = nullptr;
  ck(cudaMalloc(&p, bytes), "workspace");
  P.allocs.push_back(p);
  P.bytes += bytes;
  ck(cudaMemset(p, 0, bytes), "workspace clear");
  return p;
}

void free_plan(Plan& P) {
  for (void* p : P.allocs) cudaFree(p);
  P.allocs.clear();
}

// Pixel index (within image) read by window-major token r for shift s.
inline int token_pixel(int r, int hp, int wp, int s) {
  const int nww = wp / 8;
  const int wi = r / 64, t = r % 64;
  const int wh = wi / nww, ww = wi % nww;
  const int y = (wh * 8 + t / 8 + s) % hp;
  const int x = (ww * 8 + t % 8 + s) % wp;
  return y * wp + x;
}

int64_t plan_bytes(const s2s_handle* H, int B, int h, int w) {
  const int win = H->cfg.window;
  const int64_t hp = (h / win + 1) * win, wp = (w / win + 1) * win;
  const int64_t T = (int64_t)B * hp * wp;
  const int64_t Cp = H->Cp, s = H->cfg.scale;
  int64_t b = 0;
  b += (int64_t)B * 3 * hp * wp * 4;        // P
  b += 3 * T * Cp * 4;                      // F0, X, S
  b += 3 * T * Cp * 2;                      // F0h, X16, AO
  b += T * H->NQ * 2 + T * H->HIDp * 2;     // QKV, H16
  b += 2 * T * 4;                           // window row tables
  b += T * 64 * 2 + 3 * T * s * s * 64 * 2; // head planes
  if (H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX)
    b += (int64_t)B * 3 * hp * s * wp * s * 4 + T * s * s * 64 * 4 + (int64_t)B * 3 * hp * wp * 4;
  return b;
}

Plan* get_plan(s2s_handle* H, int B, int h, int w) {
  if (H->plan && H->plan->B == B && H->plan->h == h && H->plan->w == w) return H->plan.get();
  if (H->plan) {
    ck(cudaStreamSynchronize(H->stream), "plan change");
    free_plan(*H->plan);
    H->plan.reset();
  }
  std::unique_ptr<Plan> P(new Plan());
  const int win = H->cfg.window;
  P->B = B;
  P->h = h;
  P->w = w;
  P->hp = (h / win + 1) * win;
  P->wp = (w / win + 1) * win;
  const int hp = P->hp, wp = P->wp;
  const size_t T = (size_t)B * hp * wp;
  P->T = T;
  const int Cp = H->Cp, s = H->cfg.scale;
  try {
    P->P = (float*)dalloc(*P, (size_t)B * 3 * hp * wp * 4);
    P->F0 = (float*)dalloc(*P, T * Cp * 4);
    P->X = (float*)dalloc(*P, T * Cp * 4);
    P->S = (float*)dalloc(*P, T * Cp * 4);
    P->F0h = (__half*)dalloc(*P, T * Cp * 2);
    P->X16 = (__half*)dalloc(*P, T * Cp * 2);
    P->AO = (__half*)dalloc(*P, T * Cp * 2);
    P->QKV = (__half*)dalloc(*P, T * H->NQ * 2);
    P->H16 = (__half*)dalloc(*P, T * H->HIDp * 2);
    for (int i = 0; i < 2; i++) P->rows[i] = (int*)dalloc(*P, T * 4);
    P->HA = (__half*)dalloc(*P, T * 64 * 2);
    for (int i = 0; i < 3; i++) P->HB[i] = (__half*)dalloc(*P, T * s * s * 64 * 2);
    if (H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX) {
      P->BIC = (float*)dalloc(*P, (size_t)B * 3 * hp * s * wp * s * 4);
      P->BICF = (float*)dalloc(*P, T * s * s * 64 * 4);
      P->AUXRAW = (float*)dalloc(*P, (size_t)B * 3 * hp * wp * 4);
    }
  } catch (...) {
    free_plan(*P);
    throw;
  }
  // Window row tables (batch-offset): window-major token r of each image -> image row.
  {
    const int hw = hp * wp;
    std::vector<int> rt[2];
    for (auto& v : rt) v.resize(T);
    for (int b = 0; b < B; b++) {
      const int o = b * hw;
      for (int r = 0; r < hw; r++) {
        rt[0][o + r] = o + token_pixel(r, hp, wp, 0);
        rt[1][o + r] = o + token_pixel(r, hp, wp, win / 2);
      }
    }
    for (int i = 0; i < 2; i++)
      ck(cudaMemcpy(P->rows[i], rt[i].data(), T * 4, cudaMemcpyHostToDevice), "row table upload");
  }
  // TMA maps over the activation buffers.
  bool ok = true;
  ok &= make_map_rows(&P->mF0h, P->F0h, T, Cp, 128);
  {
    ok &= make_map_rows(&P->mX16, P->X16, T, Cp, 128);
    int bw, bh;
    conv_box(wp, &bw, &bh);
    ok &= make_map_nhwc(&P->cX16, P->X16, B, hp, wp, Cp, bw, bh);
  }
  ok &= make_map_rows(&P->mAO, P->AO, T, Cp, 128);
  ok &= make_map_rows(&P->mH16, P->H16, T, H->HIDp, 128);
  {
    int bw, bh;
    conv_box(wp, &bw, &bh);
    ok &= make_map_nhwc(&P->cAO, P->AO, B, hp, wp, Cp, bw, bh);
    ok &= make_map_nhwc(&P->cHA, P->HA, B, hp, wp, 64, bw, bh);
  }
  for (int i = 0; i < 3; i++)
    for (int r = 0; r < 3; r++) {
      const int f = 1 << r;  // resolution factor 1, 2, 4
      if (f > s && r > 0) continue;
      int bw, bh;
      conv_box(wp * f, &bw, &bh);
      ok &= make_map_nhwc(&P->cHB[i][r], P->HB[i], B, hp * f, wp * f, 64, bw, bh);
    }
  if (!ok) {
    free_plan(*P);
    fail(S2S_ERR_CUDA, "cuTensorMapEncodeTiled failed for an activation operand");
  }
  H->plan = std::move(P);
  return H->plan.get();
}

// ------------------------------------------------------------------ launches
struct Launcher {
  s2s_handle* H;
  cudaStream_t st;
  cudaEvent_t ev() {
    if (!H->ev_pool.empty()) {
      cudaEvent_t e = H->ev_pool.back();
      H->ev_pool.pop_back();
      return e;
    }
    cudaEvent_t e;
    ck(cudaEventCreate(&e), "event");
    return e;
  }
  template <typename F>
  void run(const char* name, F&& f) {
    if (H->stop_after >= 0 && H->fwd_launches >= H->stop_after) return;
    H->fwd_launches++;
    cudaEvent_t a = nullptr, b = nullptr;
    const bool timed = H->profiling && (H->prof_only.empty() ||
                                        strncmp(name, H->prof_only.c_str(), H->prof_only.size()) == 0);
    if (timed) {
      a = ev();
      b = ev();
      ck(cudaEventRecord(a, st), "event");
    }
    ck(f(), name);
    H->launches++;
    if (timed) {
      ck(cudaEventRecord(b, st), "event");
      H->prof_pending.push_back({name, a, b});
    }
  }
};

Epi epi0() {
  Epi e;
  memset(&e, 0, sizeof e);
  e.ln_eps = 1e-5f;
  e.img_range = 1.0f;
  return e;
}

GemmArgs gemm_args(int M, int N, int K, const Epi& e) {
  GemmArgs a;
  memset(&a, 0, sizeof a);
  a.M = M;
  a.N = N;
  a.K = K;
  a.epi = e;
  a.epi.n_valid = e.n_valid ? e.n_valid : N;
  return a;
}

GemmArgs conv_args(int B, int H, int W, int Cip, int N, const Epi& e) {
  GemmArgs a;
  memset(&a, 0, sizeof a);
  a.conv = 1;
  a.B = B;
  a.H = H;
  a.W = W;
  a.N = N;
  a.K = 9 * Cip;
  a.kc = Cip / 64;
  conv_box(W, &a.boxw, &a.boxh);
  a.tiles_x = (W + a.boxw - 1) / a.boxw;
  a.tiles_y = (H + a.boxh - 1) / a.boxh;
  a.epi = e;
  a.epi.n_valid = e.n_valid ? e.n_valid : N;
  return a;
}

// The STORE_ROWS outputs and the post-norm residual of a launch, as TMA maps.
OutMaps out_maps(Plan* P, const GemmArgs& a) {
  OutMaps om;
  memset(&om, 0, sizeof om);
  if (a.epi.store != STORE_ROWS) return om;
  auto mk = [&](CUtensorMap* m, const void* p, int eb, int ld) {
    if (!p) return;
    const std::array<int64_t, 8> key = {(int64_t)(uintptr_t)p, eb, ld, a.conv, a.conv ? a.B : a.M,
                                        a.H, a.W, a.boxw};
    auto it = P->omaps.find(key);
    if (it == P->omaps.end()) {
      CUtensorMap map;
      const bool ok = a.conv ? make_map_out_nhwc(&map, p, eb, a.B, a.H, a.W, ld, a.boxw)
                             : make_map_out_rows(&map, p, eb, (uint64_t)a.M, (uint64_t)ld);
      if (!ok) fail(S2S_ERR_CUDA, "cuTensorMapEncodeTiled failed for an output operand");
      it = P->omaps.emplace(key, map).first;
    }
    *m = it->second;
  };
  mk(&om.o32, a.epi.o32, 4, a.epi.ld32);
  mk(&om.o32b, a.epi.o32b, 4, a.epi.ld32b);
  mk(&om.o16, a.epi.o16, 2, a.epi.ld16);
  if (a.epi.res_post) mk(&om.res, a.epi.res_post, 4, a.epi.ld_res_post);
  return om;
}

void set_final(const s2s_handle* H, Epi& e) {
  e.img_range = H->cfg.img_range;
  e.mean0 = H->cfg.mean[0];
  e.mean1 = H->cfg.mean[1];
  e.mean2 = H->cfg.mean[2];
}

void forward_device(s2s_handle* H, int B, int h, int w, const float* d_in, float* d_out,
                    float* d_aux, cudaStream_t st) {
  const s2s_config& c = H->cfg;
  if (h < c.window || w < c.window)
    fail(S2S_ERR_INVALID, std::to_string(h) + "x" + std::to_string(w) +
                              " is smaller than one window; the reference refuses it "
                              "(src/backend.rs:60-71)");
  if (B < 1) fail(S2S_ERR_INVALID, "batch must be >= 1");
  Plan* P = get_plan(H, B, h, w);
  H->fwd_launches = 0;
  Launcher L{H, st};
  const int C = c.embed, Cp = H->Cp, hp = P->hp, wp = P->wp, s = c.scale, F = H->feat;
  const int M = (int)P->T;
  // 1. pad + conv_first (fp32 body skip F0, fp16 operand F0h).
  L.run("pad_reflect", [&] { return launch_pad_reflect(d_in, P->P, B, 3, h, w, hp, wp, st); });
  L.run("conv_first", [&] {
    return launch_conv3_small(P->P, H->cf_w, H->cf_b, B, hp, wp, C, 0, 0.0f, P->F0, Cp, P->F0h,
                              Cp, st);
  });
  // 2. top patch_embed: 1x1 + LayerNorm -> X (window order, shift 0), S (image order).
  {
    Epi e = epi0();
    e.bias = H->pe.b;
    e.ln_g = H->pe_g;
    e.ln_b = H->pe_b;
    e.ln_n = C;
    e.n_valid = C;
    e.o32 = P->X;
    e.ld32 = Cp;
    e.o16 = P->X16;
    e.ld16 = Cp;
    e.o32b = P->S;
    e.ld32b = Cp;
    GemmArgs a = gemm_args(M, Cp, Cp, e);
    L.run("gemm_patch_embed", [&] { return launch_gemm(P->mF0h, H->pe.map, out_maps(P, a), a, Cp, st); });
  }
  const int nwin = B * (hp / 8) * (wp / 8);
  for (int si = 0; si < c.n_depths; si++) {
    Stage& stg = H->stages[si];
    const int depth = c.depths[si];
    for (int b = 0; b < depth; b++) {
      Block& bl = stg.blocks[b];
      const int sh = (b % 2 == 1) ? c.window / 2 : 0;
      {  // QKV
        Epi e = epi0();
        e.bias = bl.qkv.b;
        e.o16 = P->QKV;
        e.ld16 = H->NQ;
        GemmArgs a = gemm_args(M, H->NQ, Cp, e);
        L.run("gemm_qkv", [&] { return launch_gemm(P->mX16, bl.qkv.map, out_maps(P, a), a, bl.qkv.BN, st); });
      }
      L.run("window_attention", [&] {
        return launch_window_attention(P->QKV, P->AO, bl.cpb, bl.ls, P->rows[sh ? 1 : 0], nwin,
                                       H->heads, H->hd, H->DP, Cp, hp / 8, wp / 8, hp, wp, sh, st);
      });
      {  // proj + norm1 + residual, in place
        Epi e = epi0();
        e.bias = bl.proj.b;
        e.ln_g = bl.n1g;
        e.ln_b = bl.n1b;
        e.ln_n = C;
        e.n_valid = C;
        e.res_post = P->X;
        e.ld_res_post = Cp;
        e.o32 = P->X;
        e.ld32 = Cp;
        e.o16 = P->X16;
        e.ld16 = Cp;
        GemmArgs a = gemm_args(M, Cp, Cp, e);
        L.run("gemm_proj", [&] { return launch_gemm(P->mAO, bl.proj.map, out_maps(P, a), a, Cp, st); });
      }
      if (H->fused_mlp) {  // fc1 + GELU + fc2 + norm2 + residual in one kernel
        MlpArgs m;
        m.M = M;
        m.b1 = bl.fc1.b;
        m.b2 = bl.fc2.b;
        m.g2 = bl.n2g;
        m.beta2 = bl.n2b;
        m.ln_n = C;
        m.ln_eps = 1e-5f;
        m.x = P->X;
        m.x16 = P->X16;
        L.run("mlp_fused", [&] {
          Epi eo = epi0();
          eo.o32 = P->X;
          eo.ld32 = Cp;
          eo.o16 = P->X16;
          eo.ld16 = Cp;
          const OutMaps om = out_maps(P, gemm_args(M, Cp, Cp, eo));
          return launch_mlp(P->mX16, bl.fc1.map, bl.fc2.map, om.o32, om.o16, m, Cp, H->HIDp, st);
        });
      } else {
        {  // fc1 + GELU
          Epi e = epi0();
          e.bias = bl.fc1.b;
          e.act = ACT_GELU;
          e.o16 = P->H16;
          e.ld16 = H->HIDp;
          GemmArgs a = gemm_args(M, H->HIDp, Cp, e);
          L.run("gemm_fc1", [&] { return launch_gemm(P->mX16, bl.fc1.map, out_maps(P, a), a, bl.fc1.BN, st); });
        }
        {  // fc2 + norm2 + residual, in place
          Epi e = epi0();
          e.bias = bl.fc2.b;
          e.ln_g = bl.n2g;
          e.ln_b = bl.n2b;
          e.ln_n = C;
          e.n_valid = C;
          e.res_post = P->X;
          e.ld_res_post = Cp;
          e.o32 = P->X;
          e.ld32 = Cp;
          e.o16 = P->X16;
          e.ld16 = Cp;
          GemmArgs a = gemm_args(M, Cp, H->HIDp, e);
          L.run("gemm_fc2", [&] { return launch_gemm(P->mH16, bl.fc2.map, out_maps(P, a), a, Cp, st); });
        }
      }
    }
    // RSTB tail: conv3x3 -> 1x1 patch_embed + stage residual.
    {
      Epi e = epi0();
      e.bias = stg.conv.b;
      e.n_valid = C;
      e.o16 = P->AO;
      e.ld16 = Cp;
      GemmArgs a = conv_args(B, hp, wp, Cp, Cp, e);
      L.run("conv_stage", [&] { return launch_gemm(P->cX16, stg.conv.map, out_maps(P, a), a, Cp, st); });
    }
    {
      const bool last = si + 1 == c.n_depths;
      Epi e = epi0();
      e.bias = stg.pe.b;
      e.n_valid = C;
      // the stage residual: without a norm it is added after the bias (TMA path); the
      // last stage's final LayerNorm normalises the sum, so there it comes first
      if (last) {
        e.res_pre = P->S;
        e.ld_res_pre = Cp;
      } else {
        e.res_post = P->S;
        e.ld_res_post = Cp;
      }
      if (!last) {
        e.o32 = P->X;
        e.ld32 = Cp;
        e.o16 = P->X16;
        e.ld16 = Cp;
        e.o32b = P->S;
        e.ld32b = Cp;
      } else {  // + final norm, image order, fp16 operand of conv_after_body
        e.ln_g = H->nrm_g;
        e.ln_b = H->nrm_b;
        e.ln_n = C;
        e.o16 = P->X16;
        e.ld16 = Cp;
      }
      GemmArgs a = gemm_args(M, Cp, Cp, e);
      L.run(last ? "gemm_stage_pe_norm" : "gemm_stage_pe",
            [&] { return launch_gemm(P->mAO, stg.pe.map, out_maps(P, a), a, Cp, st); });
    }
  }
  // 3. conv_after_body + body skip (conv_first output) -> Y16 (in AO).
  {
    Epi e = epi0();
    e.bias = H->cab.b;
    e.n_valid = C;
    e.res_post = P->F0;
    e.ld_res_post = Cp;
    e.o16 = P->AO;
    e.ld16 = Cp;
    GemmArgs a = conv_args(B, hp, wp, Cp, Cp, e);
    L.run("conv_after_body", [&] { return launch_gemm(P->cX16, H->cab.map, out_maps(P, a), a, Cp, st); });
  }
  // 4. head.
  auto conv_to = [&](const char* name, const CUtensorMap& mapA, const TcWeight& tw, int Hh, int Ww,
                     int Cip, Epi e) {
    GemmArgs a = conv_args(B, Hh, Ww, Cip, tw.N, e);
    L.run(name, [&] { return launch_gemm(mapA, tw.map, out_maps(P, a), a, tw.BN, st); });
  };
  auto cbu = [&]() {
    Epi e = epi0();
    e.bias = H->cbu.b;
    e.act = ACT_LRELU;
    e.slope = 0.01f;
    e.o16 = P->HA;
    e.ld16 = F;
    conv_to("conv_before_upsample", P->cAO, H->cbu, hp, wp, Cp, e);
  };
  auto final_planes = [&](const CUtensorMap& mapA, int Hh, int Ww) {
    Epi e = epi0();
    e.bias = H->last.b;
    e.store = STORE_PLANES;
    e.planes = d_out;
    e.crop_h = h * s;
    e.crop_w = w * s;
    set_final(H, e);
    conv_to("conv_last", mapA, H->last, Hh, Ww, F, e);
  };
  switch (c.upsampler) {
    case S2S_PIXELSHUFFLE:
    case S2S_PIXELSHUFFLE_AUX: {
      cbu();
      const CUtensorMap* src = &P->cHA;
      int hh = hp, ww = wp;
      const int octs = (int)std::lround(std::log2((double)s));
      if (c.upsampler == S2S_PIXELSHUFFLE_AUX) {
        // bicubic branch of the padded, mean-adjusted input, on the padded output grid
        L.run("bicubic", [&] {
          return launch_bicubic(P->P, P->BIC, B * 3, hp, wp, hp * s, wp * s, st);
        });
        L.run("conv_bicubic", [&] {
          return launch_conv3_small(P->BIC, H->cbic_w, H->cbic_b, B, hp * s, wp * s, F, 0, 0.0f,
                                    P->BICF, F, nullptr, 0, st);
        });
        Epi e = epi0();
        e.bias = H->aux.b;
        e.store = STORE_PLANES;
        e.planes = d_aux;
        e.planes_raw = P->AUXRAW;
        e.crop_h = hp;
        e.crop_w = wp;
        set_final(H, e);
        conv_to("conv_aux", P->cHA, H->aux, hp, wp, F, e);
        L.run("conv_after_aux", [&] {
          return launch_conv3_small(P->AUXRAW, H->caa_w, H->caa_b, B, hp, wp, F, 2, 0.01f,
                                    nullptr, 0, P->HB[2], F, st);
        });
        src = &P->cHB[2][0];
      }
      for (int o = 0; o < octs; o++) {
        __half* dst = P->HB[o % 2];
        Epi e = epi0();
        e.bias = H->oct[o].b;
        e.store = STORE_SHUFFLE2;
        e.o16 = dst;
        if (o + 1 == octs && c.upsampler == S2S_PIXELSHUFFLE_AUX) e.res_post = P->BICF;
        conv_to(o == 0 ? "conv_upsample0" : "conv_upsample1", *src, H->oct[o], hh, ww, F, e);
        hh *= 2;
        ww *= 2;
        src = &P->cHB[o % 2][o + 1];
      }
      final_planes(*src, hh, ww);
      break;
    }
    case S2S_PIXELSHUFFLEDIRECT: {
      Epi e = epi0();
      e.bias = H->direct.b;
      e.store = STORE_DIRECT;
      e.planes = d_out;
      e.scale = s;
      e.crop_h = h * s;
      e.crop_w = w * s;
      set_final(H, e);
      conv_to("conv_upsample_direct", P->cAO, H->direct, hp, wp, Cp, e);
      break;
    }
    case S2S_NEARESTCONV: {
      cbu();
      L.run("upsample_nearest", [&] { return launch_up2_nhwc(P->HA, P->HB[0], B, hp, wp, F, st); });
      {
        Epi e = epi0();
        e.bias = H->up1.b;
        e.act = ACT_LRELU;
        e.slope = 0.2f;
        e.o16 = P->HB[1];
        e.ld16 = F;
        conv_to("conv_up1", P->cHB[0][1], H->up1, 2 * hp, 2 * wp, F, e);
      }
      L.run("upsample_nearest",
            [&] { return launch_up2_nhwc(P->HB[1], P->HB[0], B, 2 * hp, 2 * wp, F, st); });
      {
        Epi e = epi0();
        e.bias = H->up2.b;
        e.act = ACT_LRELU;
        e.slope = 0.2f;
        e.o16 = P->HB[2];
        e.ld16 = F;
        conv_to("conv_up2", P->cHB[0][2], H->up2, 4 * hp, 4 * wp, F, e);
      }
      {
        Epi e = epi0();
        e.bias = H->hr.b;
        e.act = ACT_LRELU;
        e.slope = 0.2f;
        e.o16 = P->HB[0];
        e.ld16 = F;
        conv_to("conv_hr", P->cHB[2][2], H->hr, 4 * hp, 4 * wp, F, e);
      }
      final_planes(P->cHB[0][2], 4 * hp, 4 * wp);
      break;
    }
    default:
      fail(S2S_ERR_UNSUPPORTED, "unknown upsampler");
  }
}

void check_device_error(s2s_handle* H) {
  unsigned int e = 0;
  ck(cudaMemcpyFromSymbol(&e, g_s2s_err, sizeof e), "error word");
  if (e != 0) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_s2s_err, &z, sizeof z);
    fail(S2S_ERR_TIMEOUT, "a device-side wait gave up (code " + std::to_string(e) +
                              "); the kernel unwound without completing its tile");
  }
}

void drain_profile(s2s_handle* H) {
  for (auto& p : H->prof_pending) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
      auto& slot = H->prof[p.name];
      slot.first += 1;
      slot.second += ms;
    }
    H->ev_pool.push_back(p.a);
    H->ev_pool.push_back(p.b);
  }
  H->prof_pending.clear();
}

template <typename F>
int guarded(s2s_handle* H, F&& f) {
  try {
    ck(cudaSetDevice(H->device), "cudaSetDevice");
    f();
    return S2S_OK;
  } catch (const S2SError& e) {
    H->err = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    H->err = "host allocation failed";
    return S2S_ERR_OOM;
  }
}

void ensure_staging(s2s_handle* H, float** p, size_t* have, size_t n) {
  if (*have >= n) return;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  ck(cudaMalloc((void**)p, n * 4), "staging");
  *have = n;
}

}  // namespace

extern "C" {

int s2s_create(const s2s_config* cfg, const s2s_tensor* tensors, int n_tensors, int device,
               s2s_handle** out) {
  if (out) *out = nullptr;
  if (!cfg || !out || (!tensors && n_tensors > 0)) {
    g_create_error = "s2s_create: null argument";
    return S2S_ERR_INVALID;
  }
  std::unique_ptr<s2s_handle> H(new s2s_handle());
  H->device = device;
  H->cfg = *cfg;
  const s2s_config& c = *cfg;
  if (c.window != 8 || c.embed <= 0 || c.heads <= 0 || c.embed % c.heads != 0 ||
      c.n_depths < 1 || c.n_depths > 16 || c.mlp_ratio < 1 || (c.scale != 2 && c.scale != 4) ||
      c.upsampler < 0 || c.upsampler > 3 || (c.upsampler == S2S_NEARESTCONV && c.scale != 4)) {
    g_create_error = "s2s_create: unsupported architecture (window 8, scale 2/4, embed divisible "
                     "by heads, nearest+conv only at x4)";
    return S2S_ERR_UNSUPPORTED;
  }
  H->C = c.embed;
  H->Cp = pad_to(c.embed, 64);
  H->heads = c.heads;
  H->hd = c.embed / c.heads;
  H->DP = pad_to(H->hd, 16);
  if (H->DP > 32 || H->Cp > 256) {
    g_create_error = "s2s_create: head_dim > 32 or embed > 256 is not supported by this build";
    return S2S_ERR_UNSUPPORTED;
  }
  H->NQ = 3 * c.heads * H->DP;
  H->HIDp = pad_to(c.mlp_ratio * c.embed, 64);
  if (H->NQ % 32 != 0 || H->HIDp % 32 != 0) {
    g_create_error = "s2s_create: unsupported padded widths";
    return S2S_ERR_UNSUPPORTED;
  }
  H->fused_mlp = (H->Cp == 192 && H->HIDp == 384) || (H->Cp == 64 && H->HIDp == 128);
  {
    const char* f = getenv("S2S_UNFUSED_MLP");  // validation switch: the two-GEMM MLP path
    if (f && *f && strcmp(f, "0") != 0) H->fused_mlp = false;
  }
  TensorTable T;
  for (int i = 0; i < n_tensors; i++) T.t[tensors[i].name] = &tensors[i];
  int rc = guarded(H.get(), [&] {
    ck(cudaStreamCreateWithFlags(&H->stream, cudaStreamNonBlocking), "stream");
    build_weights(H.get(), T);
    ck(cudaDeviceSynchronize(), "weight upload");
  });
  if (rc != S2S_OK) {
    g_create_error = H->err;
    for (void* p : H->wallocs) cudaFree(p);
    if (H->stream) cudaStreamDestroy(H->stream);
    return rc;
  }
  const char* prof = getenv("SWIN2SR_PROFILE_GPU");
  H->profiling = prof && *prof && strcmp(prof, "0") != 0;
  *out = H.release();
  return S2S_OK;
}

int s2s_forward_device(s2s_handle* H, int batch, int height, int width, const float* d_in,
                       float* d_out, float* d_aux, void* stream) {
  if (!H) return S2S_ERR_INVALID;
  cudaStream_t st = stream ? (cudaStream_t)stream : H->stream;
  return guarded(H, [&] {
    if (H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX && !d_aux)
      fail(S2S_ERR_INVALID, "the pixelshuffle_aux head needs an aux buffer on the device path");
    forward_device(H, batch, height, width, d_in, d_out, d_aux, st);
  });
}

int s2s_forward_batch(s2s_handle* H, int batch, int height, int width, const float* in, float* out,
                      float* aux) {
  if (!H || !in || !out) return S2S_ERR_INVALID;
  return guarded(H, [&] {
    const int win = H->cfg.window, s = H->cfg.scale;
    const size_t nin = (size_t)batch * 3 * height * width;
    const size_t nout = (size_t)batch * 3 * height * s * width * s;
    const size_t naux = (size_t)batch * 3 * (height / win + 1) * win * (width / win + 1) * win;
    const bool has_aux = H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX;
    ensure_staging(H, &H->h_in, &H->h_in_n, nin);
    ensure_staging(H, &H->h_out, &H->h_out_n, nout);
    if (has_aux) ensure_staging(H, &H->h_aux, &H->h_aux_n, naux);
    ck(cudaMemcpyAsync(H->h_in, in, nin * 4, cudaMemcpyHostToDevice, H->stream), "upload");
    forward_device(H, batch, height, width, H->h_in, H->h_out, has_aux ? H->h_aux : nullptr,
                   H->stream);
    ck(cudaMemcpyAsync(out, H->h_out, nout * 4, cudaMemcpyDeviceToHost, H->stream), "download");
    if (has_aux && aux)
      ck(cudaMemcpyAsync(aux, H->h_aux, naux * 4, cudaMemcpyDeviceToHost, H->stream), "download");
    ck(cudaStreamSynchronize(H->stream), "forward");
    check_device_error(H);
    if (H->profiling) drain_profile(H);
  });
}

int s2s_forward(s2s_handle* H, int height, int width, const float* in_chw, float* out_chw,
                float* aux_chw) {
  return s2s_forward_batch(H, 1, height, width, in_chw, out_chw, aux_chw);
}

int s2s_aux_dims(const s2s_handle* H, int height, int width, int* aux_h, int* aux_w) {
  if (!H || H->cfg.upsampler != S2S_PIXELSHUFFLE_AUX) return S2S_ERR_INVALID;
  const int win = H->cfg.window;
  if (aux_h) *aux_h = (height / win + 1) * win;
  if (aux_w) *aux_w = (width / win + 1) * win;
  return S2S_OK;
}

int64_t s2s_uploaded_bytes(const s2s_handle* H) { return H ? (int64_t)H->uploaded : 0; }

int64_t s2s_workspace_bytes(const s2s_handle* H, int batch, int height, int width) {
  if (!H || batch < 1 || height < 1 || width < 1) return -1;
  return plan_bytes(H, batch, height, width);
}

const char* s2s_last_error(const s2s_handle* H) {
  return H ? H->err.c_str() : g_create_error.c_str();
}

int s2s_profile_enable(s2s_handle* H, int on, const char* only) {
  if (!H) return S2S_ERR_INVALID;
  H->profiling = on != 0;
  H->prof_only = only ? only : "";
  return S2S_OK;
}

int s2s_profile_report(s2s_handle* H, char* buf, int cap, int reset) {
  if (!H) return -1;
  cudaSetDevice(H->device);
  cudaDeviceSynchronize();
  drain_profile(H);
  std::string s;
  for (auto& kv : H->prof) {
    char line[160];
    snprintf(line, sizeof line, "%s %ld %.6f\n", kv.first.c_str(), kv.second.first,
             kv.second.second);
    s += line;
  }
  if (buf && cap > 0) {
    const size_t n = std::min((size_t)cap - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  if (reset) H->prof.clear();
  return (int)s.size() + 1;
}

int64_t s2s_launch_count(const s2s_handle* H) { return H ? H->launches : 0; }

int s2s_debug_stop_after(s2s_handle* H, int64_t launches) {
  if (!H) return S2S_ERR_INVALID;
  H->stop_after = launches;
  return S2S_OK;
}

int64_t s2s_debug_read(s2s_handle* H, const char* name, float* host, int64_t capacity) {
  if (!H || !name || !H->plan) return -1;
  Plan& P = *H->plan;
  const size_t T = P.T, Cp = H->Cp, s = H->cfg.scale;
  const void* p = nullptr;
  size_t n = 0;
  bool half = false;
  const std::string k(name);
  if (k == "P") { p = P.P; n = (size_t)P.B * 3 * P.hp * P.wp; }
  else if (k == "F0") { p = P.F0; n = T * Cp; }
  else if (k == "X") { p = P.X; n = T * Cp; }
  else if (k == "S") { p = P.S; n = T * Cp; }
  else if (k == "F0h") { p = P.F0h; n = T * Cp; half = true; }
  else if (k == "X16") { p = P.X16; n = T * Cp; half = true; }
  else if (k == "QKV") { p = P.QKV; n = T * H->NQ; half = true; }
  else if (k == "AO") { p = P.AO; n = T * Cp; half = true; }
  else if (k == "H16") { p = P.H16; n = T * H->HIDp; half = true; }
  else if (k == "HA") { p = P.HA; n = T * 64; half = true; }
  else if (k == "HB0") { p = P.HB[0]; n = T * s * s * 64; half = true; }
  else if (k == "HB1") { p = P.HB[1]; n = T * s * s * 64; half = true; }
  else if (k == "HB2") { p = P.HB[2]; n = T * s * s * 64; half = true; }
  else if (k == "BIC" && P.BIC) { p = P.BIC; n = (size_t)P.B * 3 * P.hp * s * P.wp * s; }
  else if (k == "BICF" && P.BICF) { p = P.BICF; n = T * s * s * 64; }
  else if (k == "AUXRAW" && P.AUXRAW) { p = P.AUXRAW; n = (size_t)P.B * 3 * P.hp * P.wp; }
  if (!p) return -1;
  if (!host || capacity < (int64_t)n) return (int64_t)n;
  cudaSetDevice(H->device);
  cudaDeviceSynchronize();
  if (!half) {
    if (cudaMemcpy(host, p, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  } else {
    std::vector<__half> tmp(n);
    if (cudaMemcpy(tmp.data(), p, n * 2, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    for (size_t i = 0; i < n; i++) host[i] = __half2float(tmp[i]);
  }
  return (int64_t)n;
}

void s2s_destroy(s2s_handle* H) {
  if (!H) return;
  cudaSetDevice(H->device);
  cudaDeviceSynchronize();
  drain_profile(H);
  for (cudaEvent_t e : H->ev_pool) cudaEventDestroy(e);
  if (H->plan) free_plan(*H->plan);
  for (void* p : H->wallocs) cudaFree(p);
  if (H->h_in) cudaFree(H->h_in);
  if (H->h_out) cudaFree(H->h_out);
  if (H->h_aux) cudaFree(H->h_aux);
  if (H->stream) cudaStreamDestroy(H->stream);
  delete H;
}

const char* s2s_version(void) { return "swin2sr-b200 0.1 (sm_100a)"; }

}  // extern "C"
