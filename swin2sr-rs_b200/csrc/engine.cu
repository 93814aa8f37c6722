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
// Per block (src/cpu.rs:1516-1575): QKV GEMM (+ q/k normalisation) -> window
// attention -> proj GEMM with norm1 + residual -> fused MLP (fc1 + GELU + fc2 + norm2
// + residual; S2S_UNFUSED_MLP=1 runs it as two GEMMs for validation). Repeated
// forwards replay a CUDA graph; a sharded forward runs the same code on a row band.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
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
#include "halo.cuh"
#include "s2s.h"

namespace s2s {
cudaError_t launch_window_attention(const __half* qkv, __half* out, const float* cpb,
                                    const int* rows, int nwin_total, int heads, int hd, int dp,
                                    int ld_out, int row_h, int split, int lo_q, int lo_out,
                                    int nwh, int nww, int hp, int wp, int shift, int wh_off,
                                    cudaStream_t st);
cudaError_t launch_pad_reflect(const float* x, float* y, int B, int c, int h, int w, int hp,
                               int wp, cudaStream_t st);
cudaError_t launch_pad_band(const float* x, float* y, int c, int h, int w, int hp, int wp, int rows,
                            int y0, cudaStream_t st);
cudaError_t launch_conv3_small(const float* in, const float* wgt, const float* bias, int B, int H,
                               int W, int co_n, int act, float slope, float* o32, int ld32,
                               __half* o16, int ld16, int lo16, cudaStream_t st);
cudaError_t launch_zero_cols_f16(__half* x, size_t rows, int c0, int ld, cudaStream_t st);
cudaError_t launch_bicubic(const float* in, float* out, int BC, int h, int w, int oh, int ow,
                           cudaStream_t st);
cudaError_t launch_up2_nhwc(const __half* in, __half* out, int B, int H, int W, int C,
                            cudaStream_t st);
cudaError_t launch_cpb_table(const float* table, const float* w0, const float* b0, const float* w2,
                             int heads, int win, int hidden, float* out, cudaStream_t st);
}  // namespace s2s

using namespace s2s;

namespace {

thread_local std::string g_create_error;

// s2s_selftest creates its comparison handles with these settings of the validation
// switches (-1: as the environment says).
struct CreateFlags {
  int unfused_mlp = -1, no_patch = -1, split = -1, mma_attn = -1, unfused_proj = -1;
};
thread_local CreateFlags g_create_flags;

// Whether 180-wide handles run QKV + attention as the one fused kernel by default. Not
// today: on classical-x4 (B200) the fused kernel takes 111 us per block against 87 us
// for the QKV GEMM + mma.sync attention pair (its per-head epilogue stages are
// latency-bound with one CTA per SM); S2S_ATTN=fused selects it.
constexpr bool kFusedAttnDefault = false;

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
  CUtensorMap mlp_map;  // fc1 only: 64-row boxes, the fused MLP's hidden part
};

struct Block {
  TcWeight qkv, proj, fc1, fc2;
  float *n1g, *n1b, *n2g, *n2b;
  float *cpb, *ls;  // bias table and q scale, both times log2 e (attention softmax is exp2)
  // the fused QKV + attention kernel's operands: Wqkv [6 x 96][Cp] (per head q, k, v
  // rows of 32), q and v biases [6][32], and the compact [6][576] position-bias table
  // (times log2 e)
  TcWeight wqkv;
  float *qb = nullptr, *vb = nullptr, *cpbc = nullptr;
};

struct Stage {
  std::vector<Block> blocks;
  TcWeight conv, pe;
};

// Activation workspace for one (B, h, w), over a local plane of hp x wp tokens per image.
//
// Whole-image plans: the local plane is the padded plane and every row is owned.
// Band plans (one rank of a sharded forward, B = 1): the local plane holds global
// padded rows [R0 - 8, R1 + 8); rows [8, 8 + R1 - R0) are owned, the 8 rows on
// either side receive neighbours' rows before the steps that read them.
struct Plan {
  int B = 0, h = 0, w = 0, hp = 0, wp = 0;
  size_t T = 0;
  int band = 0, rank = 0, world = 1, R0 = 0, R1 = 0, ghp = 0;
  int halo = 0;         // local rows above the owned rows
  int own_rows = 0;     // owned plane rows
  size_t own_off = 0;   // tokens before the first owned row
  int M_own = 0;        // owned tokens (the per-token GEMMs' M)
  size_t sh_off = 0;    // tokens before the first row the shifted windows cover
  int M_sh = 0;         // tokens the shifted blocks' QKV covers
  int nwin[2] = {0, 0}, nwh_l[2] = {0, 0}, wh_off[2] = {0, 0};  // attention, shift 0 / win/2
  int conv_row0 = 0, conv_H = 0, conv_y0 = 0, conv_y1 = 0;  // 3x3 conv: map rows, output rows
  int head_row0 = 0, head_rows = 0;  // the plane the upsampling head runs on
  int crop_y0 = 0, crop_rows = 0;    // output LR rows: head plane rows [crop_y0, +crop_rows)
  CUtensorMap mX16s;                 // QKV operand of the shifted blocks
  CUtensorMap mX16t, mX16b;          // band: the 4 halo rows above / below the owned rows
  // The forward captured as a CUDA graph for one set of I/O pointers: made on the
  // second forward with the same pointers, replayed from the third on.
  cudaGraphExec_t gexec = nullptr;
  const void *g_in = nullptr, *g_out = nullptr, *g_aux = nullptr;
  int g_seen = 0;
  long long g_launches = 0;
  std::vector<void*> allocs;
  size_t bytes = 0;
  float *P = nullptr, *F0 = nullptr, *X = nullptr, *S = nullptr;
  __half *F0h = nullptr, *X16 = nullptr, *QKV = nullptr, *AO = nullptr, *H16 = nullptr;
  __half *HA = nullptr, *HB[3] = {nullptr, nullptr, nullptr};
  float *BIC = nullptr, *BICF = nullptr, *AUXRAW = nullptr;
  int* rows[2] = {nullptr, nullptr};  // window-major token -> image row, shift 0 / win/2
  CUtensorMap mF0h, mX16, mAO, mH16, cX16, cAO, cHA;
  CUtensorMap mXw;  // X16 plane in 4 x 4-pixel boxes (the fused attention's windows)
  CUtensorMap cHB[3][3];  // head planes at 1x, 2x, 4x resolution
  CUtensorMap cHBp[3][3];                 // the same planes in (boxh + 2)-row patches
  bool hbp[3][3] = {{false}};             // ... when the plane's conv box allows them
  // Output / residual TMA maps, built on first use for each (buffer, geometry).
  std::map<std::array<int64_t, 8>, CUtensorMap> omaps;
  // Peer-store halo transport (band plans over NCCL unless S2S_HALO=nccl): this
  // rank's mailbox and its neighbours' planes and mailboxes, mapped through CUDA IPC.
  HaloMailbox* mb = nullptr;
  HaloPeer prevp, nextp;
  std::vector<void*> ipc_maps;
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
  // Two-term operands (split): every fp16 tensor-core operand of the body carries
  // hi = fp16(x) and lo = fp16(x - hi) side by side in its row ([hi | lo]), and the
  // weights [W_hi | W_hi | W_lo] along K, so one tcgen05 accumulation over three K
  // blocks is hi*W_hi + lo*W_hi + hi*W_lo: about 21 bits of each operand instead of
  // 11. The 60-wide network needs it for the 2e-3 parity bound (with single fp16
  // operands its output moves by up to 5e-3); the 180-wide ones do not (<= 7e-4).
  // Cs, NQs, HIDs: row strides (halves) of the X16/AO/F0h, QKV and H16 buffers.
  bool split = false;
  int Cs = 0, NQs = 0, HIDs = 0;
  // QKV projection and window attention in one tcgen05 kernel (k_qkv_attention) for
  // 6 heads of 32 (padded) over Cp = 192; AO rows are then [head][32] and the proj
  // weights' K follows that order. S2S_ATTN=mma / fused (validation switch): the QKV
  // GEMM + mma.sync attention kernel pair, or the fused kernel.
  bool fused_attn = false;
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
  uint8_t *b_in = nullptr, *b_out = nullptr;  // device staging of the image calls (bytes)
  size_t b_in_n = 0, b_out_n = 0;
  bool profiling = false;
  std::string prof_only;  // profile only kernel classes with this prefix
  std::vector<ProfEntry> prof_pending;
  std::vector<cudaEvent_t> ev_pool;
  std::map<std::string, std::pair<long, double>> prof;
  std::atomic<long long> launches{0};  // kernels launched (all calls on the handle)
  bool fused_mlp = false;      // (Cp, HIDp) has a fused MLP kernel
  // proj + norm1 + residual run inside the fused MLP kernel (Cp = 192);
  // S2S_UNFUSED_PROJ=1 (validation switch): the proj GEMM runs on its own
  bool fused_proj = false;
  bool graphs = true;          // replay repeated forwards as CUDA graphs (S2S_GRAPHS=0: off)
  bool no_patch = false;       // conv_last from nine tap boxes (S2S_NO_PATCH=1: validation)
  long long stop_after = -1;   // diagnostics: launches per forward before stopping
  long long fwd_launches = 0;  // launches enqueued by the forward in flight
  // Row-band sharding (s2s_band_init / s2s_band_init_local): this handle's rank.
  int band_rank = 0, band_world = 1;
  void* nccl_comm = nullptr;                  // ncclComm_t
  bool halo_ipc = true;                       // peer stores (S2S_HALO=nccl: NCCL send/recv)
  cudaStream_t side = nullptr;                // halo transfers overlapping the QKV GEMM
  cudaEvent_t fork = nullptr, join = nullptr;
  std::shared_ptr<s2s::LocalGroup> group;     // in-process group instead of NCCL
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

// Store weight value v at K block position k of a row of `kb` values: one fp16 term,
// or, two-term, [hi | hi | lo] over three K blocks (the A operand's [hi | lo] row is
// read as hi, lo, hi against them).
inline void put_w(__half* row, int k, int kb, float v, bool split) {
  const __half hi = __float2half_rn(v);
  row[k] = hi;
  if (split) {
    row[kb + k] = hi;
    row[2 * kb + k] = __float2half_rn(v - __half2float(hi));
  }
}

// Linear [n_out][n_in] -> fp16 [N][K] with row remap (dst row -> src row or -1);
// two-term: [N][3K].
void pack_linear(s2s_handle* H, TcWeight& tw, const float* W, const float* bias, int n_in, int N,
                 int K, int BN, const std::vector<int>& rowmap, bool split = false) {
  const int KK = split ? 3 * K : K;
  std::vector<__half> w((size_t)N * KK, __float2half(0.0f));
  std::vector<float> b(N, 0.0f);
  for (int r = 0; r < N; r++) {
    const int s = rowmap[r];
    if (s < 0) continue;
    for (int k = 0; k < n_in; k++) put_w(&w[(size_t)r * KK], k, K, W[(size_t)s * n_in + k], split);
    if (bias) b[r] = bias[s];
  }
  finish_tc(H, tw, w, b, N, KK, BN);
}

// Conv3x3 [co][ci][3][3] -> fp16 [N][9*Cip], K index = (ky*3+kx)*Cip + c; two-term:
// [N][9*3*Cip], each tap's block [hi | hi | lo].
void pack_conv(s2s_handle* H, TcWeight& tw, const float* W, const float* bias, int ci, int Cip,
               int N, int BN, const std::vector<int>& rowmap, bool split = false) {
  const int TB = split ? 3 * Cip : Cip;  // K per tap
  const int K = 9 * TB;
  std::vector<__half> w((size_t)N * K, __float2half(0.0f));
  std::vector<float> b(N, 0.0f);
  for (int r = 0; r < N; r++) {
    const int s = rowmap[r];
    if (s < 0) continue;
    for (int c = 0; c < ci; c++)
      for (int t = 0; t < 9; t++)
        put_w(&w[(size_t)r * K + t * TB], c, Cip, W[((size_t)s * ci + c) * 9 + t], split);
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

// The log-spaced relative coordinate table of a win x win window, [(2w-1)^2][2]
// (network_swin2sr.py:108-120, pretrained window size 0).
std::vector<float> relative_coords_table(int win) {
  const int m = 2 * win - 1;
  std::vector<float> t((size_t)m * m * 2);
  auto f = [&](int r) {
    float x = (float)r / (float)(win - 1);
    x *= 8.0f;
    const float sgn = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    return sgn * std::log2(std::fabs(x) + 1.0f) / std::log2(8.0f);
  };
  for (int a = 0; a < m; a++)
    for (int b = 0; b < m; b++) {
      t[((size_t)a * m + b) * 2] = f(a - (win - 1));
      t[((size_t)a * m + b) * 2 + 1] = f(b - (win - 1));
    }
  return t;
}

// One block's bias table from its CPB MLP (cpb_mlp.0: Linear(2, hidden) + ReLU,
// cpb_mlp.2: Linear(hidden, heads) without bias), computed by k_cpb_table into a
// device buffer the handle owns. The operands go to `tmp` (freed after the upload sync).
float* cpb_from_mlp(s2s_handle* H, const TensorTable& T, const std::string& p, int heads,
                    std::vector<void*>& tmp) {
  const int win = H->cfg.window, n = win * win;
  const auto it = T.t.find(p + "attn.cpb_mlp.0.weight");
  const int hidden = (int)it->second->shape[0];
  if (it->second->ndim != 2 || it->second->shape[1] != 2 || hidden < 1)
    fail(S2S_ERR_INVALID, "tensor `" + p + "attn.cpb_mlp.0.weight` must be [hidden][2]");
  const float* w0 = T.get(p + "attn.cpb_mlp.0.weight", (int64_t)hidden * 2);
  const float* b0 = T.get(p + "attn.cpb_mlp.0.bias", hidden);
  const float* w2 = T.get(p + "attn.cpb_mlp.2.weight", (int64_t)heads * hidden);
  auto dev = [&](const float* src, size_t cnt) {
    void* d = nullptr;
    ck(cudaMalloc(&d, cnt * 4), "cpb operands");
    tmp.push_back(d);
    ck(cudaMemcpy(d, src, cnt * 4, cudaMemcpyHostToDevice), "cpb operands");
    return static_cast<const float*>(d);
  };
  const std::vector<float> table = relative_coords_table(win);
  const float* dt = dev(table.data(), table.size());
  const float* dw0 = dev(w0, (size_t)hidden * 2);
  const float* db0 = dev(b0, hidden);
  const float* dw2 = dev(w2, (size_t)heads * hidden);
  float* out = upload(H, std::vector<float>((size_t)heads * n * n, 0.0f));
  ck(launch_cpb_table(dt, dw0, db0, dw2, heads, win, hidden, out, 0), "cpb table");
  return out;
}

void build_weights(s2s_handle* H, const TensorTable& T, std::vector<void*>& tmp) {
  const s2s_config& c = H->cfg;
  const int C = c.embed, Cp = H->Cp, hd = H->hd, DP = H->DP, heads = H->heads;
  const int HID = c.mlp_ratio * C, HIDp = H->HIDp;
  const int n = c.window * c.window;
  const bool sp = H->split;
  // top
  H->cf_w = upload(H, std::vector<float>(T.get("conv_first.weight", (int64_t)C * 27),
                                         T.get("conv_first.weight") + (size_t)C * 27));
  H->cf_b = upload(H, std::vector<float>(T.get("conv_first.bias", C), T.get("conv_first.bias") + C));
  pack_linear(H, H->pe, T.get("patch_embed.proj.weight", (int64_t)C * C),
              T.get("patch_embed.proj.bias", C), C, Cp, Cp, Cp, identity_rows(Cp, C), sp);
  H->pe_g = upload(H, padded(T.get("patch_embed.norm.weight", C), C, Cp));
  H->pe_b = upload(H, padded(T.get("patch_embed.norm.bias", C), C, Cp));
  H->nrm_g = upload(H, padded(T.get("norm.weight", C), C, Cp));
  H->nrm_b = upload(H, padded(T.get("norm.bias", C), C, Cp));
  pack_conv(H, H->cab, T.get("conv_after_body.weight", (int64_t)C * C * 9),
            T.get("conv_after_body.bias", C), C, Cp, Cp, Cp, identity_rows(Cp, C), sp);
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
      if (!H->fused_attn) {
        std::vector<int> qmap(H->NQ, -1);
        for (int part = 0; part < 3; part++)
          for (int h = 0; h < heads; h++)
            for (int d = 0; d < hd; d++) qmap[(h * 3 + part) * DP + d] = part * C + h * hd + d;
        pack_linear(H, bl.qkv, W3.data(), b3.data(), C, H->NQ, Cp, n_tile_for(H->NQ), qmap, sp);
        pack_linear(H, bl.proj, T.get(p + "attn.proj.weight", (int64_t)C * C),
                    T.get(p + "attn.proj.bias", C), C, Cp, Cp, Cp, identity_rows(Cp, C), sp);
      } else {
        // fused kernel: head h's q, k, v rows at h * 96, + 32, + 64 (head_dim padded to 32)
        std::vector<int> mqkv(heads * 96, -1);
        std::vector<float> qbp(heads * 32, 0.0f), vbp(heads * 32, 0.0f);
        for (int h = 0; h < heads; h++)
          for (int d = 0; d < hd; d++) {
            mqkv[h * 96 + d] = h * hd + d;
            mqkv[h * 96 + 32 + d] = C + h * hd + d;
            mqkv[h * 96 + 64 + d] = 2 * C + h * hd + d;
            qbp[h * 32 + d] = qb[h * hd + d];
            vbp[h * 32 + d] = vb[h * hd + d];
          }
        pack_linear(H, bl.wqkv, W3.data(), nullptr, C, heads * 96, Cp, 192, mqkv);
        bl.qb = upload(H, qbp);
        bl.vb = upload(H, vbp);
        // proj reads AO as [head][32]: K index h * 32 + d <- input channel h * hd + d
        const float* pw = T.get(p + "attn.proj.weight", (int64_t)C * C);
        std::vector<float> pwr((size_t)C * Cp, 0.0f);
        for (int o = 0; o < C; o++)
          for (int h = 0; h < heads; h++)
            for (int d = 0; d < hd; d++)
              pwr[(size_t)o * Cp + h * 32 + d] = pw[(size_t)o * C + h * hd + d];
        pack_linear(H, bl.proj, pwr.data(), T.get(p + "attn.proj.bias", C), Cp, Cp, Cp, Cp,
                    identity_rows(Cp, C));
      }
      pack_linear(H, bl.fc1, T.get(p + "mlp.fc1.weight", (int64_t)HID * C),
                  T.get(p + "mlp.fc1.bias", HID), C, HIDp, Cp, n_tile_for(HIDp),
                  identity_rows(HIDp, HID), sp);
      if (H->fused_mlp &&
          !make_map_rows(&bl.fc1.mlp_map, bl.fc1.w, (uint64_t)HIDp, (uint64_t)Cp, 64))
        fail(S2S_ERR_CUDA, "cuTensorMapEncodeTiled failed for a weight operand");
      pack_linear(H, bl.fc2, T.get(p + "mlp.fc2.weight", (int64_t)C * HID),
                  T.get(p + "mlp.fc2.bias", C), HID, Cp, HIDp, Cp, identity_rows(Cp, C), sp);
      bl.n1g = upload(H, padded(T.get(p + "norm1.weight", C), C, Cp));
      bl.n1b = upload(H, padded(T.get(p + "norm1.bias", C), C, Cp));
      bl.n2g = upload(H, padded(T.get(p + "norm2.weight", C), C, Cp));
      bl.n2b = upload(H, padded(T.get(p + "norm2.bias", C), C, Cp));
      // cpb_pre [N*N][heads] -> [heads][N][N], key column k of query row q stored at
      // k ^ ((q % 8) * 4) (the attention kernel's shared-memory reads are then free of
      // bank conflicts); logit scale -> exp(min(ls, ln 100)). Both times log2 e: the
      // attention kernel's softmax is exp2. A checkpoint without the precomputed
      // table but with the CPB MLP gets the table computed on the device, once.
      const float kLog2e = 1.4426950408889634f;
      if (T.has(p + "attn.cpb_pre") || !T.has(p + "attn.cpb_mlp.0.weight")) {
        const float* cpb = T.get(p + "attn.cpb_pre", (int64_t)n * n * heads);
        std::vector<float> cpbt((size_t)heads * n * n, 0.0f);
        for (int q = 0; q < n; q++)
          for (int k = 0; k < n; k++)
            for (int h = 0; h < heads; h++)
              cpbt[((size_t)h * n + q) * n + (k ^ ((q & 7) << 2))] =
                  cpb[((size_t)q * n + k) * heads + h] * kLog2e;
        bl.cpb = upload(H, cpbt);
        if (H->fused_attn) {
          // compact table: entry 40 (dy + 7) + dx + 7 for query - key = (dy, dx)
          std::vector<float> cc((size_t)heads * 576, 0.0f);
          for (int dy = -7; dy <= 7; dy++)
            for (int dx = -7; dx <= 7; dx++) {
              const int qy = std::max(dy, 0), qx = std::max(dx, 0);
              const int qi = qy * 8 + qx, ki = (qy - dy) * 8 + (qx - dx);
              for (int h = 0; h < heads; h++)
                cc[(size_t)h * 576 + 40 * (dy + 7) + dx + 7] =
                    cpb[((size_t)qi * n + ki) * heads + h] * kLog2e;
            }
          bl.cpbc = upload(H, cc);
        }
      } else {
        bl.cpb = cpb_from_mlp(H, T, p, heads, tmp);
        if (H->fused_attn) {
          bl.cpbc = upload(H, std::vector<float>((size_t)heads * 576, 0.0f));
          ck(launch_cpb_compact(bl.cpb, bl.cpbc, heads, 0), "cpb compact table");
        }
      }
      const float* ls = T.get(p + "attn.logit_scale", heads);
      std::vector<float> lse(heads);
      for (int h = 0; h < heads; h++)
        lse[h] = std::exp(std::fmin(ls[h], std::log(100.0f))) * kLog2e;
      bl.ls = upload(H, lse);
    }
    char cn[64], pn[64], cb[64], pb[64];
    snprintf(cn, sizeof cn, "layers.%d.conv.weight", s);
    snprintf(cb, sizeof cb, "layers.%d.conv.bias", s);
    snprintf(pn, sizeof pn, "layers.%d.patch_embed.proj.weight", s);
    snprintf(pb, sizeof pb, "layers.%d.patch_embed.proj.bias", s);
    pack_conv(H, st.conv, T.get(cn, (int64_t)C * C * 9), T.get(cb, C), C, Cp, Cp, Cp,
              identity_rows(Cp, C), sp);
    pack_linear(H, st.pe, T.get(pn, (int64_t)C * C), T.get(pb, C), C, Cp, Cp, Cp,
                identity_rows(Cp, C), sp);
  }
  // head
  const int F = H->feat;
  // body-plane convs (input: the two-term AO plane when split) and 64-channel head
  // convs (single-term planes)
  auto conv_plain = [&](TcWeight& tw, const std::string& name, int ci, int Cip, int co, int N,
                        bool two = false) {
    pack_conv(H, tw, T.get(name + ".weight", (int64_t)co * ci * 9), T.get(name + ".bias", co), ci,
              Cip, N, n_tile_for(N), identity_rows(N, co), two);
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
      conv_plain(H->cbu, "conv_before_upsample.0", C, Cp, F, F, sp);
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
      conv_plain(H->direct, "upsample.0", C, Cp, oc, pad_to(oc, 32), sp);
      break;
    }
    case S2S_NEARESTCONV:
      conv_plain(H->cbu, "conv_before_upsample.0", C, Cp, F, F, sp);
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
  if (P.gexec) cudaGraphExecDestroy(P.gexec);
  P.gexec = nullptr;
  for (void* p : P.ipc_maps) cudaIpcCloseMemHandle(p);
  P.ipc_maps.clear();
  P.mb = nullptr;
  P.prevp = HaloPeer();
  P.nextp = HaloPeer();
  for (void* p : P.allocs) cudaFree(p);
  P.allocs.clear();
}

// The peer-store halo transport of a band plan: export this rank's X16 and AO planes
// and a zeroed mailbox as CUDA IPC handles, trade them with both neighbours over the
// NCCL communicator (every rank builds its plan for the same image at the same
// time), and map the neighbours'. Collective over the ranks, like the exchanges.
struct IpcCard {
  cudaIpcMemHandle_t x16, ao, mb;
  int halo, own_rows, pad[2];
};

void setup_ipc(s2s_handle* H, Plan& P) {
  P.mb = (HaloMailbox*)dalloc(P, sizeof(HaloMailbox));
  IpcCard mine;
  memset(&mine, 0, sizeof mine);
  ck(cudaIpcGetMemHandle(&mine.x16, P.X16), "IPC handle of the X16 plane");
  ck(cudaIpcGetMemHandle(&mine.ao, P.AO), "IPC handle of the AO plane");
  ck(cudaIpcGetMemHandle(&mine.mb, P.mb), "IPC handle of the halo mailbox");
  mine.halo = P.halo;
  mine.own_rows = P.own_rows;
  const NcclApi& api = nccl_api();
  ncclComm_t comm = (ncclComm_t)H->nccl_comm;
  const int prev = (P.rank + P.world - 1) % P.world, next = (P.rank + 1) % P.world;
  IpcCard cards[2];  // from prev, from next
  char* d = (char*)dalloc(P, 3 * sizeof(IpcCard));
  ck(cudaMemcpy(d, &mine, sizeof mine, cudaMemcpyHostToDevice), "IPC card");
  auto nck = [&](ncclResult_t r) {
    if (r != ncclSuccess) fail(S2S_ERR_NCCL, std::string("IPC card exchange: ") + api.GetErrorString(r));
  };
  // sends to next before prev, receives from prev before next (pairs up at 2 ranks)
  nck(api.GroupStart());
  nck(api.Send(d, sizeof(IpcCard), ncclInt8, next, comm, H->stream));
  nck(api.Send(d, sizeof(IpcCard), ncclInt8, prev, comm, H->stream));
  nck(api.Recv(d + sizeof(IpcCard), sizeof(IpcCard), ncclInt8, prev, comm, H->stream));
  nck(api.Recv(d + 2 * sizeof(IpcCard), sizeof(IpcCard), ncclInt8, next, comm, H->stream));
  nck(api.GroupEnd());
  ck(cudaStreamSynchronize(H->stream), "IPC card exchange");
  ck(cudaMemcpy(cards, d + sizeof(IpcCard), sizeof cards, cudaMemcpyDeviceToHost), "IPC card");
  auto open = [&](const cudaIpcMemHandle_t& h) {
    void* p = nullptr;
    ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "IPC mapping of a neighbour");
    P.ipc_maps.push_back(p);
    return p;
  };
  auto peer = [&](const IpcCard& c) {
    HaloPeer q;
    q.x16 = open(c.x16);
    q.ao = open(c.ao);
    q.mb = (HaloMailbox*)open(c.mb);
    q.halo = c.halo;
    q.own_rows = c.own_rows;
    return q;
  };
  P.prevp = peer(cards[0]);
  P.nextp = prev == next ? P.prevp : peer(cards[1]);
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
  b += 3 * T * H->Cs * 2;                   // F0h, X16, AO
  b += (H->fused_attn ? 0 : T * H->NQs * 2) + (H->fused_mlp ? 0 : T * H->HIDs * 2);  // QKV, H16
  b += 2 * T * 4;                           // window row tables
  b += T * 64 * 2 + 3 * T * s * s * 64 * 2; // head planes
  if (H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX)
    b += (int64_t)B * 3 * hp * s * wp * s * 4 + T * s * s * 64 * 4 + (int64_t)B * 3 * hp * wp * 4;
  return b;
}

Plan* get_plan(s2s_handle* H, int B, int h, int w) {
  const int band = H->band_world > 1;
  if (H->plan && H->plan->B == B && H->plan->h == h && H->plan->w == w && H->plan->band == band)
    return H->plan.get();
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
  P->ghp = (h / win + 1) * win;
  P->wp = (w / win + 1) * win;
  const int wp = P->wp, nww = wp / 8;
  if (!band) {
    P->hp = P->ghp;
    P->own_rows = P->hp;
    P->M_own = P->M_sh = B * P->hp * wp;
    for (int i = 0; i < 2; i++) {
      P->nwh_l[i] = P->hp / 8;
      P->nwin[i] = B * P->nwh_l[i] * nww;
    }
    P->conv_H = P->conv_y1 = P->hp;
    P->head_rows = P->hp;
    P->crop_rows = h;
  } else {
    if (B != 1) fail(S2S_ERR_INVALID, "a row-band sharded forward takes one image");
    P->band = 1;
    P->rank = H->band_rank;
    P->world = H->band_world;
    int w0, w1;
    if (P->world > P->ghp / 8)
      fail(S2S_ERR_INVALID, std::to_string(P->world) + " bands need at least as many window "
                            "rows; the padded plane has " + std::to_string(P->ghp / 8));
    band_partition(P->ghp / 8, P->world, P->rank, &w0, &w1);
    P->R0 = 8 * w0;
    P->R1 = 8 * w1;
    const int nb = w1 - w0;
    P->halo = 8;
    P->own_rows = 8 * nb;
    P->hp = P->own_rows + 2 * P->halo;
    P->own_off = (size_t)P->halo * wp;
    P->M_own = P->own_rows * wp;
    // shifted windows cover global rows [R0 - 4, R1 + 4): local [4, hp - 4)
    P->sh_off = (size_t)(P->halo - 4) * wp;
    P->M_sh = (P->own_rows + 8) * wp;
    P->nwh_l[0] = nb;
    P->nwin[0] = nb * nww;
    P->wh_off[0] = w0;
    P->nwh_l[1] = nb + 1;
    P->nwin[1] = (nb + 1) * nww;
    P->wh_off[1] = w0 - 1;
    // 3x3 convs: the map starts one row above the owned rows and ends one below
    P->conv_row0 = P->halo - 1;
    P->conv_H = P->own_rows + 2;
    P->conv_y0 = 1;
    P->conv_y1 = P->own_rows + 1;
    // the head: 4 neighbour rows on interior sides (its receptive field is under 3
    // low-resolution rows), the plane's own edge on the outer ones
    P->head_row0 = P->rank == 0 ? P->halo : P->halo - 4;
    const int head_end = P->halo + P->own_rows + (P->rank == P->world - 1 ? 0 : 4);
    P->head_rows = head_end - P->head_row0;
    P->crop_y0 = P->halo - P->head_row0;
    P->crop_rows = std::max(0, std::min(P->R1, h) - P->R0);
  }
  const int hp = P->hp;
  const size_t T = (size_t)B * hp * wp;
  P->T = T;
  const int Cp = H->Cp, Cs = H->Cs, s = H->cfg.scale;
  const size_t Th = (size_t)B * P->head_rows * wp;  // head plane tokens
  try {
    P->P = (float*)dalloc(*P, (size_t)B * 3 * hp * wp * 4);
    P->F0 = (float*)dalloc(*P, T * Cp * 4);
    P->X = (float*)dalloc(*P, T * Cp * 4);
    P->S = (float*)dalloc(*P, T * Cp * 4);
    P->F0h = (__half*)dalloc(*P, T * Cs * 2);
    P->X16 = (__half*)dalloc(*P, T * Cs * 2);
    P->AO = (__half*)dalloc(*P, T * Cs * 2);
    if (!H->fused_attn) P->QKV = (__half*)dalloc(*P, T * H->NQs * 2);
    if (!H->fused_mlp) P->H16 = (__half*)dalloc(*P, T * H->HIDs * 2);
    for (int i = 0; i < 2; i++) P->rows[i] = (int*)dalloc(*P, (size_t)P->nwin[i] * 64 * 4);
    P->HA = (__half*)dalloc(*P, Th * 64 * 2);
    for (int i = 0; i < 3; i++) P->HB[i] = (__half*)dalloc(*P, Th * s * s * 64 * 2);
    if (H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX) {
      P->BIC = (float*)dalloc(*P, (size_t)B * 3 * hp * s * wp * s * 4);
      P->BICF = (float*)dalloc(*P, T * s * s * 64 * 4);
      P->AUXRAW = (float*)dalloc(*P, (size_t)B * 3 * hp * wp * 4);
    }
  } catch (...) {
    free_plan(*P);
    throw;
  }
  // Window row tables: window-major token -> local plane row.
  {
    std::vector<int> rt[2];
    if (!band) {
      const int hw = hp * wp;
      for (auto& v : rt) v.resize(T);
      for (int b = 0; b < B; b++) {
        const int o = b * hw;
        for (int r = 0; r < hw; r++) {
          rt[0][o + r] = o + token_pixel(r, hp, wp, 0);
          rt[1][o + r] = o + token_pixel(r, hp, wp, win / 2);
        }
      }
    } else {
      // unshifted: the owned window rows; shifted: window rows straddling them,
      // local rows [4 + 8j, 12 + 8j), columns rolled by 4 with the plane's wrap
      for (int sh = 0; sh < 2; sh++) {
        rt[sh].resize((size_t)P->nwin[sh] * 64);
        const int y00 = sh ? P->halo - 4 : P->halo, x0 = sh ? win / 2 : 0;
        for (int wi = 0; wi < P->nwin[sh]; wi++)
          for (int t = 0; t < 64; t++) {
            const int y = y00 + (wi / nww) * 8 + t / 8;
            const int x = ((wi % nww) * 8 + t % 8 + x0) % wp;
            rt[sh][(size_t)wi * 64 + t] = y * wp + x;
          }
      }
    }
    for (int i = 0; i < 2; i++)
      ck(cudaMemcpy(P->rows[i], rt[i].data(), rt[i].size() * 4, cudaMemcpyHostToDevice),
         "row table upload");
  }
  // TMA maps over the activation buffers (the per-token GEMMs read the owned rows).
  bool ok = true;
  ok &= make_map_rows(&P->mF0h, P->F0h + P->own_off * Cs, P->M_own, Cs, 128);
  ok &= make_map_rows(&P->mX16, P->X16 + P->own_off * Cs, P->M_own, Cs, 128);
  ok &= make_map_rows(&P->mX16s, P->X16 + P->sh_off * Cs, P->M_sh, Cs, 128);
  if (band) {
    ok &= make_map_rows(&P->mX16t, P->X16 + P->sh_off * Cs, (uint64_t)4 * wp, Cs, 128);
    ok &= make_map_rows(&P->mX16b, P->X16 + (P->own_off + P->M_own) * Cs, (uint64_t)4 * wp, Cs,
                        128);
  }
  ok &= make_map_rows(&P->mAO, P->AO + P->own_off * Cs, P->M_own, Cs, 128);
  if (P->H16) ok &= make_map_rows(&P->mH16, P->H16 + P->own_off * H->HIDs, P->M_own, H->HIDs, 128);
  {
    int bw, bh;
    conv_box(wp, &bw, &bh);
    ok &= make_map_nhwc(&P->cX16, P->X16 + (size_t)P->conv_row0 * wp * Cs, B, P->conv_H, wp, Cs,
                        bw, bh);
    ok &= make_map_nhwc(&P->cAO, P->AO + (size_t)P->head_row0 * wp * Cs, B, P->head_rows, wp, Cs,
                        bw, bh);
    ok &= make_map_nhwc(&P->cHA, P->HA, B, P->head_rows, wp, 64, bw, bh);
    if (H->fused_attn) ok &= make_map_nhwc(&P->mXw, P->X16, B, hp, wp, Cs, 4, 4);
  }
  for (int i = 0; i < 3; i++)
    for (int r = 0; r < 3; r++) {
      const int f = 1 << r;  // resolution factor 1, 2, 4
      if (f > s && r > 0) continue;
      int bw, bh;
      conv_box(wp * f, &bw, &bh);
      ok &= make_map_nhwc(&P->cHB[i][r], P->HB[i], B, P->head_rows * f, wp * f, 64, bw, bh);
      P->hbp[i][r] = bw <= 32 && bw % 8 == 0 &&
                     make_map_nhwc(&P->cHBp[i][r], P->HB[i], B, P->head_rows * f, wp * f, 64,
                                   bw, bh + 2);
    }
  if (!ok) {
    free_plan(*P);
    fail(S2S_ERR_CUDA, "cuTensorMapEncodeTiled failed for an activation operand");
  }
  if (band && H->nccl_comm && H->halo_ipc) {
    try {
      setup_ipc(H, *P);
    } catch (...) {
      free_plan(*P);
      throw;
    }
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
  // A transfer between bands (NCCL's kernels or copies, not ours): timed like a
  // launch, not counted as one.
  template <typename F>
  void comm(const char* name, cudaStream_t cs, F&& f) {
    if (H->stop_after >= 0 && H->fwd_launches >= H->stop_after) return;
    const bool timed = H->profiling && (H->prof_only.empty() ||
                                        strncmp(name, H->prof_only.c_str(), H->prof_only.size()) == 0);
    cudaEvent_t a = nullptr, b = nullptr;
    if (timed) {
      a = ev();
      b = ev();
      ck(cudaEventRecord(a, cs), "event");
    }
    f();
    if (timed) {
      ck(cudaEventRecord(b, cs), "event");
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

// A 3x3 convolution over the B x H x W plane of the A map, writing output rows [y0, y1).
GemmArgs conv_args(int B, int H, int W, int Cip, int N, const Epi& e, int y0, int y1) {
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
  a.y_off = y0;
  a.y_end = y1;
  a.tiles_y = (y1 - y0 + a.boxh - 1) / a.boxh;
  a.epi = e;
  a.epi.n_valid = e.n_valid ? e.n_valid : N;
  return a;
}

// Two-term operands: A rows [hi | lo] of `kc` 64-column chunks each, B [hi | hi | lo]
// (three K blocks per tap for a convolution).
void two_term(GemmArgs& a, bool split) {
  if (!split) return;
  if (a.conv) {
    a.amod = 2 * a.kc;
    a.kc *= 3;
    a.K *= 3;
  } else {
    a.amod = 2 * (a.K / 64);
    a.K *= 3;
  }
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

// ------------------------------------------------------------------ band halos
// Exchange `n` plane rows of `buf` ([local plane][ld] fp16) with the neighbouring
// bands (halo_ops); without `cyclic`, halo rows beyond the plane's true edges are
// zeroed when `zero_edges`.
void halo_exchange(s2s_handle* H, Plan* P, __half* buf, int ld, int n, bool cyclic,
                   bool zero_edges, cudaStream_t st) {
  const size_t row = (size_t)P->wp * ld;  // halves per plane row
  HaloOp ops[4];
  const int k = halo_ops(P->rank, P->world, P->halo, P->own_rows, n, cyclic, ops);
  if (P->mb) {
    // peer stores: the neighbours' copy of this plane
    auto peer_plane = [&](const HaloPeer& q) -> void* {
      if (buf == P->X16) return q.x16;
      if (buf == P->AO) return q.ao;
      fail(S2S_ERR_INVALID, "halo exchange: a plane without a peer mapping");
      return nullptr;
    };
    const bool has_prev = cyclic || P->rank != 0, has_next = cyclic || P->rank != P->world - 1;
    ck(launch_halo_push(buf, has_prev ? peer_plane(P->prevp) : nullptr,
                        has_next ? peer_plane(P->nextp) : nullptr, P->mb, &P->prevp, &P->nextp,
                        row * 2, n, P->halo, P->own_rows, zero_edges, zero_edges, st,
                        10000000000ull, false),
       "halo push");
    H->launches++;
    return;
  }
  if (H->nccl_comm) {
    const NcclApi& api = nccl_api();
    ncclComm_t comm = (ncclComm_t)H->nccl_comm;
    auto nck = [&](ncclResult_t r) {
      if (r != ncclSuccess)
        fail(S2S_ERR_NCCL, std::string("halo exchange: ") + api.GetErrorString(r));
    };
    nck(api.GroupStart());
    for (int i = 0; i < k; i++) {
      __half* p = buf + (size_t)ops[i].row0 * row;
      if (ops[i].kind == 0)
        nck(api.Send(p, (size_t)ops[i].rows * row, ncclFloat16, ops[i].peer, comm, st));
      else
        nck(api.Recv(p, (size_t)ops[i].rows * row, ncclFloat16, ops[i].peer, comm, st));
    }
    nck(api.GroupEnd());
  } else if (H->group) {
    LocalGroup& G = *H->group;
    const int r = P->rank;
    G.buf[r] = reinterpret_cast<const char*>(buf);
    G.halo[r] = P->halo;
    G.own_rows[r] = P->own_rows;
    ck(cudaEventRecord(G.ready[r], st), "halo event");
    if (!G.barrier(120.0)) fail(S2S_ERR_TIMEOUT, "halo exchange: a band of the group never arrived");
    const size_t rb = row * 2;
    for (int i = 0; i < k; i++) {
      if (ops[i].kind != 1) continue;
      const int q = ops[i].peer;
      // from the rank above: its last n owned rows; from below: its first n
      const bool from_above = ops[i].row0 < P->halo;
      const int src_row = from_above ? G.halo[q] + G.own_rows[q] - n : G.halo[q];
      ck(cudaStreamWaitEvent(st, G.ready[q], 0), "halo wait");
      ck(cudaMemcpyAsync(buf + (size_t)ops[i].row0 * row, G.buf[q] + (size_t)src_row * rb,
                         (size_t)n * rb, cudaMemcpyDeviceToDevice, st),
         "halo copy");
    }
    ck(cudaEventRecord(G.done[r], st), "halo event");
    if (!G.barrier(120.0)) fail(S2S_ERR_TIMEOUT, "halo exchange: a band of the group never arrived");
    // my rows are read by both neighbours' copies: later writes wait for them
    const int prev = (r + P->world - 1) % P->world, next = (r + 1) % P->world;
    ck(cudaStreamWaitEvent(st, G.done[prev], 0), "halo wait");
    ck(cudaStreamWaitEvent(st, G.done[next], 0), "halo wait");
  } else {
    fail(S2S_ERR_INVALID, "band forward without a communicator");
  }
  if (!cyclic && zero_edges) {
    if (P->rank == 0)
      ck(cudaMemsetAsync(buf + (size_t)(P->halo - n) * row, 0, n * row * 2, st), "halo zero");
    if (P->rank == P->world - 1)
      ck(cudaMemsetAsync(buf + (size_t)(P->halo + P->own_rows) * row, 0, n * row * 2, st),
         "halo zero");
  }
}

// ------------------------------------------------------------------ the forward
// One forward over the plan's plane: the whole padded image (B images), or, for a
// sharded forward, this rank's row band (the owned rows' output only; d_out is then
// [3][crop_rows * s][w * s]).
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
  // fp16 operand rows: stride Cs, and with two-term operands the lo terms Cp after hi
  const int Cs = H->Cs, lo = H->split ? Cp : 0;
  const bool sp = H->split;
  const int M = P->M_own;
  const bool band = P->band != 0;
  float* const X = P->X + P->own_off * Cp;       // owned rows of the residual stream
  __half* const X16 = P->X16 + P->own_off * Cs;
  float* const S = P->S + P->own_off * Cp;
  // Halo transfers run on the side stream behind an event, so they start only once
  // every kernel before them has completed (kernels signal their dependents early).
  auto exchange = [&](const char* name, __half* buf, int n, bool cyclic, bool zero_edges) {
    ck(cudaEventRecord(H->fork, st), "fork");
    ck(cudaStreamWaitEvent(H->side, H->fork, 0), "fork");
    L.comm(name, H->side, [&] { halo_exchange(H, P, buf, Cs, n, cyclic, zero_edges, H->side); });
    ck(cudaEventRecord(H->join, H->side), "join");
    ck(cudaStreamWaitEvent(st, H->join, 0), "join");
  };
  // 1. pad + conv_first (fp32 body skip F0, fp16 operand F0h).
  if (!band) {
    L.run("pad_reflect", [&] { return launch_pad_reflect(d_in, P->P, B, 3, h, w, hp, wp, st); });
  } else {
    L.run("pad_reflect", [&] {
      return launch_pad_band(d_in, P->P, 3, h, w, P->ghp, wp, hp, P->R0 - P->halo, st);
    });
  }
  L.run("conv_first", [&] {
    return launch_conv3_small(P->P, H->cf_w, H->cf_b, B, hp, wp, C, 0, 0.0f, P->F0, Cp, P->F0h,
                              Cs, lo, st);
  });
  // 2. top patch_embed: 1x1 + LayerNorm -> X, X16 and the stage input S.
  {
    Epi e = epi0();
    e.bias = H->pe.b;
    e.ln_g = H->pe_g;
    e.ln_b = H->pe_b;
    e.ln_n = C;
    e.n_valid = C;
    e.o32 = X;
    e.ld32 = Cp;
    e.o16 = X16;
    e.ld16 = Cs;
    e.lo_off = lo;
    e.o32b = S;
    e.ld32b = Cp;
    GemmArgs a = gemm_args(M, Cp, Cp, e);
    two_term(a, sp);
    L.run("gemm_patch_embed", [&] { return launch_gemm(P->mF0h, H->pe.map, out_maps(P, a), a, Cp, st); });
  }
  for (int si = 0; si < c.n_depths; si++) {
    Stage& stg = H->stages[si];
    const int depth = c.depths[si];
    for (int b = 0; b < depth; b++) {
      Block& bl = stg.blocks[b];
      const int sh = (b % 2 == 1) ? c.window / 2 : 0;
      const int k = sh ? 1 : 0;
      auto qkv = [&](const CUtensorMap& mA, size_t off, int rows) {
        Epi e = epi0();
        e.bias = bl.qkv.b;
        e.act = ACT_QKNORM;  // normalised q (times the logit scale) and k for the attention
        e.qk_scale = bl.ls;
        e.qk_dp = H->DP;
        e.o16 = P->QKV + off * H->NQs;
        e.ld16 = H->NQs;
        e.lo_off = sp ? H->NQ : 0;
        GemmArgs a = gemm_args(rows, H->NQ, Cp, e);
        two_term(a, sp);
        L.run("gemm_qkv", [&] { return launch_gemm(mA, bl.qkv.map, out_maps(P, a), a, bl.qkv.BN, st); });
      };
      if (H->fused_attn) {
        // QKV projection + attention in one kernel; the shifted windows' 4 rows from each
        // neighbouring band (cyclically) arrive first
        if (band && sh) exchange("halo_shift", P->X16, 4, true, false);
        QaArgs qa;
        memset(&qa, 0, sizeof qa);
        qa.out = P->AO;
        qa.ld_out = Cs;
        qa.qb = bl.qb;
        qa.vb = bl.vb;
        qa.ls = bl.ls;
        qa.bias = bl.cpbc;
        qa.nww = wp / 8;
        qa.wp = wp;
        qa.hp_l = hp;
        qa.ghp = P->ghp;
        qa.y_mod = hp;
        qa.shift = sh;
        if (!band) {
          qa.B = B;
          qa.nw_img = (hp / 8) * (wp / 8);
          qa.y_base = sh;
        } else {
          qa.B = 1;
          qa.nw_img = P->nwin[k];
          qa.y_base = P->halo - sh;
          qa.wh_off = P->wh_off[k];
        }
        qa.nwin_total = P->nwin[k];
        L.run("qkv_attention", [&] { return launch_qkv_attention(P->mXw, bl.wqkv.map, qa, st); });
      } else if (band && sh) {
        // The shifted windows reach 4 rows into each neighbouring band (cyclically).
        // Those rows travel on the side stream while the owned rows' QKV runs; the
        // halo rows' QKV follows their arrival.
        ck(cudaEventRecord(H->fork, st), "fork");
        ck(cudaStreamWaitEvent(H->side, H->fork, 0), "fork");
        L.comm("halo_shift", H->side,
               [&] { halo_exchange(H, P, P->X16, Cs, 4, true, false, H->side); });
        ck(cudaEventRecord(H->join, H->side), "join");
        qkv(P->mX16, P->own_off, M);
        ck(cudaStreamWaitEvent(st, H->join, 0), "join");
        qkv(P->mX16t, P->sh_off, 4 * wp);
        qkv(P->mX16b, P->own_off + M, 4 * wp);
      } else {
        qkv(P->mX16, P->own_off, M);
      }
      if (!H->fused_attn)
        L.run("window_attention", [&] {
          return launch_window_attention(P->QKV, P->AO, bl.cpb, P->rows[k], P->nwin[k],
                                         H->heads, H->hd, H->DP, Cs, H->NQs, sp, H->NQ, lo,
                                         P->nwh_l[k], wp / 8, P->ghp, wp, sh, P->wh_off[k], st);
        });
      if (!H->fused_proj) {  // proj + norm1 + residual, in place
        Epi e = epi0();
        e.bias = bl.proj.b;
        e.ln_g = bl.n1g;
        e.ln_b = bl.n1b;
        e.ln_n = C;
        e.n_valid = C;
        e.res_post = X;
        e.ld_res_post = Cp;
        e.o32 = X;
        e.ld32 = Cp;
        e.o16 = X16;
        e.ld16 = Cs;
        e.lo_off = lo;
        GemmArgs a = gemm_args(M, Cp, Cp, e);
        two_term(a, sp);
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
        m.x = X;
        m.x16 = X16;
        m.bp = bl.proj.b;
        m.g1 = bl.n1g;
        m.beta1 = bl.n1b;
        // with fused_proj the kernel starts from AO: proj + norm1 + residual, then the MLP
        L.run(H->fused_proj ? "proj_mlp" : "mlp_fused", [&] {
          Epi eo = epi0();
          eo.o32 = X;
          eo.ld32 = Cp;
          eo.o16 = X16;
          eo.ld16 = Cs;
          const OutMaps om = out_maps(P, gemm_args(M, Cp, Cp, eo));
          return launch_mlp(H->fused_proj ? P->mAO : P->mX16, bl.fc1.mlp_map, bl.fc2.map, om.o32,
                            om.o16, m, Cp, H->HIDp, st, H->fused_proj ? &bl.proj.map : nullptr);
        });
      } else {
        {  // fc1 + GELU
          Epi e = epi0();
          e.bias = bl.fc1.b;
          e.act = ACT_GELU;
          e.o16 = P->H16 + P->own_off * H->HIDs;
          e.ld16 = H->HIDs;
          e.lo_off = sp ? H->HIDp : 0;
          GemmArgs a = gemm_args(M, H->HIDp, Cp, e);
          two_term(a, sp);
          L.run("gemm_fc1", [&] { return launch_gemm(P->mX16, bl.fc1.map, out_maps(P, a), a, bl.fc1.BN, st); });
        }
        {  // fc2 + norm2 + residual, in place
          Epi e = epi0();
          e.bias = bl.fc2.b;
          e.ln_g = bl.n2g;
          e.ln_b = bl.n2b;
          e.ln_n = C;
          e.n_valid = C;
          e.res_post = X;
          e.ld_res_post = Cp;
          e.o32 = X;
          e.ld32 = Cp;
          e.o16 = X16;
          e.ld16 = Cs;
          e.lo_off = lo;
          GemmArgs a = gemm_args(M, Cp, H->HIDp, e);
          two_term(a, sp);
          L.run("gemm_fc2", [&] { return launch_gemm(P->mH16, bl.fc2.map, out_maps(P, a), a, Cp, st); });
        }
      }
    }
    // RSTB tail: conv3x3 -> 1x1 patch_embed + stage residual.
    if (band) exchange("halo_conv", P->X16, 1, false, true);
    {
      Epi e = epi0();
      e.bias = stg.conv.b;
      e.n_valid = C;
      e.o16 = P->AO + (size_t)P->conv_row0 * wp * Cs;
      e.ld16 = Cs;
      e.lo_off = lo;
      GemmArgs a = conv_args(B, P->conv_H, wp, Cp, Cp, e, P->conv_y0, P->conv_y1);
      two_term(a, sp);
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
        e.res_pre = S;
        e.ld_res_pre = Cp;
      } else {
        e.res_post = S;
        e.ld_res_post = Cp;
      }
      if (!last) {
        e.o32 = X;
        e.ld32 = Cp;
        e.o16 = X16;
        e.ld16 = Cs;
        e.o32b = S;
        e.ld32b = Cp;
      } else {  // + final norm, image order, fp16 operand of conv_after_body
        e.ln_g = H->nrm_g;
        e.ln_b = H->nrm_b;
        e.ln_n = C;
        e.o16 = X16;
        e.ld16 = Cs;
      }
      e.lo_off = lo;
      GemmArgs a = gemm_args(M, Cp, Cp, e);
      two_term(a, sp);
      L.run(last ? "gemm_stage_pe_norm" : "gemm_stage_pe",
            [&] { return launch_gemm(P->mAO, stg.pe.map, out_maps(P, a), a, Cp, st); });
    }
  }
  // 3. conv_after_body + body skip (conv_first output) -> Y16 (in AO).
  if (band) exchange("halo_conv", P->X16, 1, false, true);
  {
    Epi e = epi0();
    e.bias = H->cab.b;
    e.n_valid = C;
    e.res_post = P->F0 + (size_t)P->conv_row0 * wp * Cp;
    e.ld_res_post = Cp;
    e.o16 = P->AO + (size_t)P->conv_row0 * wp * Cs;
    e.ld16 = Cs;
    e.lo_off = lo;
    GemmArgs a = conv_args(B, P->conv_H, wp, Cp, Cp, e, P->conv_y0, P->conv_y1);
    two_term(a, sp);
    L.run("conv_after_body", [&] { return launch_gemm(P->cX16, H->cab.map, out_maps(P, a), a, Cp, st); });
  }
  // 4. head, on its own plane: head_rows x wp (the whole padded plane unless banded).
  if (band) exchange("halo_head", P->AO, 4, false, false);
  const int hh0 = P->head_rows;
  // `two`: the input plane is the body's two-term AO plane
  auto conv_to = [&](const char* name, const CUtensorMap& mapA, const TcWeight& tw, int Hh, int Ww,
                     int Cip, Epi e, bool two = false) {
    GemmArgs a = conv_args(B, Hh, Ww, Cip, tw.N, e, 0, Hh);
    two_term(a, two && sp);
    L.run(name, [&] { return launch_gemm(mapA, tw.map, out_maps(P, a), a, tw.BN, st); });
  };
  // a 64-channel conv over head plane HB[i] at resolution 2^r, from kx patches when
  // the plane's conv box allows them
  auto conv_plane = [&](const char* name, int i, int r, const TcWeight& tw, int Hh, int Ww,
                        Epi e) {
    if (!P->hbp[i][r] || H->no_patch) {
      conv_to(name, P->cHB[i][r], tw, Hh, Ww, F, e);
      return;
    }
    GemmArgs a = conv_args(B, Hh, Ww, F, tw.N, e, 0, Hh);
    a.patch = 1;
    L.run(name, [&] { return launch_gemm(P->cHBp[i][r], tw.map, out_maps(P, a), a, tw.BN, st); });
  };
  auto cbu = [&]() {
    Epi e = epi0();
    e.bias = H->cbu.b;
    e.act = ACT_LRELU;
    e.slope = 0.01f;
    e.o16 = P->HA;
    e.ld16 = F;
    conv_to("conv_before_upsample", P->cAO, H->cbu, hh0, wp, Cp, e, true);
  };
  // conv_last over head plane HB[i] at resolution 2^r: from kx patches of the plane
  // when its conv box allows them (three input fetches per tile instead of nine)
  auto final_planes = [&](int i, int r, int Hh, int Ww) {
    Epi e = epi0();
    e.bias = H->last.b;
    e.store = STORE_PLANES;
    e.planes = d_out;
    e.crop_y0 = P->crop_y0 * s;
    e.crop_h = P->crop_rows * s;
    e.crop_w = w * s;
    set_final(H, e);
    if (!P->hbp[i][r] || H->no_patch) {
      conv_to("conv_last", P->cHB[i][r], H->last, Hh, Ww, F, e);
      return;
    }
    GemmArgs a = conv_args(B, Hh, Ww, F, H->last.N, e, 0, Hh);
    a.patch = 1;
    L.run("conv_last", [&] {
      return launch_gemm(P->cHBp[i][r], H->last.map, out_maps(P, a), a, H->last.BN, st);
    });
  };
  switch (c.upsampler) {
    case S2S_PIXELSHUFFLE:
    case S2S_PIXELSHUFFLE_AUX: {
      cbu();
      const CUtensorMap* src = &P->cHA;
      int hh = hh0, ww = wp;
      const int octs = (int)std::lround(std::log2((double)s));
      if (c.upsampler == S2S_PIXELSHUFFLE_AUX) {
        if (band) fail(S2S_ERR_UNSUPPORTED, "the pixelshuffle_aux head has no band mode");
        // bicubic branch of the padded, mean-adjusted input, on the padded output grid
        L.run("bicubic", [&] {
          return launch_bicubic(P->P, P->BIC, B * 3, hp, wp, hp * s, wp * s, st);
        });
        L.run("conv_bicubic", [&] {
          return launch_conv3_small(P->BIC, H->cbic_w, H->cbic_b, B, hp * s, wp * s, F, 0, 0.0f,
                                    P->BICF, F, nullptr, 0, 0, st);
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
                                    nullptr, 0, P->HB[2], F, 0, st);
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
      final_planes((octs - 1) % 2, octs, hh, ww);
      break;
    }
    case S2S_PIXELSHUFFLEDIRECT: {
      Epi e = epi0();
      e.bias = H->direct.b;
      e.store = STORE_DIRECT;
      e.planes = d_out;
      e.scale = s;
      e.crop_y0 = P->crop_y0 * s;
      e.crop_h = P->crop_rows * s;
      e.crop_w = w * s;
      set_final(H, e);
      conv_to("conv_upsample_direct", P->cAO, H->direct, hh0, wp, Cp, e, true);
      break;
    }
    case S2S_NEARESTCONV: {
      cbu();
      L.run("upsample_nearest", [&] { return launch_up2_nhwc(P->HA, P->HB[0], B, hh0, wp, F, st); });
      {
        Epi e = epi0();
        e.bias = H->up1.b;
        e.act = ACT_LRELU;
        e.slope = 0.2f;
        e.o16 = P->HB[1];
        e.ld16 = F;
        conv_plane("conv_up1", 0, 1, H->up1, 2 * hh0, 2 * wp, e);
      }
      L.run("upsample_nearest",
            [&] { return launch_up2_nhwc(P->HB[1], P->HB[0], B, 2 * hh0, 2 * wp, F, st); });
      {
        Epi e = epi0();
        e.bias = H->up2.b;
        e.act = ACT_LRELU;
        e.slope = 0.2f;
        e.o16 = P->HB[2];
        e.ld16 = F;
        conv_plane("conv_up2", 0, 2, H->up2, 4 * hh0, 4 * wp, e);
      }
      {
        Epi e = epi0();
        e.bias = H->hr.b;
        e.act = ACT_LRELU;
        e.slope = 0.2f;
        e.o16 = P->HB[0];
        e.ld16 = F;
        conv_plane("conv_hr", 2, 2, H->hr, 4 * hh0, 4 * wp, e);
      }
      final_planes(0, 2, 4 * hh0, 4 * wp);
      break;
    }
    default:
      fail(S2S_ERR_UNSUPPORTED, "unknown upsampler");
  }
}

// forward_device, replayed from a CUDA graph when the same plan and I/O pointers
// come back: the first forward runs eagerly (and sets up every kernel), the second
// is captured on the handle's stream and launched, later ones only launch. Eager
// always under the profiler, a debug stop, or an in-process band group (whose
// exchange synchronises on the host).
void run_forward(s2s_handle* H, int B, int h, int w, const float* d_in, float* d_out,
                 float* d_aux, cudaStream_t st) {
  if (!H->graphs || H->profiling || H->stop_after >= 0 || H->group) {
    forward_device(H, B, h, w, d_in, d_out, d_aux, st);
    return;
  }
  Plan* P = get_plan(H, B, h, w);
  if (P->g_in != d_in || P->g_out != d_out || P->g_aux != d_aux) {
    if (P->gexec) cudaGraphExecDestroy(P->gexec);
    P->gexec = nullptr;
    P->g_in = d_in;
    P->g_out = d_out;
    P->g_aux = d_aux;
    P->g_seen = 0;
  }
  if (P->gexec) {
    ck(cudaGraphLaunch(P->gexec, st), "graph launch");
    H->launches += P->g_launches;
    return;
  }
  if (P->g_seen++ == 0) {
    forward_device(H, B, h, w, d_in, d_out, d_aux, st);
    return;
  }
  // capture on the handle's own (non-blocking) stream, ordered after `st`
  cudaEvent_t e0 = nullptr;
  ck(cudaEventCreateWithFlags(&e0, cudaEventDisableTiming), "graph event");
  cudaStream_t cs = H->stream;
  ck(cudaEventRecord(e0, st), "graph event");
  ck(cudaStreamWaitEvent(cs, e0, 0), "graph event");
  cudaEventDestroy(e0);
  ck(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "graph capture");
  const long long l0 = H->launches;
  cudaGraph_t g = nullptr;
  try {
    forward_device(H, B, h, w, d_in, d_out, d_aux, cs);
  } catch (...) {
    cudaStreamEndCapture(cs, &g);
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    throw;
  }
  ck(cudaStreamEndCapture(cs, &g), "graph capture");
  const cudaError_t ie = cudaGraphInstantiate(&P->gexec, g, 0);
  cudaGraphDestroy(g);
  ck(ie, "graph instantiate");
  P->g_launches = H->launches - l0;
  H->launches = l0;
  ck(cudaGraphLaunch(P->gexec, st), "graph launch");
  H->launches += P->g_launches;
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

// The device address of a page-locked (pinned, mapped) host buffer, or null for
// pageable memory: the final kernels then store the output straight into the
// caller's buffer and no separate download runs.
float* pinned_alias(float* host) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, host) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
  return static_cast<float*>(at.devicePointer);
}

void ensure_staging(s2s_handle* H, float** p, size_t* have, size_t n) {
  if (*have >= n) return;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  ck(cudaMalloc((void**)p, n * 4), "staging");
  *have = n;
}

const char* const kBandHandle =
    "this handle is one band of a sharded forward (s2s_band_init): use s2s_forward_band";

// Leave band mode: destroy the communicator / leave the group (the plan is rebuilt
// for the new geometry on the next forward).
void release_band(s2s_handle* H) {
  if (H->plan) {  // its graph may hold the communicator's work
    cudaStreamSynchronize(H->stream);
    free_plan(*H->plan);
    H->plan.reset();
  }
  if (H->nccl_comm) {
    const NcclApi& api = nccl_api();
    if (api.ok) api.CommDestroy((ncclComm_t)H->nccl_comm);
    H->nccl_comm = nullptr;
  }
  H->group.reset();
  H->band_rank = 0;
  H->band_world = 1;
}

// The side stream and fork/join events band forwards use (once per handle).
void ensure_side(s2s_handle* H) {
  if (!H->side) ck(cudaStreamCreateWithFlags(&H->side, cudaStreamNonBlocking), "side stream");
  if (!H->fork) ck(cudaEventCreateWithFlags(&H->fork, cudaEventDisableTiming), "event");
  if (!H->join) ck(cudaEventCreateWithFlags(&H->join, cudaEventDisableTiming), "event");
}

// Output rows [r0, r1) of an h-row image that `rank` of `world` bands produces.
void band_out_rows(int h, int window, int world, int rank, int* r0, int* r1) {
  if (world <= 1) {
    *r0 = 0;
    *r1 = h;
    return;
  }
  int w0, w1;
  band_partition((h / window + 1), world, rank, &w0, &w1);
  *r0 = std::min(8 * w0, h);
  *r1 = std::min(8 * w1, h);
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
  // Two-term operands by default for the narrow (Cp = 64) networks; S2S_SPLIT=0 / 1
  // (validation switch) turns them off / on for every width.
  H->split = H->Cp == 64;
  {
    const char* v = getenv("S2S_SPLIT");
    if (v && strcmp(v, "0") == 0) H->split = false;
    if (v && strcmp(v, "1") == 0) H->split = true;
    if (g_create_flags.split >= 0) H->split = g_create_flags.split != 0;
  }
  H->Cs = H->split ? 2 * H->Cp : H->Cp;
  H->NQs = H->split ? 2 * H->NQ : H->NQ;
  H->HIDs = H->split ? 2 * H->HIDp : H->HIDp;
  const bool can_fuse_attn = !H->split && H->Cp == 192 && H->heads == 6 && H->DP == 32;
  H->fused_attn = can_fuse_attn && kFusedAttnDefault;
  {
    const char* v = getenv("S2S_ATTN");
    if (v && strcmp(v, "mma") == 0) H->fused_attn = false;
    if (v && strcmp(v, "fused") == 0) H->fused_attn = can_fuse_attn;
    if (g_create_flags.mma_attn >= 0) H->fused_attn = can_fuse_attn && !g_create_flags.mma_attn;
  }
  // the fused MLP keeps its hidden activation in single-term fp16
  const bool can_fuse = !H->split && ((H->Cp == 192 && H->HIDp == 384) ||
                                      (H->Cp == 64 && H->HIDp == 128));
  H->fused_mlp = can_fuse;
  {
    const char* f = getenv("S2S_UNFUSED_MLP");  // validation switch: the two-GEMM MLP path
    if (f && *f && strcmp(f, "0") != 0) H->fused_mlp = false;
    const char* np = getenv("S2S_NO_PATCH");  // validation switch: conv_last by tap boxes
    H->no_patch = np && strcmp(np, "1") == 0;
    const char* g = getenv("S2S_GRAPHS");
    if (g && strcmp(g, "0") == 0) H->graphs = false;
    if (g_create_flags.unfused_mlp >= 0) H->fused_mlp = can_fuse && g_create_flags.unfused_mlp == 0;
    if (g_create_flags.no_patch >= 0) H->no_patch = g_create_flags.no_patch != 0;
    H->fused_proj = H->fused_mlp && H->Cp == 192 && H->HIDp == 384;
    const char* up = getenv("S2S_UNFUSED_PROJ");
    if (up && strcmp(up, "1") == 0) H->fused_proj = false;
    if (g_create_flags.unfused_proj >= 0)
      H->fused_proj = H->fused_mlp && H->Cp == 192 && H->HIDp == 384 &&
                      g_create_flags.unfused_proj == 0;
  }
  TensorTable T;
  for (int i = 0; i < n_tensors; i++) T.t[tensors[i].name] = &tensors[i];
  int rc = guarded(H.get(), [&] {
    ck(cudaStreamCreateWithFlags(&H->stream, cudaStreamNonBlocking), "stream");
    std::vector<void*> tmp;  // device operands of tables computed at upload
    try {
      build_weights(H.get(), T, tmp);
      ck(cudaDeviceSynchronize(), "weight upload");
    } catch (...) {
      cudaDeviceSynchronize();
      for (void* q : tmp) cudaFree(q);
      throw;
    }
    for (void* q : tmp) cudaFree(q);
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
    if (H->band_world > 1) fail(S2S_ERR_INVALID, kBandHandle);
    if (H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX && !d_aux)
      fail(S2S_ERR_INVALID, "the pixelshuffle_aux head needs an aux buffer on the device path");
    run_forward(H, batch, height, width, d_in, d_out, d_aux, st);
  });
}

int s2s_forward_batch(s2s_handle* H, int batch, int height, int width, const float* in, float* out,
                      float* aux) {
  if (!H || !in || !out) return S2S_ERR_INVALID;
  return guarded(H, [&] {
    if (H->band_world > 1) fail(S2S_ERR_INVALID, kBandHandle);
    const int win = H->cfg.window, s = H->cfg.scale;
    const size_t nin = (size_t)batch * 3 * height * width;
    const size_t nout = (size_t)batch * 3 * height * s * width * s;
    const size_t naux = (size_t)batch * 3 * (height / win + 1) * win * (width / win + 1) * win;
    const bool has_aux = H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX;
    ensure_staging(H, &H->h_in, &H->h_in_n, nin);
    // pinned caller buffers are written by the final kernels directly
    float* d_out = pinned_alias(out);
    float* d_aux = has_aux && aux ? pinned_alias(aux) : nullptr;
    if (!d_out) ensure_staging(H, &H->h_out, &H->h_out_n, nout);
    if (has_aux && !d_aux) ensure_staging(H, &H->h_aux, &H->h_aux_n, naux);
    ck(cudaMemcpyAsync(H->h_in, in, nin * 4, cudaMemcpyHostToDevice, H->stream), "upload");
    run_forward(H, batch, height, width, H->h_in, d_out ? d_out : H->h_out,
                has_aux ? (d_aux ? d_aux : H->h_aux) : nullptr, H->stream);
    if (!d_out)
      ck(cudaMemcpyAsync(out, H->h_out, nout * 4, cudaMemcpyDeviceToHost, H->stream), "download");
    if (has_aux && aux && !d_aux)
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

int64_t s2s_launch_count(const s2s_handle* H) { return H ? H->launches.load() : 0; }

int s2s_debug_halo_loopback(s2s_handle* H, int rows, int missing) {
  if (!H) return S2S_ERR_INVALID;
  return guarded(H, [&] {
    if (rows < 1 || rows > 8) fail(S2S_ERR_INVALID, "s2s_debug_halo_loopback: rows must be in [1, 8]");
    ck(cudaStreamSynchronize(H->stream), "halo loopback");
    // a band plane of 16 owned rows between two 8-row halos, 1 KB a row
    const int halo = 8, own = 16, hp = own + 2 * halo;
    const size_t rb = 1024, plane = (size_t)hp * rb;
    struct Scratch {
      void* p = nullptr;
      ~Scratch() {
        if (p) cudaFree(p);
      }
    } d;
    ck(cudaMalloc(&d.p, plane + 2 * sizeof(HaloMailbox)), "halo loopback scratch");
    uint8_t* dplane = static_cast<uint8_t*>(d.p);
    HaloMailbox* mine = reinterpret_cast<HaloMailbox*>(dplane + plane);
    HaloMailbox* nobody = mine + 1;  // a neighbour that never runs
    std::vector<uint8_t> h(plane, 0);
    for (int r = halo; r < halo + own; r++)
      for (size_t c = 0; c < rb; c++) h[r * rb + c] = (uint8_t)((r * 131 + c * 7 + 1) & 0xff);
    ck(cudaMemcpy(dplane, h.data(), plane, cudaMemcpyHostToDevice), "halo loopback");
    ck(cudaMemset(mine, 0, 2 * sizeof(HaloMailbox)), "halo loopback");
    // both neighbours are this plane; with `missing` their mailbox is one nobody serves
    HaloPeer self;
    self.x16 = dplane;
    self.mb = missing ? nobody : mine;
    self.halo = halo;
    self.own_rows = own;
    for (int e = 1; e <= 2; e++) {
      ck(launch_halo_push(dplane, dplane, dplane, mine, &self, &self, rb, rows, halo, own, false,
                          false, H->stream, 1000000000ull, true),
         "halo loopback");
      ck(cudaStreamSynchronize(H->stream), "halo loopback");
      check_device_error(H);
      unsigned seq = 0;
      ck(cudaMemcpy(&seq, &mine->seq, sizeof seq, cudaMemcpyDeviceToHost), "halo loopback");
      if (seq != (unsigned)e)
        fail(S2S_ERR_CUDA, "halo loopback: exchange " + std::to_string(e) + " left epoch " +
                               std::to_string(seq));
    }
    std::vector<uint8_t> out(plane);
    ck(cudaMemcpy(out.data(), dplane, plane, cudaMemcpyDeviceToHost), "halo loopback");
    // top halo <- the last `rows` owned rows, bottom halo <- the first; the rest as sent
    for (int r = 0; r < hp; r++) {
      int src = r;
      if (r >= halo - rows && r < halo) src = r + own;
      else if (r >= halo + own && r < halo + own + rows) src = r - own;
      if (memcmp(out.data() + r * rb, h.data() + (size_t)src * rb, rb) != 0)
        fail(S2S_ERR_CUDA, "halo loopback: plane row " + std::to_string(r) + " differs");
    }
  });
}

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
  else if (k == "F0h") { p = P.F0h; n = T * H->Cs; half = true; }
  else if (k == "X16") { p = P.X16; n = T * H->Cs; half = true; }
  else if (k == "QKV") { p = P.QKV; n = T * H->NQs; half = true; }
  else if (k == "AO") { p = P.AO; n = T * H->Cs; half = true; }
  else if (k == "H16") { p = P.H16; n = T * H->HIDs; half = true; }
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

int s2s_band_unique_id(void* out, int cap) {
  const NcclApi& api = nccl_api();
  if (!api.ok) {
    g_create_error = api.err;
    return S2S_ERR_NCCL;
  }
  if (!out || cap < (int)sizeof(ncclUniqueId)) {
    g_create_error = "s2s_band_unique_id: the buffer must hold S2S_BAND_ID_BYTES";
    return S2S_ERR_INVALID;
  }
  ncclUniqueId id;
  const ncclResult_t r = api.GetUniqueId(&id);
  if (r != ncclSuccess) {
    g_create_error = std::string("ncclGetUniqueId: ") + api.GetErrorString(r);
    return S2S_ERR_NCCL;
  }
  memcpy(out, &id, sizeof id);
  return S2S_OK;
}

int s2s_band_init(s2s_handle* H, int rank, int world, const void* id, int id_bytes) {
  if (!H) return S2S_ERR_INVALID;
  return guarded(H, [&] {
    if (world < 1 || rank < 0 || rank >= world)
      fail(S2S_ERR_INVALID, "s2s_band_init: rank must be in [0, world)");
    if (world > 1 && H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX)
      fail(S2S_ERR_UNSUPPORTED, "the pixelshuffle_aux head has no band mode (its input is a "
                                "batch of small images: split the batch instead)");
    ck(cudaStreamSynchronize(H->stream), "band init");
    release_band(H);
    if (world > 1) {
      // halo transport: peer stores through IPC mappings, or NCCL send/recv
      const char* ht = getenv("S2S_HALO");
      if (ht && strcmp(ht, "nccl") != 0 && strcmp(ht, "ipc") != 0)
        fail(S2S_ERR_INVALID, std::string("S2S_HALO must be ipc or nccl, not ") + ht);
      H->halo_ipc = !(ht && strcmp(ht, "nccl") == 0);
      if (!id || id_bytes != (int)sizeof(ncclUniqueId))
        fail(S2S_ERR_INVALID, "s2s_band_init: the id must be the S2S_BAND_ID_BYTES of "
                              "s2s_band_unique_id");
      const NcclApi& api = nccl_api();
      if (!api.ok) fail(S2S_ERR_NCCL, api.err);
      ncclUniqueId uid;
      memcpy(&uid, id, sizeof uid);
      ncclComm_t comm = nullptr;
      const ncclResult_t r = api.CommInitRank(&comm, world, uid, rank);
      if (r != ncclSuccess) fail(S2S_ERR_NCCL, std::string("ncclCommInitRank: ") + api.GetErrorString(r));
      H->nccl_comm = comm;
      ensure_side(H);
    }
    H->band_rank = rank;
    H->band_world = world;
  });
}

int s2s_band_init_local(s2s_handle** hs, int world) {
  if (!hs || world < 1) return S2S_ERR_INVALID;
  for (int i = 0; i < world; i++)
    if (!hs[i]) return S2S_ERR_INVALID;
  auto G = std::make_shared<LocalGroup>();
  G->world = world;
  G->buf.assign(world, nullptr);
  G->halo.assign(world, 0);
  G->own_rows.assign(world, 0);
  G->ready.assign(world, nullptr);
  G->done.assign(world, nullptr);
  G->device.assign(world, 0);
  for (int i = 0; i < world; i++) {
    s2s_handle* H = hs[i];
    const int rc = guarded(H, [&] {
      if (world > 1 && H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX)
        fail(S2S_ERR_UNSUPPORTED, "the pixelshuffle_aux head has no band mode");
      ck(cudaStreamSynchronize(H->stream), "band init");
      G->device[i] = H->device;
      ensure_side(H);
      ck(cudaEventCreateWithFlags(&G->ready[i], cudaEventDisableTiming), "band event");
      ck(cudaEventCreateWithFlags(&G->done[i], cudaEventDisableTiming), "band event");
    });
    if (rc != S2S_OK) return rc;
  }
  for (int i = 0; i < world; i++) {
    release_band(hs[i]);
    hs[i]->group = G;
    hs[i]->band_rank = i;
    hs[i]->band_world = world;
  }
  return S2S_OK;
}

int s2s_band_rows(const s2s_handle* H, int height, int* row0, int* row1) {
  if (!H || height < 1) return S2S_ERR_INVALID;
  int r0, r1;
  band_out_rows(height, H->cfg.window, H->band_world, H->band_rank, &r0, &r1);
  if (row0) *row0 = r0;
  if (row1) *row1 = r1;
  return S2S_OK;
}

int s2s_band_partition(int window_rows, int world, int rank, int* w0, int* w1) {
  if (window_rows < 1 || world < 1 || world > window_rows || rank < 0 || rank >= world)
    return S2S_ERR_INVALID;
  band_partition(window_rows, world, rank, w0, w1);
  return S2S_OK;
}

int s2s_band_halo_ops(int rank, int world, int own_rows, int rows, int cyclic, int* ops, int cap) {
  if (world < 2 || rank < 0 || rank >= world || own_rows < rows || rows < 1 || rows > 8 || !ops ||
      cap < 16)
    return -1;
  HaloOp o[4];
  const int k = halo_ops(rank, world, 8, own_rows, rows, cyclic != 0, o);
  for (int i = 0; i < k; i++) {
    ops[4 * i] = o[i].kind;
    ops[4 * i + 1] = o[i].peer;
    ops[4 * i + 2] = o[i].row0;
    ops[4 * i + 3] = o[i].rows;
  }
  return k;
}

int s2s_forward_band(s2s_handle* H, int height, int width, const float* d_in, float* d_out,
                     void* stream) {
  if (!H || !d_in || !d_out) return S2S_ERR_INVALID;
  cudaStream_t st = stream ? (cudaStream_t)stream : H->stream;
  return guarded(H, [&] { run_forward(H, 1, height, width, d_in, d_out, nullptr, st); });
}

int s2s_forward_band_host(s2s_handle* H, int height, int width, const float* in, float* out) {
  if (!H || !in || !out) return S2S_ERR_INVALID;
  return guarded(H, [&] {
    const int s = H->cfg.scale;
    int r0, r1;
    band_out_rows(height, H->cfg.window, H->band_world, H->band_rank, &r0, &r1);
    const size_t nin = (size_t)3 * height * width;
    const size_t nout = (size_t)3 * (r1 - r0) * s * width * s;
    ensure_staging(H, &H->h_in, &H->h_in_n, nin);
    float* d_out = pinned_alias(out);  // pinned caller buffers are written directly
    if (!d_out) ensure_staging(H, &H->h_out, &H->h_out_n, std::max(nout, (size_t)1));
    ck(cudaMemcpyAsync(H->h_in, in, nin * 4, cudaMemcpyHostToDevice, H->stream), "upload");
    run_forward(H, 1, height, width, H->h_in, d_out ? d_out : H->h_out, nullptr, H->stream);
    if (nout && !d_out)
      ck(cudaMemcpyAsync(out, H->h_out, nout * 4, cudaMemcpyDeviceToHost, H->stream), "download");
    ck(cudaStreamSynchronize(H->stream), "forward");
    check_device_error(H);
    if (H->profiling) drain_profile(H);
  });
}

int s2s_selftest(const s2s_config* cfg, const s2s_tensor* tensors, int n_tensors, int device,
                 char* report, int cap) {
  if (!cfg || !tensors) return S2S_ERR_INVALID;
  std::string rep;
  bool all_ok = true;
  int status = S2S_OK;
  s2s_handle* hs[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  auto check = [&](const char* name, double err, double tol) {
    char b[192];
    const bool ok = err <= tol;
    snprintf(b, sizeof b, "%s %s max-abs %.3e (tolerance %.1e)\n", name, ok ? "ok" : "FAILED", err,
             tol);
    rep += b;
    if (!ok) all_ok = false;
  };
  // handle k with the given validation switches; false (and the error in the report)
  // when it cannot be made
  auto make = [&](int k, int unfused_mlp, int no_patch, int split = -1,
                  int mma_attn = -1, int unfused_proj = -1) -> bool {
    g_create_flags.unfused_proj = unfused_proj;
    g_create_flags.unfused_mlp = unfused_mlp;
    g_create_flags.no_patch = no_patch;
    g_create_flags.split = split;
    g_create_flags.mma_attn = mma_attn;
    const int rc = s2s_create(cfg, tensors, n_tensors, device, &hs[k]);
    g_create_flags = CreateFlags{};
    if (rc != S2S_OK) {
      rep += std::string("create failed: ") + s2s_last_error(nullptr) + "\n";
      status = rc;
      return false;
    }
    return true;
  };
  auto ran = [&](s2s_handle* h, int rc, const char* what) -> bool {
    if (rc == S2S_OK) return true;
    rep += std::string(what) + " failed: " + s2s_last_error(h) + "\n";
    status = rc;
    return false;
  };
  auto maxabs = [](const float* a, const float* b, size_t n) {
    double m = 0.0;
    for (size_t i = 0; i < n; i++) m = std::max(m, (double)std::fabs(a[i] - b[i]));
    return m;
  };
  // two mean-adjusted images of an odd size (not a window multiple), fixed seed
  const int win = cfg->window, sc = cfg->scale;
  const int h = 2 * win + 3, w = 3 * win + 5, B = 2;
  const size_t hw = (size_t)h * w, nin = 3 * hw, nout = (size_t)3 * h * sc * w * sc;
  std::vector<float> in(B * nin), batch(B * nout), eager(nout), other(nout), replay(nout);
  uint32_t st = 0x9E3779B9u;
  for (int b = 0; b < B; b++)
    for (int c = 0; c < 3; c++)
      for (size_t i = 0; i < hw; i++) {
        st = st * 1664525u + 1013904223u;
        const float v = (float)(st >> 8) * (1.0f / 16777216.0f);
        in[b * nin + c * hw + i] = (v - cfg->mean[c]) * cfg->img_range;
      }
  bool go = make(0, 0, 0);
  // one call over the batch, then each image alone: the first alone runs eagerly, the
  // second is captured as a graph, the third (image 0 again) replays it
  go = go && ran(hs[0], s2s_forward_batch(hs[0], B, h, w, in.data(), batch.data(), nullptr),
                 "batch forward");
  go = go && ran(hs[0], s2s_forward(hs[0], h, w, in.data(), eager.data(), nullptr), "forward");
  go = go && ran(hs[0], s2s_forward(hs[0], h, w, in.data() + nin, other.data(), nullptr),
                 "forward");
  go = go && ran(hs[0], s2s_forward(hs[0], h, w, in.data(), replay.data(), nullptr), "forward");
  if (go) {
    check("batch_vs_single", std::max(maxabs(batch.data(), eager.data(), nout),
                                      maxabs(batch.data() + nout, other.data(), nout)), 0.0);
    check("graph_replay_vs_eager", maxabs(replay.data(), eager.data(), nout), 0.0);
  }
  // the 64-channel head convs from tap boxes instead of kx patches
  go = go && make(1, 0, 1) &&
       ran(hs[1], s2s_forward(hs[1], h, w, in.data(), other.data(), nullptr), "forward");
  if (go) check("patches_vs_tap_boxes", maxabs(other.data(), eager.data(), nout), 1e-4);
  // the MLP as two GEMMs with the hidden activation in HBM
  go = go && make(2, 1, 0) &&
       ran(hs[2], s2s_forward(hs[2], h, w, in.data(), other.data(), nullptr), "forward");
  if (go) check("fused_vs_unfused_mlp", maxabs(other.data(), eager.data(), nout), 2e-3);
  // two-term operands against single-term ones (the other of the two for this width)
  go = go && make(3, 1, 0, hs[0]->split ? 0 : 1) &&
       ran(hs[3], s2s_forward(hs[3], h, w, in.data(), other.data(), nullptr), "forward");
  if (go) check("two_term_vs_single_term", maxabs(other.data(), eager.data(), nout), 2e-2);
  // the fused QKV + attention kernel against the QKV GEMM + mma.sync attention pair (the
  // other of the two for this handle)
  if (go && !hs[0]->split && hs[0]->Cp == 192 && hs[0]->heads == 6 && hs[0]->DP == 32) {
    go = make(4, 0, 0, -1, hs[0]->fused_attn ? 1 : 0) &&
         ran(hs[4], s2s_forward(hs[4], h, w, in.data(), other.data(), nullptr), "forward");
    if (go) check("fused_vs_unfused_attention", maxabs(other.data(), eager.data(), nout), 2e-3);
  }
  // proj inside the fused MLP kernel against the proj GEMM on its own: the same
  // operations in the same order
  if (go && hs[0]->fused_proj) {
    go = make(5, 0, 0, -1, -1, 1) &&
         ran(hs[5], s2s_forward(hs[5], h, w, in.data(), other.data(), nullptr), "forward");
    if (go) check("fused_vs_unfused_proj", maxabs(other.data(), eager.data(), nout), 1e-5);
  }
  for (s2s_handle*& x : hs)
    if (x) s2s_destroy(x);
  if (report && cap > 0) {
    const size_t n = std::min(rep.size(), (size_t)cap - 1);
    memcpy(report, rep.data(), n);
    report[n] = 0;
  }
  if (status != S2S_OK) return status;
  return all_ok ? S2S_OK : S2S_ERR_SELFTEST;
}

void s2s_destroy(s2s_handle* H) {
  if (!H) return;
  cudaSetDevice(H->device);
  cudaDeviceSynchronize();
  release_band(H);
  drain_profile(H);
  for (cudaEvent_t e : H->ev_pool) cudaEventDestroy(e);
  if (H->plan) free_plan(*H->plan);
  for (void* p : H->wallocs) cudaFree(p);
  if (H->h_in) cudaFree(H->h_in);
  if (H->h_out) cudaFree(H->h_out);
  if (H->h_aux) cudaFree(H->h_aux);
  if (H->b_in) cudaFree(H->b_in);
  if (H->b_out) cudaFree(H->b_out);
  if (H->side) cudaStreamDestroy(H->side);
  if (H->fork) cudaEventDestroy(H->fork);
  if (H->join) cudaEventDestroy(H->join);
  if (H->stream) cudaStreamDestroy(H->stream);
  delete H;
}

const char* s2s_version(void) { return "swin2sr-b200 0.1 (sm_100a)"; }

}  // extern "C"
