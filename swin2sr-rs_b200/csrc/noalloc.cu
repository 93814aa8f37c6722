// Window attention of one block over caller-owned device buffers, allocating nothing.
//
// The attention kernel reads token rows through a window -> image row table. A
// forward keeps that table in its plan workspace (device memory the handle
// allocates); this entry point keeps it instead in one fixed device array of the
// library, `g_noalloc_rows`, so a caller that owns every buffer and forbids
// allocation can still run the kernel. The table is rebuilt on the device at every
// call, on the caller's stream, before the attention reads it: nothing in the
// scratch has to start at zero, and calls that overlap on one device (two streams,
// two threads) race on it.
#include <mutex>

namespace s2s {
namespace {

constexpr int kNoAllocMaxDevices = 64;

// batch * hp * wp window-major tokens -> image rows, int32 (4 MiB).
static __device__ __align__(256) int g_noalloc_rows[S2S_NOALLOC_MAX_TOKENS];

std::mutex g_noalloc_mu;
int* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Set-up, once per device, with that device current: the array's device address.
int* noalloc_rows(int device) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (device < 0 || device >= kNoAllocMaxDevices)
    fail(S2S_ERR_INVALID, "s2s_window_attention_noalloc: device ordinal out of range");
  if (!g_noalloc_ptr[device]) {
    int* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_rows);
    if (e != cudaSuccess || !ptr)
      fail(S2S_ERR_CUDA, std::string("s2s_window_attention_noalloc: cudaGetSymbolAddress of the "
                                     "row scratch failed: ") + cudaGetErrorString(e));
    g_noalloc_ptr[device] = ptr;
  }
  return g_noalloc_ptr[device];
}

// The row table the plan builds on the host (window-major token r of image b ->
// image row b*hp*wp + y*wp + x, the window grid shifted by `shift`), made on the device.
__global__ void k_window_rows(int* __restrict__ rows, int B, int hp, int wp, int shift) {
  const int hw = hp * wp, nww = wp / 8;
  const int n = B * hw;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int b = i / hw, r = i - b * hw;
    const int wi = r >> 6, t = r & 63;
    const int y = ((wi / nww) * 8 + (t >> 3) + shift) % hp;
    const int x = ((wi % nww) * 8 + (t & 7) + shift) % wp;
    rows[i] = b * hw + y * wp + x;
  }
}

}  // namespace
}  // namespace s2s

extern "C" int s2s_window_attention_noalloc(s2s_handle* H, int stage, int block, int batch,
                                            int hp, int wp, const void* d_qkv, void* d_out,
                                            int ld_out, void* stream) {
  using namespace s2s;
  if (!H) return S2S_ERR_INVALID;
  cudaStream_t st = stream ? (cudaStream_t)stream : H->stream;
  return guarded(H, [&] {
    const s2s_config& c = H->cfg;
    if (stage < 0 || stage >= c.n_depths || block < 0 || block >= c.depths[stage])
      fail(S2S_ERR_INVALID, "s2s_window_attention_noalloc: no such stage/block");
    if (batch < 1 || hp < c.window || wp < c.window || hp % c.window || wp % c.window)
      fail(S2S_ERR_INVALID, "s2s_window_attention_noalloc: the plane must be a positive "
                            "multiple of the window in both directions");
    const long long tokens = (long long)batch * hp * wp;
    if (tokens > S2S_NOALLOC_MAX_TOKENS)
      fail(S2S_ERR_INVALID, "s2s_window_attention_noalloc: batch*hp*wp = " +
                                std::to_string(tokens) + " tokens is more than the fixed row "
                                "scratch holds (S2S_NOALLOC_MAX_TOKENS = " +
                                std::to_string((long long)S2S_NOALLOC_MAX_TOKENS) + ")");
    if (!d_qkv || !d_out || ((uintptr_t)d_qkv & 15) || ((uintptr_t)d_out & 3))
      fail(S2S_ERR_INVALID, "s2s_window_attention_noalloc: qkv must be 16-byte and out "
                            "4-byte aligned device pointers");
    if (ld_out < H->C || ld_out % 2)
      fail(S2S_ERR_INVALID, "s2s_window_attention_noalloc: ld_out must be even and >= embed");
    ck(cudaSetDevice(H->device), "cudaSetDevice");
    int* rows = noalloc_rows(H->device);
    const int shift = (block % 2 == 1) ? c.window / 2 : 0;
    const int n = (int)tokens;
    k_window_rows<<<(unsigned)std::min((n + 255) / 256, 148 * 16), 256, 0, st>>>(rows, batch, hp,
                                                                                 wp, shift);
    ck(cudaGetLastError(), "window_rows");
    const Block& bl = H->stages[stage].blocks[block];
    ck(launch_window_attention((const __half*)d_qkv, (__half*)d_out, bl.cpb, rows,
                               batch * (hp / 8) * (wp / 8), H->heads, H->hd, H->DP, ld_out, H->NQ,
                               0, 0, 0, hp / 8, wp / 8, hp, wp, shift, 0, st),
       "window_attention");
    H->launches.fetch_add(2, std::memory_order_relaxed);
  });
}
