// Halo exchange by peer stores: one kernel per exchange on each rank of a row-band
// sharded forward (one GPU per rank). The neighbours' planes and mailboxes are CUDA
// IPC mappings of their device memory, reached over NVLink; nothing here reads a
// peer's memory except through plain loads of a mailbox word.
//
// Exchange e on rank R (the same e on every rank; has_prev / has_next: R has that
// neighbour in this exchange - always when cyclic, else not at the plane's edges):
//   1. block 0 tells each neighbour that R's halo rows it fills are free: every
//      kernel before this one (the readers of exchange e - 1) has completed;
//   2. every block waits for the neighbours' "free" words of exchange e, then writes
//      its share of R's last n owned rows into the next band's top halo and of R's
//      first n owned rows into the previous band's bottom halo, and raises its own
//      flag in each neighbour's mailbox (system-scope fence before the release);
//   3. every block waits for all kHaloBlocks flags of exchange e from each neighbour
//      it expects rows from, so the kernel completes only once R's halo is filled;
//      without a neighbour (non-cyclic edges) the halo rows are zeroed when asked;
//   4. the last block to finish records e as R's completed exchange.
// Every wait is bounded (DEV_TIMEOUT_HALO after ~10 s in a forward, or at once when
// another wait of the library already gave up); the host then fails the forward.
#include "common.cuh"
#include "halo.cuh"

namespace s2s {
namespace {

struct HaloPushArgs {
  const uint4* src;        // this rank's plane (16-byte units)
  uint4* next_dst;         // the next band's plane (peer mapping), null: no next
  uint4* prev_dst;         // the previous band's plane, null: no previous
  HaloMailbox* mine;       // this rank's mailbox (local)
  HaloMailbox* next_mb;    // the neighbours' mailboxes (peer mappings)
  HaloMailbox* prev_mb;
  uint64_t row_u4;         // 16-byte units per plane row
  int n;                   // rows moved each way
  int halo, own_rows;      // this rank's plane: owned rows [halo, halo + own_rows)
  int next_halo;           // the next band's top halo ends at its row next_halo
  int prev_end;            // the previous band's bottom halo starts at its row prev_end
  int zero_top, zero_bottom;  // no neighbour on that side: zero this rank's halo rows
  uint64_t limit_ns;          // how long each wait may last
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *p has reached epoch e (wrap-safe), for at most limit_ns of wall time.
__device__ bool wait_epoch(const unsigned* p, unsigned e, uint64_t limit_ns) {
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if ((int)(ld_acquire_sys(p) - e) >= 0) return true;
    if ((it & 63u) == 63u) {
      if (global_timer_ns() - t0 > limit_ns) {
        record_error(DEV_TIMEOUT_HALO);
        return false;
      }
      if (*(volatile unsigned*)&g_s2s_err != 0u) return false;
      __nanosleep(200);
    }
  }
}

__global__ void __launch_bounds__(128) k_halo_push(const HaloPushArgs a) {
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const unsigned e = *(volatile unsigned*)&a.mine->seq + 1u;
    s_epoch = e;
    if (blockIdx.x == 0) {
      // this rank's halo rows are free for exchange e
      if (a.prev_mb) st_release_sys(&a.prev_mb->may_push_next, e);
      if (a.next_mb) st_release_sys(&a.next_mb->may_push_prev, e);
    }
    bool ok = true;
    if (a.next_dst) ok = wait_epoch(&a.mine->may_push_next, e, a.limit_ns);
    if (ok && a.prev_dst) ok = wait_epoch(&a.mine->may_push_prev, e, a.limit_ns);
    s_ok = ok;
  }
  __syncthreads();
  const unsigned e = s_epoch;
  if (s_ok) {
    const uint64_t cnt = (uint64_t)a.n * a.row_u4;
    const uint4* last = a.src + (uint64_t)(a.halo + a.own_rows - a.n) * a.row_u4;
    const uint4* first = a.src + (uint64_t)a.halo * a.row_u4;
    uint4* dn = a.next_dst ? a.next_dst + (uint64_t)(a.next_halo - a.n) * a.row_u4 : nullptr;
    uint4* dp = a.prev_dst ? a.prev_dst + (uint64_t)a.prev_end * a.row_u4 : nullptr;
    uint4* zt = a.zero_top ? const_cast<uint4*>(first) - cnt : nullptr;
    uint4* zb = a.zero_bottom ? const_cast<uint4*>(last) + cnt : nullptr;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < cnt;
         k += (uint64_t)gridDim.x * blockDim.x) {
      if (dn) dn[k] = last[k];
      if (dp) dp[k] = first[k];
      if (zt) zt[k] = z;
      if (zb) zb[k] = z;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      if (a.next_mb && a.next_dst) st_release_sys(&a.next_mb->top_in[blockIdx.x], e);
      if (a.prev_mb && a.prev_dst) st_release_sys(&a.prev_mb->bottom_in[blockIdx.x], e);
    }
    // this rank's halo: the top rows from the previous band, the bottom from the next
    if (threadIdx.x < kHaloBlocks) {
      bool ok = true;
      if (a.prev_dst) ok = wait_epoch(&a.mine->top_in[threadIdx.x], e, a.limit_ns);
      if (ok && a.next_dst) wait_epoch(&a.mine->bottom_in[threadIdx.x], e, a.limit_ns);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.mine->arrive, 1u) == gridDim.x - 1) {
      // every block has read seq: exchange e is this rank's last completed one
      a.mine->arrive = 0u;
      *(volatile unsigned*)&a.mine->seq = e;
      __threadfence();
    }
  }
}

}  // namespace

// One exchange of `n` rows of the plane `buf` (row_bytes per row) with the
// neighbours `prev` / `next` (their copy of the same plane: prev_buf / next_buf;
// null when this rank has no such neighbour in this exchange). `cooperative`: the
// blocks are launched together (the loopback diagnostic, where they wait on each
// other's flags).
cudaError_t launch_halo_push(const void* buf, void* prev_buf, void* next_buf, HaloMailbox* mine,
                             const HaloPeer* prev, const HaloPeer* next, size_t row_bytes, int n,
                             int halo, int own_rows, bool zero_top, bool zero_bottom,
                             cudaStream_t st, uint64_t limit_ns, bool cooperative) {
  if (row_bytes % 16 != 0 || n < 1 || n > halo || n > own_rows)
    return cudaErrorInvalidValue;
  HaloPushArgs a;
  a.src = static_cast<const uint4*>(buf);
  a.next_dst = static_cast<uint4*>(next_buf);
  a.prev_dst = static_cast<uint4*>(prev_buf);
  a.mine = mine;
  a.next_mb = next_buf ? next->mb : nullptr;
  a.prev_mb = prev_buf ? prev->mb : nullptr;
  a.row_u4 = row_bytes / 16;
  a.n = n;
  a.halo = halo;
  a.own_rows = own_rows;
  a.next_halo = next_buf ? next->halo : 0;
  a.prev_end = prev_buf ? prev->halo + prev->own_rows : 0;
  a.zero_top = zero_top && !prev_buf;
  a.zero_bottom = zero_bottom && !next_buf;
  a.limit_ns = limit_ns;
  if (cooperative) {
    void* args[] = {&a};
    return cudaLaunchCooperativeKernel((const void*)k_halo_push, dim3(kHaloBlocks), dim3(128), args,
                                       0, st);
  }
  k_halo_push<<<kHaloBlocks, 128, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace s2s
