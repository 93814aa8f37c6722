// Halo exchange of the row-band sharded forward.
//
// A single image is split into window-aligned row bands, one per rank. Before a
// shifted block a rank needs the 4 rows either side of its band (cyclically: the
// first and last bands are neighbours through the roll's wrap), before a 3x3
// convolution 1 row (zeros beyond the plane's true edges), before the upsampling
// head 4 rows. Three transports move them:
//   * peer stores (ranks are processes, one GPU each; the default): each rank maps
//     its neighbours' planes and mailboxes through CUDA IPC and one kernel per
//     exchange writes its boundary rows straight into their halo rows over NVLink,
//     with flags in the mailboxes ordering the writes (k_halo_push);
//   * NCCL point-to-point (S2S_HALO=nccl). libnccl.so.2 is resolved at run time -
//     the copy the process already loaded (PyTorch's) when there is one - so
//     libs2s.so has no link-time dependency on it. NCCL also carries the IPC
//     handles to the neighbours when a band plan is built;
//   * an in-process group of handles, one host thread each (tests on one GPU, and
//     embedders that drive several GPUs from one process): device-to-device copies
//     ordered by CUDA events, with a host barrier on either side.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <mutex>
#include <string>
#include <vector>

namespace s2s {

// One transfer of an exchange: a send (kind 0) or receive (kind 1) of `rows` plane
// rows starting at local row `row0`, to / from rank `peer`.
struct HaloOp {
  int kind, peer, row0, rows;
};

// The transfers of one exchange of `n` rows, in issue order. Owned rows are local
// [halo, halo + own_rows). Sends go to `next` before `prev` and receives come from
// `prev` before `next`, so with two ranks (prev == next) the two messages each way
// pair up in order: my last rows -> the peer's top halo, my first rows -> its
// bottom halo. Without `cyclic` the plane's first rank has no top neighbour and its
// last rank no bottom neighbour.
inline int halo_ops(int rank, int world, int halo, int own_rows, int n, bool cyclic,
                    HaloOp* ops) {
  const int prev = (rank + world - 1) % world, next = (rank + 1) % world;
  const bool first = rank == 0, last = rank == world - 1;
  int k = 0;
  if (cyclic || !last) ops[k++] = {0, next, halo + own_rows - n, n};
  if (cyclic || !first) ops[k++] = {0, prev, halo, n};
  if (cyclic || !first) ops[k++] = {1, prev, halo - n, n};
  if (cyclic || !last) ops[k++] = {1, next, halo + own_rows, n};
  return k;
}

// Window rows of the padded plane split as evenly as possible, the first ranks
// taking one more when they do not divide: rank's window rows [*w0, *w1).
inline void band_partition(int window_rows, int world, int rank, int* w0, int* w1) {
  const int base = window_rows / world, extra = window_rows % world;
  *w0 = rank * base + (rank < extra ? rank : extra);
  *w1 = *w0 + base + (rank < extra ? 1 : 0);
}

// ------------------------------------------------------------------ peer-store mailboxes
// Blocks of k_halo_push (each signals its share of the rows by its own flag).
constexpr int kHaloBlocks = 32;

// One per rank and band plan, in the rank's device memory, mapped by both
// neighbours. Words are exchange epochs (1, 2, ... per plan, the same on every rank:
// all ranks run the same exchanges in the same order) written by the neighbours:
//   may_push_next  my next band's top halo rows are free for exchange e (its readers
//                  of exchange e - 1 have finished)
//   may_push_prev  my previous band's bottom halo rows are free
//   top_in[b]      block b of my previous band has written its share of my top halo
//   bottom_in[b]   block b of my next band has written its share of my bottom halo
// and two local words: seq, the last exchange this rank completed, and arrive, the
// blocks of the running exchange that have finished.
struct HaloMailbox {
  unsigned may_push_next, may_push_prev;
  unsigned top_in[kHaloBlocks], bottom_in[kHaloBlocks];
  unsigned seq, arrive;
};

// What a rank needs of a neighbour's band plan: its planes, mailbox and layout.
struct HaloPeer {
  void* x16 = nullptr;
  void* ao = nullptr;
  HaloMailbox* mb = nullptr;
  int halo = 0, own_rows = 0;
};

// ------------------------------------------------------------------ NCCL, resolved at run time
struct NcclApi {
  bool ok = false;
  std::string err;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) =
      nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

inline const NcclApi& nccl_api() {
  static NcclApi api = [] {
    NcclApi a;
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) {
      const char* e = dlerror();
      a.err = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "?");
      return a;
    }
    bool ok = true;
    auto sym = [&](const char* name) {
      void* p = dlsym(lib, name);
      if (!p) ok = false;
      return p;
    };
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
    a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(sym("ncclCommInitRank"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
    a.Send = reinterpret_cast<decltype(a.Send)>(sym("ncclSend"));
    a.Recv = reinterpret_cast<decltype(a.Recv)>(sym("ncclRecv"));
    a.GroupStart = reinterpret_cast<decltype(a.GroupStart)>(sym("ncclGroupStart"));
    a.GroupEnd = reinterpret_cast<decltype(a.GroupEnd)>(sym("ncclGroupEnd"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
    a.ok = ok;
    if (!ok) a.err = "libnccl.so.2 lacks a point-to-point entry point";
    return a;
  }();
  return api;
}

// ------------------------------------------------------------------ in-process group
struct LocalGroup {
  int world = 0;
  std::mutex mu;
  std::condition_variable cv;
  int arrived = 0;
  long long gen = 0;
  bool broken = false;
  // per rank, published before the first barrier of an exchange
  std::vector<const char*> buf;
  std::vector<int> halo, own_rows;
  std::vector<cudaEvent_t> ready, done;  // created on each rank's device
  std::vector<int> device;

  // All ranks arrive or none passes: false when the wait ran out (the group is then
  // marked broken, so every rank's later exchanges fail at once).
  bool barrier(double seconds) {
    std::unique_lock<std::mutex> lk(mu);
    if (broken) return false;
    const long long g = gen;
    if (++arrived == world) {
      arrived = 0;
      gen++;
      cv.notify_all();
      return true;
    }
    const bool ok = cv.wait_for(lk, std::chrono::duration<double>(seconds),
                                [&] { return gen != g || broken; });
    if (!ok || broken) {
      broken = true;
      cv.notify_all();
      return false;
    }
    return true;
  }
  ~LocalGroup() {
    for (size_t r = 0; r < ready.size(); r++) {
      cudaSetDevice(device[r]);
      if (ready[r]) cudaEventDestroy(ready[r]);
      if (done[r]) cudaEventDestroy(done[r]);
    }
  }
};

}  // namespace s2s
