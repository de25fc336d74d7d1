// Device runtime of the `cuda` backend: the storage allocator, streams, events, CUDA-graph
// capture and the NCCL communicator, all behind the C ABI (include/mtorch_cuda.h), so that a host
// layer needs nothing but this library to own device memory and order work.
//
// The reference keeps a tensor's bytes in a host `Storage` (cpp/mtorch/core/tensor.h:60-63, a
// `std::vector<uint8_t>` behind a shared pointer); the device counterpart here is a caching
// allocator of device blocks:
//
// * one free list per (device, pool), best fit by size; blocks come from cudaMalloc in 512-byte
//   (small) or 2 MiB (large) granules and are never split, so freeing is O(log n) and a block
//   keeps its size for life;
// * blocks are reused in stream order: the host layer issues every kernel and copy of a device on
//   one stream (the library stream below), so a freed block's last use is ordered before any
//   later use of the same block without events;
// * pool 0 is the default pool; a CUDA-graph capture opens a private pool that serves every
//   allocation made during the capture and keeps its blocks for as long as the graph exists, so
//   the graph's intermediate buffers are never handed to work outside the graph (and a block
//   freed during the capture is reused only by later captured work, which replays in the same
//   order);
// * when cudaMalloc reports out of memory, the cached free blocks of the device are released
//   (cudaFree, after a device synchronisation) and the allocation is retried once.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2): the library links no communication
// library, and a process that never builds a communicator never loads one.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "runtime.h"

namespace mt {
namespace {

constexpr size_t kSmallLimit = 1 << 20;     // requests below 1 MiB round to 512 B
constexpr size_t kSmallGranule = 512;
constexpr size_t kLargeGranule = 2 << 20;   // larger requests round to 2 MiB
constexpr int kMaxDevices = 64;

struct Pool {
  std::multimap<size_t, void*> free_blocks;  // size -> block
  int live = 0;                              // blocks of this pool currently handed out
  bool released = false;                     // the owning graph is gone: free blocks on return
};

struct Block {
  size_t size;
  int device;
  int pool;
};

struct DeviceState {
  std::vector<Pool> pools{Pool{}};  // pool 0 = default
  int active_pool = 0;              // pool serving allocations on this device
  size_t in_use = 0, cached = 0;    // bytes handed out / bytes held in free lists
  void* stream = nullptr;           // library stream (created on first request)
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
std::unordered_map<void*, Block> g_live;

size_t round_size(size_t n) {
  if (n == 0) n = 1;
  return n < kSmallLimit ? align_up(n, kSmallGranule) : align_up(n, kLargeGranule);
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return (d >= 0 && d < kMaxDevices) ? d : 0;
}

// cudaMalloc in relaxed capture mode: a capture in progress on this thread does not forbid it.
cudaError_t raw_malloc(void** p, size_t bytes) {
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  cudaError_t e = cudaMalloc(p, bytes);
  cudaThreadExchangeStreamCaptureMode(&mode);
  return e;
}

// Releases every cached (free) block of `dev` in pools that no capture is using; g_mu held.
void release_cached(int dev) {
  DeviceState& s = g_dev[dev];
  cudaDeviceSynchronize();
  for (size_t p = 0; p < s.pools.size(); ++p) {
    if ((int)p == s.active_pool && p != 0) continue;
    for (auto& kv : s.pools[p].free_blocks) {
      cudaFree(kv.second);
      s.cached -= kv.first;
    }
    s.pools[p].free_blocks.clear();
  }
}

}  // namespace
}  // namespace mt

using namespace mt;

static cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- storage allocator -------------------------------------------------------------------

extern "C" int mt_cuda_malloc(void** out, size_t bytes) {
  if (!out) return fail(MT_ERR_INVALID, "mt_cuda_malloc: null output pointer");
  *out = nullptr;
  const size_t size = round_size(bytes);
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& s = g_dev[dev];
  Pool& pool = s.pools[s.active_pool];
  // best fit, accepting a cached block up to 1/8 (large) or 2x (small) bigger than asked for
  auto it = pool.free_blocks.lower_bound(size);
  const size_t slack = size < kSmallLimit ? size : size / 8;
  if (it != pool.free_blocks.end() && it->first <= size + slack) {
    void* p = it->second;
    const size_t bsize = it->first;
    pool.free_blocks.erase(it);
    s.cached -= bsize;
    s.in_use += bsize;
    pool.live++;
    g_live[p] = Block{bsize, dev, s.active_pool};
    *out = p;
    return MT_OK;
  }
  void* p = nullptr;
  cudaError_t e = raw_malloc(&p, size);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    release_cached(dev);
    e = raw_malloc(&p, size);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MT_ERR_LAUNCH, "mt_cuda_malloc(%zu bytes) on device %d: %s (in use %zu, cached %zu)", bytes, dev,
                cudaGetErrorString(e), s.in_use, s.cached);
  }
  s.in_use += size;
  s.pools[s.active_pool].live++;
  g_live[p] = Block{size, dev, s.active_pool};
  *out = p;
  return MT_OK;
}

extern "C" int mt_cuda_free(void* p) {
  if (!p) return MT_OK;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_live.find(p);
  if (it == g_live.end()) return fail(MT_ERR_INVALID, "mt_cuda_free: %p was not allocated by mt_cuda_malloc", p);
  const Block b = it->second;
  g_live.erase(it);
  DeviceState& s = g_dev[b.device];
  Pool& pool = s.pools[b.pool];
  s.in_use -= b.size;
  pool.live--;
  if (pool.released) {  // its graph is gone: nothing can reuse the block any more
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(b.device);
    cudaFree(p);
    cudaSetDevice(prev);
    return MT_OK;
  }
  pool.free_blocks.emplace(b.size, p);
  s.cached += b.size;
  return MT_OK;
}

extern "C" int mt_cuda_memory_stats(int device, size_t* in_use, size_t* cached) {
  if (device < 0 || device >= kMaxDevices) return fail(MT_ERR_INVALID, "bad device %d", device);
  std::lock_guard<std::mutex> lock(g_mu);
  if (in_use) *in_use = g_dev[device].in_use;
  if (cached) *cached = g_dev[device].cached;
  return MT_OK;
}

extern "C" int mt_cuda_empty_cache(void) {
  std::lock_guard<std::mutex> lock(g_mu);
  release_cached(current_device());
  return cuda_check(cudaGetLastError(), "empty_cache");
}

// ---- pinned host memory (staging buffers for host<->device copies) ------------------------

extern "C" int mt_cuda_host_alloc(void** out, size_t bytes) {
  if (!out) return fail(MT_ERR_INVALID, "mt_cuda_host_alloc: null output pointer");
  return cuda_check(cudaMallocHost(out, bytes ? bytes : 1), "cudaMallocHost");
}

extern "C" int mt_cuda_host_free(void* p) { return p ? cuda_check(cudaFreeHost(p), "cudaFreeHost") : MT_OK; }

// ---- streams and events --------------------------------------------------------------------

extern "C" int mt_cuda_stream_create(void** out) {
  if (!out) return fail(MT_ERR_INVALID, "mt_cuda_stream_create: null output pointer");
  cudaStream_t s = nullptr;
  int rc = cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  *out = s;
  return rc;
}

extern "C" int mt_cuda_stream_destroy(void* s) { return s ? cuda_check(cudaStreamDestroy(S(s)), "cudaStreamDestroy") : MT_OK; }

extern "C" int mt_cuda_library_stream(int device, void** out) {
  if (!out || device < 0 || device >= kMaxDevices) return fail(MT_ERR_INVALID, "mt_cuda_library_stream: bad arguments");
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& s = g_dev[device];
  if (!s.stream) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaStream_t st = nullptr;
    int rc = cuda_check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
    cudaSetDevice(prev);
    if (rc) return rc;
    s.stream = st;
  }
  *out = s.stream;
  return MT_OK;
}

extern "C" int mt_cuda_event_create(void** out) {
  if (!out) return fail(MT_ERR_INVALID, "mt_cuda_event_create: null output pointer");
  cudaEvent_t e = nullptr;
  int rc = cuda_check(cudaEventCreate(&e), "cudaEventCreate");
  *out = e;
  return rc;
}

extern "C" int mt_cuda_event_destroy(void* e) {
  return e ? cuda_check(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(e)), "cudaEventDestroy") : MT_OK;
}

extern "C" int mt_cuda_event_record(void* e, void* stream) {
  return cuda_check(cudaEventRecord(reinterpret_cast<cudaEvent_t>(e), S(stream)), "cudaEventRecord");
}

extern "C" int mt_cuda_event_synchronize(void* e) {
  return cuda_check(cudaEventSynchronize(reinterpret_cast<cudaEvent_t>(e)), "cudaEventSynchronize");
}

extern "C" int mt_cuda_event_elapsed_ms(void* start, void* end, float* ms) {
  if (!ms) return fail(MT_ERR_INVALID, "mt_cuda_event_elapsed_ms: null output pointer");
  return cuda_check(cudaEventElapsedTime(ms, reinterpret_cast<cudaEvent_t>(start), reinterpret_cast<cudaEvent_t>(end)),
                    "cudaEventElapsedTime");
}

// ---- CUDA graphs ---------------------------------------------------------------------------

namespace {
struct Graph {
  cudaGraphExec_t exec = nullptr;
  int device = 0;
  int pool = 0;
};
}  // namespace

extern "C" int mt_cuda_graph_begin(void* stream) {
  if (!stream) return fail(MT_ERR_INVALID, "mt_cuda_graph_begin: capture needs a created stream, not the legacy one");
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceState& s = g_dev[dev];
    if (s.active_pool != 0) return fail(MT_ERR_INVALID, "mt_cuda_graph_begin: a capture is already open on device %d", dev);
    s.pools.push_back(Pool{});
    s.active_pool = (int)s.pools.size() - 1;
  }
  int rc = cuda_check(cudaStreamBeginCapture(S(stream), cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  if (rc) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_dev[dev].active_pool = 0;
  }
  return rc;
}

extern "C" int mt_cuda_graph_end(void* stream, void** out) {
  if (!out) return fail(MT_ERR_INVALID, "mt_cuda_graph_end: null output pointer");
  *out = nullptr;
  const int dev = current_device();
  int pool = 0;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    pool = g_dev[dev].active_pool;
    g_dev[dev].active_pool = 0;
  }
  cudaGraph_t graph = nullptr;
  int rc = cuda_check(cudaStreamEndCapture(S(stream), &graph), "cudaStreamEndCapture");
  if (rc) return rc;
  cudaGraphExec_t exec = nullptr;
  rc = cuda_check(cudaGraphInstantiate(&exec, graph, 0), "cudaGraphInstantiate");
  cudaGraphDestroy(graph);
  if (rc) return rc;
  *out = new Graph{exec, dev, pool};
  return MT_OK;
}

extern "C" int mt_cuda_graph_launch(void* g, void* stream) {
  if (!g) return fail(MT_ERR_INVALID, "mt_cuda_graph_launch: null graph");
  return cuda_check(cudaGraphLaunch(static_cast<Graph*>(g)->exec, S(stream)), "cudaGraphLaunch");
}

extern "C" int mt_cuda_graph_destroy(void* g) {
  if (!g) return MT_OK;
  Graph* gr = static_cast<Graph*>(g);
  int rc = cuda_check(cudaGraphExecDestroy(gr->exec), "cudaGraphExecDestroy");
  {
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceState& s = g_dev[gr->device];
    if (gr->pool > 0 && gr->pool < (int)s.pools.size()) {
      Pool& p = s.pools[gr->pool];
      cudaDeviceSynchronize();  // a replay may still be running
      for (auto& kv : p.free_blocks) {
        cudaFree(kv.second);
        s.cached -= kv.first;
      }
      p.free_blocks.clear();
      p.released = true;  // live blocks (e.g. the graph's outputs) are freed when returned
    }
  }
  delete gr;
  return rc;
}

// ---- NCCL (loaded at run time) ---------------------------------------------------------------

namespace {
struct Nccl {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
  std::string why;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      n.why = e ? e : "dlopen(libnccl.so.2) failed";
      return;
    }
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.init_rank = reinterpret_cast<decltype(n.init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "ncclCommDestroy"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.init_rank && n.all_gather && n.destroy && n.error_string;
    if (!n.ok) n.why = "libnccl.so.2 lacks a required symbol";
  });
  return n;
}

int nccl_check(const Nccl& n, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return MT_OK;
  return fail(MT_ERR_LAUNCH, "%s: %s", what, n.error_string(r));
}
}  // namespace

extern "C" int mt_nccl_available(void) { return nccl().ok ? 1 : 0; }

extern "C" int mt_nccl_unique_id(void* out, size_t bytes) {
  const Nccl& n = nccl();
  if (!n.ok) return fail(MT_ERR_UNSUPPORTED, "NCCL unavailable: %s", n.why.c_str());
  if (!out || bytes < sizeof(ncclUniqueId)) return fail(MT_ERR_INVALID, "mt_nccl_unique_id: buffer below %zu bytes", sizeof(ncclUniqueId));
  ncclUniqueId id;
  int rc = nccl_check(n, n.get_unique_id(&id), "ncclGetUniqueId");
  if (!rc) std::memcpy(out, &id, sizeof(id));
  return rc;
}

extern "C" int mt_nccl_comm_init(void** comm, const void* unique_id, size_t bytes, int world, int rank) {
  const Nccl& n = nccl();
  if (!n.ok) return fail(MT_ERR_UNSUPPORTED, "NCCL unavailable: %s", n.why.c_str());
  if (!comm || !unique_id || bytes != sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
    return fail(MT_ERR_INVALID, "mt_nccl_comm_init: bad arguments (rank %d of %d)", rank, world);
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclComm_t c = nullptr;
  int rc = nccl_check(n, n.init_rank(&c, world, id, rank), "ncclCommInitRank");
  *comm = rc ? nullptr : c;
  return rc;
}

extern "C" int mt_nccl_all_gather(const void* send, void* recv, size_t bytes_per_rank, void* comm, void* stream) {
  const Nccl& n = nccl();
  if (!n.ok) return fail(MT_ERR_UNSUPPORTED, "NCCL unavailable: %s", n.why.c_str());
  if (!comm || (!send && bytes_per_rank) || (!recv && bytes_per_rank)) return fail(MT_ERR_INVALID, "mt_nccl_all_gather: bad arguments");
  return nccl_check(n, n.all_gather(send, recv, bytes_per_rank, ncclUint8, static_cast<ncclComm_t>(comm), S(stream)),
                    "ncclAllGather");
}

extern "C" int mt_nccl_comm_destroy(void* comm) {
  if (!comm) return MT_OK;
  const Nccl& n = nccl();
  if (!n.ok) return fail(MT_ERR_UNSUPPORTED, "NCCL unavailable: %s", n.why.c_str());
  return nccl_check(n, n.destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}
