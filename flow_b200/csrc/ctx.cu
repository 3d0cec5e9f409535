// ctx.cu — context lifecycle, machine profile, trap protocol, NCCL binding.
//
// The context replaces the emitted prelude's process globals
// (crates/backends/cuda/src/module.rs:61-95): the device trap flag, its
// initialisation (trap_init, :74-77) and the launch-then-read-flag check
// (trap_check_after_launch, :86-94). Instead of exiting (101 / 102) the
// library returns the status to its caller, which owns the process.
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include <climits>

#include "common.cuh"

// ---- errors -------------------------------------------------------------------

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  std::string m = std::string("CUDA error at ") + what + ": " + cudaGetErrorString(e);
  return set_error(e == cudaErrorMemoryAllocation ? MAPAL_ERR_NOMEM : MAPAL_ERR_CUDA, m);
}

extern "C" const char* mapal_gpu_last_error(void) { return g_last_error.c_str(); }
extern "C" int mapal_gpu_abi_version(void) { return MAPAL_GPU_ABI_VERSION; }

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
extern "C" uint64_t mapal_gpu_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

// ---- NCCL -----------------------------------------------------------------------

static NcclApi g_nccl;
static std::once_flag g_nccl_once;

NcclApi* nccl_api() {
  std::call_once(g_nccl_once, [] {
    // An NCCL already loaded in the process (for example by torch) is reused:
    // dlopen of the same soname returns that library.
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    void* h = nullptr;
    for (const char* n : names)
      if ((h = dlopen(n, RTLD_NOW | RTLD_GLOBAL)) != nullptr) break;
    if (!h) {
      g_nccl.error = std::string("libnccl.so.2 not loadable: ") + dlerror();
      return;
    }
    bool ok = true;
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (!p) ok = false;
      return p;
    };
    g_nccl.GetUniqueId = (int (*)(NcclId*))sym("ncclGetUniqueId");
    g_nccl.CommInitRank = (int (*)(ncclComm_t*, int, NcclId, int))sym("ncclCommInitRank");
    g_nccl.CommInitAll = (int (*)(ncclComm_t*, int, const int*))sym("ncclCommInitAll");
    g_nccl.CommDestroy = (int (*)(ncclComm_t))sym("ncclCommDestroy");
    g_nccl.AllReduce = (int (*)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t))sym(
        "ncclAllReduce");
    g_nccl.Broadcast = (int (*)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t))sym(
        "ncclBroadcast");
    g_nccl.GroupStart = (int (*)())sym("ncclGroupStart");
    g_nccl.GroupEnd = (int (*)())sym("ncclGroupEnd");
    g_nccl.GetErrorString = (const char* (*)(int))sym("ncclGetErrorString");
    g_nccl.AllGather = (int (*)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t))sym("ncclAllGather");
    if (!ok) {
      g_nccl.error = "libnccl.so.2 lacks a required symbol";
      return;
    }
    g_nccl.CommInitRankConfig = (int (*)(ncclComm_t*, int, NcclId, int, void*))dlsym(h, "ncclCommInitRankConfig");
    g_nccl.loaded = true;
  });
  return &g_nccl;
}

static int nccl_fail(int rc, const char* what) {
  NcclApi* n = nccl_api();
  std::string m = std::string("NCCL error at ") + what + ": " +
                  (n->GetErrorString ? n->GetErrorString(rc) : "?");
  return set_error(MAPAL_ERR_NCCL, m);
}

// ---- profile ----------------------------------------------------------------------

static int read_profile(int device, MapalGpuProfile* p) {
  cudaDeviceProp prop;
  MAPAL_CUDA(cudaGetDeviceProperties(&prop, device));
  memset(p, 0, sizeof *p);
  p->device = device;
  p->cc_major = prop.major;
  p->cc_minor = prop.minor;
  p->sm_count = prop.multiProcessorCount;
  p->warp_size = prop.warpSize;
  p->max_threads_per_block = prop.maxThreadsPerBlock;
  p->max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
  p->regs_per_sm = prop.regsPerMultiprocessor;
  p->smem_per_sm = (int64_t)prop.sharedMemPerMultiprocessor;
  p->smem_per_block_optin = (int64_t)prop.sharedMemPerBlockOptin;
  p->l2_bytes = prop.l2CacheSize;
  // Tensor memory is architectural on sm_100: 128 lanes x 512 columns x 32 bit.
  p->tmem_bytes_per_sm = prop.major == 10 ? 128 * 512 * 4 : 0;
  p->hbm_bytes = (int64_t)prop.totalGlobalMem;
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrClockRate, device);
  p->sm_clock_khz = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrMemoryClockRate, device);
  p->mem_clock_khz = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrGlobalMemoryBusWidth, device);
  p->mem_bus_bits = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrClusterLaunch, device);
  p->cluster_launch = v;
  snprintf(p->name, sizeof p->name, "%s", prop.name);
  return 0;
}

// ---- lifecycle ---------------------------------------------------------------------

extern "C" int mapal_gpu_device_count(int* count) {
  if (!count) return set_error(MAPAL_ERR_INVALID, "count is null");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  *count = n;
  return 0;
}

static int init_slot(DeviceSlot& d, int device) {
  d.device = device;
  MAPAL_CUDA(cudaSetDevice(device));
  MAPAL_TRY(read_profile(device, &d.prof));
  if (d.prof.cc_major != 10)
    return set_error(MAPAL_ERR_UNSUPPORTED,
                     "libmapal_gpu is built for sm_100a (B200); device " + std::to_string(device) +
                         " is sm_" + std::to_string(d.prof.cc_major) +
                         std::to_string(d.prof.cc_minor));
  MAPAL_CUDA(cudaStreamCreateWithFlags(&d.own_stream, cudaStreamNonBlocking));
  d.stream = d.own_stream;
  MAPAL_CUDA(cudaMalloc(&d.trap, sizeof(unsigned)));
  MAPAL_CUDA(cudaMemset(d.trap, 0, sizeof(unsigned)));
  MAPAL_CUDA(cudaMallocHost(&d.trap_host, sizeof(unsigned)));
  MAPAL_CUDA(cudaMalloc(&d.fold_partials, sizeof(double) * kFoldMaxBlocks));
  MAPAL_CUDA(cudaMalloc(&d.fold_counter, sizeof(unsigned)));
  MAPAL_CUDA(cudaMemset(d.fold_counter, 0, sizeof(unsigned)));
  MAPAL_CUDA(cudaMalloc(&d.fold_total, sizeof(double)));
  MAPAL_CUDA(cudaDeviceSynchronize());
  return 0;
}

static void free_slot(DeviceSlot& d) {
  if (d.device < 0) return;
  cudaSetDevice(d.device);
  if (d.own_stream) cudaStreamSynchronize(d.own_stream);
  if (d.stream && d.stream != d.own_stream) cudaStreamSynchronize(d.stream);
  if (d.comm && nccl_api()->loaded) nccl_api()->CommDestroy(d.comm);
  cudaFree(d.trap);
  cudaFreeHost(d.trap_host);
  cudaFree(d.fold_partials);
  cudaFree(d.fold_counter);
  cudaFree(d.fold_total);
  cudaFree(d.arena);
  if (d.comm_stream) {
    cudaStreamSynchronize(d.comm_stream);
    cudaStreamDestroy(d.comm_stream);
  }
  for (cudaEvent_t e : d.events) cudaEventDestroy(e);
  for (cudaStream_t s : {d.h2d_stream, d.d2h_stream, d.aux_stream}) {
    if (s) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  }
  for (cudaEvent_t e : d.host_events) cudaEventDestroy(e);
  cudaFree(d.stage);
  for (int q = 0; q < kMaxPeers; ++q)
    if (d.peer_ipc[q]) cudaIpcCloseMemHandle(d.peer_blk[q]);
  cudaFree(d.xblk);
  if (d.own_stream) cudaStreamDestroy(d.own_stream);
  d = DeviceSlot{};
}

int slot_events(DeviceSlot& d, size_t n) {
  MAPAL_CUDA(cudaSetDevice(d.device));
  if (!d.comm_stream) MAPAL_CUDA(cudaStreamCreateWithFlags(&d.comm_stream, cudaStreamNonBlocking));
  while (d.events.size() < n) {
    cudaEvent_t e;
    MAPAL_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    d.events.push_back(e);
  }
  return 0;
}

extern "C" int mapal_gpu_ctx_create(uint32_t device_mask, MapalGpuCtx** out) {
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  *out = nullptr;
  int count = 0;
  mapal_gpu_device_count(&count);
  if (count == 0) return set_error(MAPAL_ERR_CUDA, "no CUDA device visible");
  std::vector<int> devs;
  for (int d = 0; d < 32; ++d)
    if (device_mask & (1u << d)) {
      if (d >= count)
        return set_error(MAPAL_ERR_INVALID, "device " + std::to_string(d) + " does not exist");
      devs.push_back(d);
    }
  if (devs.empty()) return set_error(MAPAL_ERR_INVALID, "empty device mask");
  MapalGpuCtx* ctx = new MapalGpuCtx();
  ctx->dev.resize(devs.size());
  ctx->nranks = (int)devs.size();
  for (size_t i = 0; i < devs.size(); ++i) {
    int rc = init_slot(ctx->dev[i], devs[i]);
    if (rc) {
      mapal_gpu_ctx_destroy(ctx);
      return rc;
    }
  }
  if (devs.size() > 1) {
    NcclApi* n = nccl_api();
    if (!n->loaded) {
      mapal_gpu_ctx_destroy(ctx);
      return set_error(MAPAL_ERR_NCCL, n->error);
    }
    std::vector<ncclComm_t> comms(devs.size());
    int rc = n->CommInitAll(comms.data(), (int)devs.size(), devs.data());
    if (rc) {
      mapal_gpu_ctx_destroy(ctx);
      return nccl_fail(rc, "ncclCommInitAll");
    }
    for (size_t i = 0; i < devs.size(); ++i) ctx->dev[i].comm = comms[i];
  }
  *out = ctx;
  return 0;
}

extern "C" int mapal_gpu_nccl_unique_id(uint8_t id[128]) {
  if (!id) return set_error(MAPAL_ERR_INVALID, "id is null");
  NcclApi* n = nccl_api();
  if (!n->loaded) return set_error(MAPAL_ERR_NCCL, n->error);
  NcclId u;
  int rc = n->GetUniqueId(&u);
  if (rc) return nccl_fail(rc, "ncclGetUniqueId");
  memcpy(id, u.internal, 128);
  return 0;
}

extern "C" int mapal_gpu_ctx_create_rank(int device, int nranks, int rank, const uint8_t id[128],
                                         MapalGpuCtx** out) {
  if (!out || nranks < 1 || rank < 0 || rank >= nranks || (nranks > 1 && !id))
    return set_error(MAPAL_ERR_INVALID, "bad rank arguments");
  *out = nullptr;
  MapalGpuCtx* ctx = new MapalGpuCtx();
  ctx->dev.resize(1);
  ctx->nranks = nranks;
  ctx->rank0 = rank;
  int rc = init_slot(ctx->dev[0], device);
  if (rc) {
    mapal_gpu_ctx_destroy(ctx);
    return rc;
  }
  if (nranks > 1) {
    NcclApi* n = nccl_api();
    if (!n->loaded) {
      mapal_gpu_ctx_destroy(ctx);
      return set_error(MAPAL_ERR_NCCL, n->error);
    }
    NcclId u;
    memcpy(u.internal, id, 128);
    if (n->CommInitRankConfig) {
      // The config as NCCL 2.14 laid it out (NCCL reads a config by its size
      // and version fields, so later libraries take it and keep their
      // defaults for the fields it lacks); only maxCTAs is set.
      struct {
        size_t size;
        unsigned int magic, version;
        int blocking, cgaClusterSize, minCTAs, maxCTAs;
        const char* netName;
      } cfg = {sizeof(cfg), 0xcafebeefu, 2 * 10000 + 14 * 100, INT_MIN, INT_MIN, INT_MIN, kCollectiveCtas, nullptr};
      rc = n->CommInitRankConfig(&ctx->dev[0].comm, nranks, u, rank, &cfg);
      // a library that rejects the config (ncclInvalidArgument, raised while
      // the config is read, before any rank connects) gets a plain init
      if (rc == 4) rc = n->CommInitRank(&ctx->dev[0].comm, nranks, u, rank);
    } else {
      rc = n->CommInitRank(&ctx->dev[0].comm, nranks, u, rank);
    }
    if (rc) {
      mapal_gpu_ctx_destroy(ctx);
      return nccl_fail(rc, "ncclCommInitRank");
    }
  }
  *out = ctx;
  return 0;
}

extern "C" int mapal_gpu_ctx_destroy(MapalGpuCtx* ctx) {
  if (!ctx) return 0;
  for (auto& d : ctx->dev) free_slot(d);
  delete ctx;
  return 0;
}

extern "C" int mapal_gpu_ctx_local_devices(MapalGpuCtx* ctx, int* n) {
  if (!ctx || !n) return set_error(MAPAL_ERR_INVALID, "null argument");
  *n = (int)ctx->dev.size();
  return 0;
}

extern "C" int mapal_gpu_ctx_world(MapalGpuCtx* ctx, int* nranks, int* rank) {
  if (!ctx || !nranks || !rank) return set_error(MAPAL_ERR_INVALID, "null argument");
  *nranks = ctx->nranks;
  *rank = ctx->rank0;
  return 0;
}

extern "C" int mapal_gpu_ctx_sum_combine(MapalGpuCtx* ctx, int* mode) {
  if (!ctx || !mode) return set_error(MAPAL_ERR_INVALID, "null argument");
  *mode = ctx->peer_state;
  return 0;
}

extern "C" int mapal_gpu_profile(MapalGpuCtx* ctx, int local, MapalGpuProfile* out) {
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  MAPAL_TRY(enter(ctx, local));
  *out = ctx->dev[local].prof;
  return 0;
}

extern "C" int mapal_gpu_get_stream(MapalGpuCtx* ctx, int local, void** stream) {
  if (!stream) return set_error(MAPAL_ERR_INVALID, "stream is null");
  MAPAL_TRY(enter(ctx, local));
  *stream = (void*)ctx->dev[local].stream;
  return 0;
}

extern "C" int mapal_gpu_set_stream(MapalGpuCtx* ctx, int local, void* stream) {
  MAPAL_TRY(enter(ctx, local));
  // Taken as given, as everywhere in CUDA: NULL is the legacy default stream.
  // The context's own stream is the value mapal_gpu_get_stream returned
  // before any set_stream.
  ctx->dev[local].stream = (cudaStream_t)stream;
  return 0;
}

extern "C" int mapal_gpu_set_sync(MapalGpuCtx* ctx, int sync) {
  if (!ctx) return set_error(MAPAL_ERR_INVALID, "ctx is null");
  ctx->sync = sync != 0;
  return 0;
}

// ---- launch protocol -----------------------------------------------------------------

int enter(MapalGpuCtx* ctx, int local) {
  if (!ctx) return set_error(MAPAL_ERR_INVALID, "ctx is null");
  if (local < 0 || local >= (int)ctx->dev.size())
    return set_error(MAPAL_ERR_INVALID, "local device index out of range");
  MAPAL_CUDA(cudaSetDevice(ctx->dev[local].device));
  return 0;
}

// Synchronous readback of the flag (module.rs:86-94): the copy is the sync
// point; a nonzero flag is decoded, then cleared for the next launch.
int drain(DeviceSlot& d) {
  MAPAL_CUDA(cudaSetDevice(d.device));
  MAPAL_CUDA(cudaMemcpyAsync(d.trap_host, d.trap, sizeof(unsigned), cudaMemcpyDeviceToHost, d.stream));
  MAPAL_CUDA(cudaStreamSynchronize(d.stream));
  unsigned kind = *d.trap_host;
  if (kind != 0) {
    MAPAL_CUDA(cudaMemsetAsync(d.trap, 0, sizeof(unsigned), d.stream));
    MAPAL_CUDA(cudaStreamSynchronize(d.stream));
    if (kind == 1) return set_error(MAPAL_TRAP_DIV_ZERO, "mapal trap: div_zero");
    if (kind == 2) return set_error(MAPAL_TRAP_INDEX_OOB, "mapal trap: index_oob");
    if (kind & kPeerOutOfStep)
      return set_error(MAPAL_ERR_NCCL, "ranks out of step in the sharded-sum exchange (a rank skipped a call)");
    if (kind & 0x100u) return set_error(MAPAL_ERR_TIMEOUT, "a bounded device wait gave up");
    return set_error(MAPAL_ERR_CUDA, "trap flag holds an unknown kind");
  }
  return 0;
}

int finish(MapalGpuCtx* ctx, int local, bool trap_capable) {
  MAPAL_CUDA(cudaGetLastError());
  if (!ctx->sync) return 0;
  DeviceSlot& d = ctx->dev[local];
  if (trap_capable) return drain(d);
  MAPAL_CUDA(cudaStreamSynchronize(d.stream));
  return 0;
}

extern "C" int mapal_gpu_synchronize(MapalGpuCtx* ctx) {
  if (!ctx) return set_error(MAPAL_ERR_INVALID, "ctx is null");
  int first = 0;
  for (auto& d : ctx->dev) {
    int rc = drain(d);
    if (rc && !first) first = rc;
  }
  return first;
}

int arena_reserve(DeviceSlot& d, size_t bytes) {
  if (bytes <= d.arena_bytes) return 0;
  MAPAL_CUDA(cudaSetDevice(d.device));
  if (d.arena) {
    MAPAL_CUDA(cudaStreamSynchronize(d.stream));
    MAPAL_CUDA(cudaFree(d.arena));
    d.arena = nullptr;
    d.arena_bytes = 0;
  }
  size_t round = (bytes + (64u << 20) - 1) & ~((size_t)(64u << 20) - 1);
  MAPAL_CUDA(cudaMalloc(&d.arena, round));
  d.arena_bytes = round;
  return 0;
}

// ---- the sharding rule ---------------------------------------------------------------

extern "C" int mapal_gpu_shard_range(uint64_t n, int nranks, int r, uint64_t* lo, uint64_t* hi) {
  if (nranks < 1 || r < 0 || r >= nranks || !lo || !hi)
    return set_error(MAPAL_ERR_INVALID, "bad shard arguments");
  // Contiguous, equal up to one unit: the first n % nranks ranks get one more.
  uint64_t base = n / (uint64_t)nranks, extra = n % (uint64_t)nranks;
  uint64_t rr = (uint64_t)r;
  *lo = rr * base + (rr < extra ? rr : extra);
  *hi = *lo + base + (rr < extra ? 1 : 0);
  return 0;
}

// NCCL helpers used by the sharded entry points.
int nccl_allreduce_f64(MapalGpuCtx* ctx, double* const* buf, size_t count) {
  NcclApi* n = nccl_api();
  if (ctx->nranks == 1) return 0;
  if (!n->loaded) return set_error(MAPAL_ERR_NCCL, n->error);
  int rc = n->GroupStart();
  if (rc) return nccl_fail(rc, "ncclGroupStart");
  for (auto i = 0u; i < ctx->dev.size(); ++i) {
    DeviceSlot& d = ctx->dev[i];
    rc = n->AllReduce(buf[i], buf[i], count, kNcclFloat64, kNcclSum, d.comm, d.stream);
    if (rc) {
      n->GroupEnd();
      return nccl_fail(rc, "ncclAllReduce");
    }
  }
  rc = n->GroupEnd();
  if (rc) return nccl_fail(rc, "ncclGroupEnd");
  return 0;
}

int nccl_broadcast_f32(MapalGpuCtx* ctx, float* const* buf, size_t count, int root) {
  return nccl_broadcast_f32_on(ctx, buf, 0, count, root, false);
}

// Broadcast buf[i][offset, offset + count) from `root` on every local device,
// on the devices' comm streams when on_comm (slot_events must have run).
int nccl_broadcast_f32_on(MapalGpuCtx* ctx, float* const* buf, size_t offset, size_t count, int root,
                          bool on_comm) {
  NcclApi* n = nccl_api();
  if (ctx->nranks == 1) return 0;
  if (!n->loaded) return set_error(MAPAL_ERR_NCCL, n->error);
  int rc = n->GroupStart();
  if (rc) return nccl_fail(rc, "ncclGroupStart");
  for (auto i = 0u; i < ctx->dev.size(); ++i) {
    DeviceSlot& d = ctx->dev[i];
    rc = n->Broadcast(buf[i] + offset, buf[i] + offset, count, kNcclFloat32, root, d.comm,
                      on_comm ? d.comm_stream : d.stream);
    if (rc) {
      n->GroupEnd();
      return nccl_fail(rc, "ncclBroadcast");
    }
  }
  rc = n->GroupEnd();
  if (rc) return nccl_fail(rc, "ncclGroupEnd");
  return 0;
}

// ---- peer exchange setup ---------------------------------------------------------------
//
// One process over several devices: peer access between every pair, and the
// blocks are plain device pointers. One process per device: each rank exports
// its block as an IPC handle, the handles are all-gathered over NCCL and
// opened. Every rank then agrees (an NCCL sum of the ranks that succeeded), so
// either all ranks combine over peer memory or all use ncclAllReduce.
// MAPAL_GPU_PEER_COMBINE=0 in any rank's environment selects ncclAllReduce;
// MAPAL_GPU_PEER_WAIT_MS bounds the wait for the other ranks (default 10 s).
int peer_setup(MapalGpuCtx* ctx) {
  if (ctx->peer_state) return 0;
  const int R = ctx->nranks, L = (int)ctx->dev.size();
  if (R < 2) {
    ctx->peer_state = -1;
    return 0;
  }
  NcclApi* n = nccl_api();
  if (!n->loaded) return set_error(MAPAL_ERR_NCCL, n->error);
  const char* env = getenv("MAPAL_GPU_PEER_COMBINE");
  if (const char* w = getenv("MAPAL_GPU_PEER_WAIT_MS")) {
    const long long ms = atoll(w);
    if (ms > 0 && ms <= 600000) ctx->peer_wait_ns = (unsigned long long)ms * 1000000ull;
  }
  if (L != R && L != 1) {  // not a layout the context constructors make
    ctx->peer_state = -1;
    return 0;
  }
  bool ok = R <= kMaxPeers && !(env && env[0] == '0');
  constexpr size_t kBlockBytes = 64 << 10;
  static_assert(sizeof(PeerBlock) <= kBlockBytes, "peer block");
  for (auto& d : ctx->dev) {
    MAPAL_CUDA(cudaSetDevice(d.device));
    if (!d.xblk) {
      MAPAL_CUDA(cudaMalloc(&d.xblk, kBlockBytes));
      MAPAL_CUDA(cudaMemset(d.xblk, 0, kBlockBytes));
      MAPAL_CUDA(cudaDeviceSynchronize());
    }
  }
  if (L == R) {
    // every rank is a local device of this process
    for (int i = 0; i < L && ok; ++i) {
      MAPAL_CUDA(cudaSetDevice(ctx->dev[i].device));
      for (int j = 0; j < L && ok; ++j) {
        ctx->dev[i].peer_blk[j] = ctx->dev[j].xblk;
        if (i == j) continue;
        int can = 0;
        cudaDeviceCanAccessPeer(&can, ctx->dev[i].device, ctx->dev[j].device);
        cudaError_t e = can ? cudaDeviceEnablePeerAccess(ctx->dev[j].device, 0) : cudaErrorPeerAccessUnsupported;
        if (e == cudaErrorPeerAccessAlreadyEnabled) e = cudaSuccess;
        if (e != cudaSuccess) ok = false;
        cudaGetLastError();
      }
    }
    ctx->peer_state = ok ? 1 : -1;
    return 0;
  }
  // one device per process: exchange IPC handles
  DeviceSlot& d = ctx->dev[0];
  const int me = ctx->rank0;
  cudaIpcMemHandle_t mine{};
  if (ok && cudaIpcGetMemHandle(&mine, d.xblk) != cudaSuccess) {
    ok = false;
    cudaGetLastError();
  }
  if (n->AllGather == nullptr) return set_error(MAPAL_ERR_NCCL, "libnccl lacks ncclAllGather");
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  std::vector<uint8_t> all(hb * R);
  uint8_t* dbuf = nullptr;
  MAPAL_CUDA(cudaMalloc(&dbuf, hb * R));
  MAPAL_CUDA(cudaMemcpy(dbuf + hb * me, &mine, hb, cudaMemcpyHostToDevice));
  int rc = n->AllGather(dbuf + hb * me, dbuf, hb, kNcclUint8, d.comm, d.stream);
  if (rc) {
    cudaFree(dbuf);
    return nccl_fail(rc, "ncclAllGather");
  }
  MAPAL_CUDA(cudaStreamSynchronize(d.stream));
  MAPAL_CUDA(cudaMemcpy(all.data(), dbuf, hb * R, cudaMemcpyDeviceToHost));
  MAPAL_CUDA(cudaFree(dbuf));
  for (int q = 0; q < R && ok; ++q) {
    if (q == me) {
      d.peer_blk[q] = d.xblk;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, all.data() + hb * q, hb);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      ok = false;
      cudaGetLastError();
      break;
    }
    d.peer_blk[q] = (PeerBlock*)p;
    d.peer_ipc[q] = true;
  }
  // agreement: the number of ranks that mapped every peer
  double flag = ok ? 1.0 : 0.0;
  MAPAL_CUDA(cudaMemcpy(d.fold_total, &flag, sizeof flag, cudaMemcpyHostToDevice));
  double* tot[1] = {d.fold_total};
  MAPAL_TRY(nccl_allreduce_f64(ctx, tot, 1));
  MAPAL_CUDA(cudaStreamSynchronize(d.stream));
  MAPAL_CUDA(cudaMemcpy(&flag, d.fold_total, sizeof flag, cudaMemcpyDeviceToHost));
  ctx->peer_state = flag == (double)R ? 1 : -1;
  return 0;
}
