// common.cuh — shared internals of libmapal_gpu (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <vector>

#include "../../include/mapal_gpu.h"

// ---- NCCL, bound at run time ------------------------------------------------
// The library never links libnccl: it dlopens libnccl.so.2 the first time a
// multi-device context is created, so single-GPU users and CPU-only loads need
// no NCCL. Only the handful of entry points below are used.
typedef struct ncclComm* ncclComm_t;
struct NcclId {
  char internal[128];
};
enum NcclDtype { kNcclUint8 = 1, kNcclFloat32 = 7, kNcclFloat64 = 8 };
enum NcclOp { kNcclSum = 0 };

struct NcclApi {
  bool loaded = false;
  std::string error;
  int (*GetUniqueId)(NcclId*) = nullptr;
  int (*CommInitRank)(ncclComm_t*, int, NcclId, int) = nullptr;
  int (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
  int (*CommDestroy)(ncclComm_t) = nullptr;
  int (*AllReduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  int (*Broadcast)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  int (*GroupStart)() = nullptr;
  int (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(int) = nullptr;
  int (*AllGather)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
  // optional (NCCL >= 2.14): rank init with a config, used to cap the CTAs
  int (*CommInitRankConfig)(ncclComm_t*, int, NcclId, int, void*) = nullptr;
};
NcclApi* nccl_api();  // loads on first use; check ->loaded

// The most CTAs a rank communicator's collectives use (NCCL's maxCTAs). A
// collective launched beside a multiply runs in the SMs the multiply's
// part-filled wave leaves free, and completes only when all its CTAs have
// run, so it must fit there: the strict matmul's plan keeps at least this
// many SMs free beside a collective (20 at the row-sharded 4096^2 site's
// 8-GPU block, 40 at its 4-GPU block).
constexpr int kCollectiveCtas = 16;

// ---- peer exchange --------------------------------------------------------------
// The sharded sum combines its per-rank partials over peer memory inside the
// fold kernel: every rank stores its partial into every rank's block and
// raises its flag there, then waits for every rank's flag in its own block and
// adds the partials in rank order. Values are double-buffered by the parity of
// a per-call epoch, so a rank one call ahead never overwrites a value that a
// slower rank has yet to read.
constexpr int kMaxPeers = 8;  // one NVSwitch node
struct PeerSlot {
  double v;
  unsigned long long epoch;  // the call that wrote v
};
struct PeerBlock {
  PeerSlot val[2][kMaxPeers];          // [epoch parity][source rank]
  unsigned long long flag[kMaxPeers];  // last epoch each source rank published
};
struct PeerArgs {
  PeerBlock* blk[kMaxPeers];  // every rank's block as this device addresses it
  PeerBlock* own;             // this device's block
  int nranks;
  int rank;
  unsigned long long epoch;
  unsigned long long wait_ns;  // how long to wait for a rank that has not published
  unsigned* trap;              // 0x100: a wait gave up; 0x200: ranks out of step
};
constexpr unsigned kPeerTimeout = 0x100u;
constexpr unsigned kPeerOutOfStep = 0x200u;

// ---- context ------------------------------------------------------------------

struct DeviceSlot {
  int device = -1;
  cudaStream_t stream = nullptr;      // the stream work is enqueued on
  cudaStream_t own_stream = nullptr;  // created by the context
  unsigned* trap = nullptr;           // device trap flag: 0 quiescent, kind+1 after a trap
  unsigned* trap_host = nullptr;      // pinned readback slot
  // Fold scratch: one f64 partial per block, a block-arrival counter and a
  // f64 cell for cross-rank combination. Allocated once at context creation.
  double* fold_partials = nullptr;
  unsigned* fold_counter = nullptr;
  double* fold_total = nullptr;
  // Growable arena for the 3xTF32 operand splits (cudaMalloc on growth only).
  void* arena = nullptr;
  size_t arena_bytes = 0;
  ncclComm_t comm = nullptr;
  // Collectives that overlap compute run on this stream, ordered against
  // `stream` with events from `events` (created on first use, reused).
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> events;
  // Host-array entry points: copy streams (one per PCIe direction), their
  // events and a growable device staging buffer, all created on first use.
  cudaStream_t h2d_stream = nullptr;
  cudaStream_t d2h_stream = nullptr;
  cudaStream_t aux_stream = nullptr;  // a second compute stream: row blocks alternate with `stream`
  std::vector<cudaEvent_t> host_events;
  void* stage = nullptr;
  size_t stage_bytes = 0;
  // Peer exchange (set up by the first sharded sum): this device's block and
  // every rank's block as mapped here (peer access or an IPC mapping).
  PeerBlock* xblk = nullptr;
  PeerBlock* peer_blk[kMaxPeers] = {};
  bool peer_ipc[kMaxPeers] = {};  // opened with cudaIpcOpenMemHandle
  MapalGpuProfile prof{};
};

struct MapalGpuCtx {
  std::vector<DeviceSlot> dev;
  int nranks = 1;  // ranks of the communicator
  int rank0 = 0;   // global rank of local device 0
  bool sync = true;
  int peer_state = 0;              // 0 not tried, 1 peer combine ready, -1 NCCL only
  unsigned long long xepoch = 0;   // sharded-sum calls made through the peer combine
  unsigned long long peer_wait_ns = 10ull * 1000 * 1000 * 1000;  // MAPAL_GPU_PEER_WAIT_MS
};

// Blocks per fold launch is fixed per n (deterministic); this bounds it.
constexpr int kFoldMaxBlocks = 4 * 148 * 4;

// ---- error plumbing -------------------------------------------------------------
int set_error(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
#define MAPAL_CUDA(call)                                   \
  do {                                                     \
    cudaError_t _e = (call);                               \
    if (_e != cudaSuccess) return cuda_fail(_e, #call);    \
  } while (0)
#define MAPAL_TRY(expr)          \
  do {                           \
    int _rc = (expr);            \
    if (_rc != 0) return _rc;    \
  } while (0)

// Raise a kernel's dynamic shared-memory limit on the current device (device
// number `device`) the first time it is launched there. `done` keeps one bit
// per device; two host threads launching first at once may both set the
// attribute, which is harmless (the value is the same). Devices beyond 63 set
// it on every launch.
inline int ensure_smem_attr(std::atomic<uint64_t>& done, const void* kernel, int device, size_t bytes,
                            const char* what) {
  const uint64_t bit = device >= 0 && device < 64 ? 1ull << device : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return 0;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return cuda_fail(e, what);
  done.fetch_or(bit, std::memory_order_release);
  return 0;
}

// One kernel launch issued by this library (process-wide count, read by
// mapal_gpu_launch_count).
void count_launch();

// Validate ctx and local index; make the device current.
int enter(MapalGpuCtx* ctx, int local = 0);
// After a launch: report launch errors; in sync mode wait and decode traps.
int finish(MapalGpuCtx* ctx, int local, bool trap_capable);
// Wait and decode the trap flag of one device.
int drain(DeviceSlot& d);
// Ensure the arena of a device holds `bytes` (grows, never shrinks).
int arena_reserve(DeviceSlot& d, size_t bytes);

// Grid size for a streaming kernel: enough resident blocks to fill every SM.
inline unsigned stream_grid(uint64_t work_items, int threads, int sms, int blocks_per_sm) {
  uint64_t want = (work_items + threads - 1) / threads;
  uint64_t cap = (uint64_t)sms * blocks_per_sm;
  if (want > cap) want = cap;
  if (want == 0) want = 1;
  return (unsigned)want;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// ---- site-class launchers (one per .cu file) -----------------------------------
int launch_fill(cudaStream_t s, int sms, float* out, float v, uint64_t n);
int launch_gen_affine(cudaStream_t s, int sms, float* out, uint64_t n, int64_t start, int32_t mul,
                      int32_t add, int32_t mod, int32_t sub);
int launch_gen_f32(cudaStream_t s, int sms, float* out, uint64_t n, int32_t seed, int64_t offset,
                   int kind);
int launch_saxpy(cudaStream_t s, int sms, float a, const float* x, const float* y0, float* y,
                 uint64_t n);
int launch_gather(cudaStream_t s, int sms, const float* x, uint64_t n_x, const int32_t* idx,
                  float* out, uint64_t n, unsigned* trap);
int launch_fold_sum(cudaStream_t s, int sms, const float* x, uint64_t n, float seed, double* partials,
                    unsigned* counter, float* out_f32, double* out_f64);
int launch_finalize_sum(cudaStream_t s, const double* total, float seed, float* out);
// The fold with the cross-rank combine in its last block (out = seed + the
// rank-ordered sum of every rank's partial).
int launch_fold_sum_peer(cudaStream_t s, int sms, const float* x, uint64_t n, float seed, double* partials,
                         unsigned* counter, float* out, const PeerArgs& P);
// Map every rank's exchange block (collective on the first call; sets
// ctx->peer_state, -1 when any rank cannot map its peers).
int peer_setup(MapalGpuCtx* ctx);
int launch_matmul_strict(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M,
                         uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed);
// acc_from_c: continue every cell from C's value (a later k-range).
// beside_collective: an SM-based collective (an NCCL kernel) runs beside
// this launch, so the plan keeps a part-filled wave for it to run in.
int launch_matmul_strict_ex(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M,
                            uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed,
                            int acc_from_c, int beside_collective);
// Record checks of tile.cu: status, and whether the record is matmul-shaped.
int validate_tile_site(const MapalTileSite* site, const void* a, const void* b, const void* out, bool* empty,
                       bool* matmul_shaped);
// At least n reusable events on a device slot; the comm stream on first use.
int slot_events(DeviceSlot& d, size_t n);
int nccl_broadcast_f32_on(MapalGpuCtx* ctx, float* const* buf, size_t offset, size_t count, int root,
                          bool on_comm);
int launch_matmul_tf32x3(DeviceSlot& d, const float* A, const float* B, float* C, uint64_t M,
                         uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed);
