/*
 * mapal_gpu.h — C ABI of libmapal_gpu, the sm_100a (B200) runtime for Mapal's
 * bulk array sites.
 *
 * What this replaces. The reference compiles each bulk site of a sealed
 * CategoryIr into its own `__global__` function and launches it from emitted
 * host code:
 *   - `emit` / `emit_with_opts` produce one .cu translation unit
 *     (crates/backends/cuda/src/lib.rs:72-111);
 *   - each site becomes a kernel from the emitters in
 *     crates/backends/cuda/src/kernel.rs:1156-1642;
 *   - emitted host glue launches it and checks the trap flag
 *     (crates/backends/cuda/src/func.rs:1159-1197, module.rs:61-95).
 * Here the kernels are fixed, hand-written sm_100a kernels. A backend calls
 * one entry point per recognized site class, passing the site's record
 * (TileSite, crates/mapal-ir/src/algo.rs:335-345; MoveSite, algo.rs:309-333)
 * and caller-owned device buffers. No C++ type crosses this boundary.
 *
 * Status protocol (every entry point returns int):
 *    0  ok
 *    1  trap div_zero   } the device trap-flag decode of module.rs:86-94:
 *    2  trap index_oob  } flag = kind + 1, host maps to exit 101
 *   <0  infrastructure error (the reference's exit-102 class, module.rs:66-71);
 *       mapal_gpu_last_error() returns the message.
 *
 * Threading: one host thread per context. Calls are stream-ordered on the
 * context's stream for the device. With sync mode on (the default) a call
 * returns after its work finished and any trap has been decoded, which is the
 * reference's launch-then-check order. With sync mode off a call returns
 * after enqueueing, and traps surface at mapal_gpu_synchronize().
 *
 * Floating point: every f32 `+` and `*` of a site is separately rounded
 * (round-to-nearest-even, no contraction, denormals kept), as the
 * interpreter evaluates them (crates/mapal-interp/src/eval.rs:572-585).
 * Exceptions, each stated where it applies: fold sums reassociate
 * (mapal_gpu_fold_sum_f32) and MAPAL_MATMUL_TF32X3 uses tensor cores.
 */
#ifndef MAPAL_GPU_H
#define MAPAL_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Every symbol declared here is exported even when the library is built with
 * hidden default visibility. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define MAPAL_GPU_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------ */
#define MAPAL_OK 0
#define MAPAL_TRAP_DIV_ZERO 1  /* mapal_trap(0) in mapal-rt/src/lib.rs:71-81 */
#define MAPAL_TRAP_INDEX_OOB 2 /* mapal_trap(1) */
#define MAPAL_ERR_INVALID (-1)     /* bad argument or descriptor */
#define MAPAL_ERR_UNSUPPORTED (-2) /* site shape this library has no kernel for
                                      (EmitError::Unsupported, cuda/src/lib.rs:74-80) */
#define MAPAL_ERR_CUDA (-3)        /* CUDA runtime / driver error */
#define MAPAL_ERR_NCCL (-4)        /* NCCL error or NCCL unavailable */
#define MAPAL_ERR_NOMEM (-5)       /* device allocation of internal scratch failed */
#define MAPAL_ERR_TIMEOUT (-6)     /* a bounded device wait gave up */

/* ---- records ------------------------------------------------------------ */

/* The `k = kq*div + kr` decomposition of a fold axis (TileKSplit,
 * crates/mapal-ir/src/algo.rs:245-257). div == 0 means "no split". */
typedef struct MapalKSplit {
  uint64_t div;
  uint64_t cq; /* address coefficient on k / div */
  uint64_t cr; /* address coefficient on k % div */
} MapalKSplit;

/* One affine array read of a tiled site (TileRead, algo.rs:227-240):
 *   addr(i, lane, k) = base + ci*i + clane*lane + ck*k
 *                      + ksplit.cq*(k/div) + ksplit.cr*(k%div)
 * `len` is the read array's length in elements; reads at addr >= len trap
 * index_oob, as the interpreter's Index does (eval.rs:655-669). */
typedef struct MapalTileRead {
  uint64_t base;
  uint64_t ci;
  uint64_t ck;
  uint64_t clane;
  MapalKSplit ksplit;
  uint64_t len;
} MapalTileRead;

/* A recognized map-of-fold site (TileSite, algo.rs:335-345). The site
 * computes rows*c cells, cell t = i*c + lane (i = t / c, lane = t % c):
 *   acc = seed
 *   for k in 0..k:  p   = mul_a_first ? a[addr_a] * b[addr_b] : b[addr_b] * a[addr_a]
 *                   acc = add_acc_first ? acc + p : p + acc
 *   out[t] = acc
 * with the fold strictly left to right (eval.rs:326-359). */
typedef struct MapalTileSite {
  uint64_t rows;
  uint64_t c;
  uint64_t k;
  MapalTileRead a;
  MapalTileRead b;
  float seed;
  uint8_t mul_a_first;
  uint8_t add_acc_first;
  uint8_t reserved[2];
} MapalTileSite;

/* A fold-less move site (MoveSite, algo.rs:309-333): the map over
 * t in [0, rows*width) computes out[t] = in[cq*(t/width) + cr*(t%width)].
 * A transpose of an R x C row-major matrix is width=R, rows=C, cq=1, cr=C. */
typedef struct MapalMoveSite {
  uint64_t width;
  uint64_t rows;
  uint64_t cq;
  uint64_t cr;
  uint64_t len; /* length of `in` in elements */
} MapalMoveSite;

/* Machine facts for the tiler: the sm_100a counterpart of the reference's
 * placeholder Machine::Gpu / CUDA_ADA profile
 * (crates/backends/llvm/src/profile.rs:99-156, 781-800). */
typedef struct MapalGpuProfile {
  int32_t device;
  int32_t cc_major;
  int32_t cc_minor;
  int32_t sm_count;
  int32_t warp_size;
  int32_t max_threads_per_block;
  int32_t max_threads_per_sm;
  int32_t regs_per_sm;
  int64_t smem_per_sm;          /* bytes */
  int64_t smem_per_block_optin; /* bytes, the opt-in maximum */
  int64_t l2_bytes;
  int64_t tmem_bytes_per_sm;    /* tensor memory: 128 lanes x 512 columns x 4 B */
  int64_t hbm_bytes;
  int32_t sm_clock_khz;         /* maximum SM clock */
  int32_t mem_clock_khz;
  int32_t mem_bus_bits;
  int32_t cluster_launch;       /* 1 if thread-block clusters are supported */
  char name[96];
} MapalGpuProfile;

/* matmul precision modes */
#define MAPAL_MATMUL_STRICT 0 /* SIMT, separately rounded mul and add in the
                                 interpreter's order: bit-identical */
#define MAPAL_MATMUL_TF32X3 1 /* tcgen05 tensor cores, 3xTF32 split; opt-in,
                                 within a stated relative error (ADR-0032's
                                 tf32-class contract): per cell
                                 |C - A.B| <= 2e-6 * ||A_i,:|| * ||B_:,j|| for
                                 K <= 4096 (the tensor pipe's accumulation
                                 error grows with K; B200-measured at most
                                 1.1e-6 at K = 4096 and 1.9e-6 at K = 16384).
                                 A cell that reads a NaN is NaN; one that
                                 reads an infinity is not finite. */

/* generator kinds for mapal_gpu_gen_f32 */
#define MAPAL_GEN_U11 0 /* uniform[-1,1) */
#define MAPAL_GEN_U01 1 /* uniform[0,1) */

typedef struct MapalGpuCtx MapalGpuCtx;

/* ---- lifecycle ------------------------------------------------------------ */

/* Library ABI version (MAPAL_GPU_ABI_VERSION). */
int mapal_gpu_abi_version(void);

/* Message of the last error on this thread ("" if none). */
const char* mapal_gpu_last_error(void);

/* Kernel launches this library has issued in this process, all devices and
 * contexts (a diagnostic: take the difference around a region of calls). */
uint64_t mapal_gpu_launch_count(void);

/* Number of visible CUDA devices (0 when no driver or no device). */
int mapal_gpu_device_count(int* count);

/* Create a context over the devices whose bits are set in device_mask (bit d =
 * CUDA device d). Owns one stream per device, the device trap flags and, for
 * more than one device, one NCCL communicator per device (single-process
 * multi-GPU: the auto-partitioner's shape). Replaces the per-process
 * trap_init() of the emitted prelude (module.rs:74-77). */
int mapal_gpu_ctx_create(uint32_t device_mask, MapalGpuCtx** out);

/* Create a context for one rank of a multi-process job (one process per GPU).
 * All ranks pass the same 128-byte id, made once by
 * mapal_gpu_nccl_unique_id() on one rank and shared by the caller. The
 * rank's communicator caps its collectives at 16 CTAs (NCCL maxCTAs, where
 * the loaded NCCL has ncclCommInitRankConfig), so a collective overlapped
 * with a multiply fits in the SMs the multiply leaves free. */
int mapal_gpu_nccl_unique_id(uint8_t id[128]);
int mapal_gpu_ctx_create_rank(int device, int nranks, int rank, const uint8_t id[128],
                              MapalGpuCtx** out);

int mapal_gpu_ctx_destroy(MapalGpuCtx* ctx);

/* Number of devices this context drives in this process. */
int mapal_gpu_ctx_local_devices(MapalGpuCtx* ctx, int* n);
/* Total ranks of the context's communicator (1 for a one-device context). */
int mapal_gpu_ctx_world(MapalGpuCtx* ctx, int* nranks, int* rank);

/* Machine facts of local device `local`. */
int mapal_gpu_profile(MapalGpuCtx* ctx, int local, MapalGpuProfile* out);

/* Stream of local device `local` (a cudaStream_t). Replace it with a caller
 * stream to order this library's work with the caller's; NULL selects the
 * legacy default stream. The context's own stream is what get_stream returns
 * before the first set_stream. */
int mapal_gpu_get_stream(MapalGpuCtx* ctx, int local, void** stream);
int mapal_gpu_set_stream(MapalGpuCtx* ctx, int local, void* stream);

/* 1 (default): calls return after completion with traps decoded.
 * 0: calls return after enqueueing; traps surface at mapal_gpu_synchronize. */
int mapal_gpu_set_sync(MapalGpuCtx* ctx, int sync);

/* Wait for all work of the context; decode and clear the trap flags. */
int mapal_gpu_synchronize(MapalGpuCtx* ctx);

/* ---- input generators (iota / fill / widen and the seeded stream) ------- */
/* The reference's Iota, Fill and Widen kernels (kernel.rs:1335-1378;
 * eval.rs:238-248, 402-427), plus fused generators that recompute an element
 * from its index the way elem_plan lets a consumer do (algo.rs:434-512). */

/* out[i] = i for i < n (n <= 2^31) */
int mapal_gpu_iota_i32(MapalGpuCtx* ctx, int32_t* out, uint64_t n);
/* out[i] = v */
int mapal_gpu_fill_f32(MapalGpuCtx* ctx, float* out, float v, uint64_t n);
/* out[i] = (float)in[i]  (Widen i32 -> f32, round to nearest) */
int mapal_gpu_widen_i32_f32(MapalGpuCtx* ctx, const int32_t* in, float* out, uint64_t n);
/* out[i] = widen_f32((t*mul + add) % mod - sub), t = start + i, i32 wrapping
 * arithmetic: the integer generators of the benches/shapes sources, fused. */
int mapal_gpu_gen_affine_f32(MapalGpuCtx* ctx, float* out, uint64_t n, int64_t start,
                             int32_t mul, int32_t add, int32_t mod, int32_t sub);
/* out[i] = element (offset + i) of the seeded uniform stream `seed`
 * (kind MAPAL_GEN_U11 or MAPAL_GEN_U01). */
int mapal_gpu_gen_f32(MapalGpuCtx* ctx, float* out, uint64_t n, int32_t seed, int64_t offset,
                      int kind);
/* out[i] = index draw (offset + i) of stream `seed`, uniform in [0, range). */
int mapal_gpu_gen_index_i32(MapalGpuCtx* ctx, int32_t* out, uint64_t n, int32_t seed,
                            int64_t offset, int32_t range);

/* ---- site classes ---------------------------------------------------------- */

/* saxpy: y[i] = a*x[i] + y0[i] (benches/shapes/saxpy_1048576.mapal:11; the zip
 * then map of kernel.rs:1249-1293 and 1156-1247, fused: 12 bytes/element).
 * y may alias y0. */
int mapal_gpu_map_saxpy(MapalGpuCtx* ctx, float a, const float* x, const float* y0, float* y,
                        uint64_t n);

/* Elementwise zip-map out[i] = x[i] OP y[i] for the float binary ops of
 * eval.rs:572-585 (ADD, SUB, MUL, DIV, MOD = fmodf, as Rust's `%`). */
#define MAPAL_OP_ADD 0
#define MAPAL_OP_SUB 1
#define MAPAL_OP_MUL 2
#define MAPAL_OP_DIV 3
#define MAPAL_OP_MOD 4
int mapal_gpu_zip_map_f32(MapalGpuCtx* ctx, int op, const float* x, const float* y, float* out,
                          uint64_t n);

/* General map body, for Map sites whose element body is scalar arithmetic
 * (Map eval.rs:297-324 with the element ops of eval.rs:544-596; the rung-0
 * map kernels kernel.rs:1156-1333 cover the same ground with generated code).
 * out[t] for t in [0, n) is the value a stack program leaves, evaluated per
 * element over 32-bit values:
 *   T_I32            push t (the element index, < 2^31)
 *   CONST_I32/F32    push the immediate i / f
 *   IN_I32/F32 s     push arrays[s][t]   (the mapped or zipped inputs)
 *   LOAD_I32/F32 s   pop an i32 index j, push arrays[s][j]; j outside
 *                    [0, lens[s]) traps index_oob (the Index rule)
 *   ADD/SUB/MUL/DIV/REM/NEG _I32   wrapping i32; DIV and REM by zero trap
 *                    div_zero, MIN / -1 wraps, % takes the dividend's sign
 *   ADD/SUB/MUL/DIV/REM/NEG _F32   IEEE binary32, each op rounded (REM = fmodf)
 *   WIDEN_I32_F32    convert to f32, round to nearest
 *   STORE_I32/F32    pop the result; must be the last op
 * The program is checked on the host (types, stack depth <= 16, slots,
 * at most 64 ops) and rejected with MAPAL_ERR_INVALID if malformed. */
#define MAPAL_X_T_I32 0
#define MAPAL_X_CONST_I32 1
#define MAPAL_X_CONST_F32 2
#define MAPAL_X_IN_I32 3
#define MAPAL_X_IN_F32 4
#define MAPAL_X_LOAD_I32 5
#define MAPAL_X_LOAD_F32 6
#define MAPAL_X_ADD_I32 10
#define MAPAL_X_SUB_I32 11
#define MAPAL_X_MUL_I32 12
#define MAPAL_X_DIV_I32 13
#define MAPAL_X_REM_I32 14
#define MAPAL_X_NEG_I32 15
#define MAPAL_X_ADD_F32 20
#define MAPAL_X_SUB_F32 21
#define MAPAL_X_MUL_F32 22
#define MAPAL_X_DIV_F32 23
#define MAPAL_X_REM_F32 24
#define MAPAL_X_NEG_F32 25
#define MAPAL_X_WIDEN_I32_F32 30
#define MAPAL_X_STORE_I32 40
#define MAPAL_X_STORE_F32 41
#define MAPAL_X_MAX_OPS 64
#define MAPAL_X_MAX_ARRAYS 8

typedef struct MapalExprOp {
  uint16_t code;
  uint16_t slot;
  int32_t i;
  float f;
} MapalExprOp;

int mapal_gpu_map_expr(MapalGpuCtx* ctx, const MapalExprOp* prog, uint32_t nops, const void* const* arrays,
                       const uint64_t* lens, uint32_t narrays, void* out, uint64_t n);

/* Move site (transpose and other affine permutations),
 * benches/shapes/transpose_1024.mapal:11; MoveSite algo.rs:309-333. */
int mapal_gpu_transpose(MapalGpuCtx* ctx, const MapalMoveSite* site, const float* in,
                        float* out);

/* Gather out[i] = x[idx[i]] with the Index bounds rule (eval.rs:655-669;
 * kernel.rs:2655-2663): any idx outside [0, n_x) returns MAPAL_TRAP_INDEX_OOB
 * (out is then unspecified), as the emitted guard stores kind+1 = 2. */
int mapal_gpu_gather(MapalGpuCtx* ctx, const float* x, uint64_t n_x, const int32_t* idx,
                     float* out, uint64_t n);

/* Sum fold out = seed + x[0] + ... + x[n-1] (benches/shapes/reduce_1048576.mapal:10).
 * out is a device pointer to one float. NOT bit-exact with the interpreter's
 * left fold (ADR-0028 pins f32 folds sequential): this is a fixed-shape tree,
 * accumulated in f64 and rounded once, so it is deterministic run to run and
 * within 1e-6 * sum|x| of the exact sum. */
int mapal_gpu_fold_sum_f32(MapalGpuCtx* ctx, float seed, const float* x, uint64_t n, float* out);

/* Integer sum fold out = seed + x[0] + ... + x[n-1], wrapping i32 arithmetic
 * (eval.rs:552-569). Wrapping addition is associative and commutative, so any
 * order gives the interpreter's left-fold result exactly: one launch of
 * per-thread sums, a warp and block tree, and a wrapping atomic add per block.
 * out is a device pointer to one int32. */
int mapal_gpu_fold_sum_i32(MapalGpuCtx* ctx, int32_t seed, const int32_t* x, uint64_t n, int32_t* out);

/* The sum fold in the interpreter's order: acc = seed; acc = acc + x[i] for
 * i ascending, each add rounded to f32 (eval.rs:326-359), bit-exact with the
 * interpreter and with the reference's one-thread fold kernel
 * (kernel.rs:1484-1642). One block stages x through shared memory while one
 * thread runs the dependent chain, so its time is n times the f32 add
 * latency (about 2 ms per 2^20 elements), not a bandwidth bound. */
int mapal_gpu_fold_sum_f32_strict(MapalGpuCtx* ctx, float seed, const float* x, uint64_t n, float* out);

/* The same sum fold for callers that cannot allocate device memory: no
 * context, and no cudaMalloc / cudaFree or other allocation anywhere in the
 * call. This entry point has no counterpart in the reference.
 * Who needs it: a host runtime that serves every device byte from one arena it
 * sized up front and must not have a library allocate behind it, a process
 * already at its HBM limit, or a latency-bound loop that cannot take
 * cudaMalloc's implicit device synchronisation.
 * Scratch: a fixed 8 KiB + 8 B array in the library's device data (1024 f64
 * partial slots and a counter), present on every GPU that loads the library
 * until the process exits. A device whose fold launch would need more than
 * 1024 slots (more than 256 SMs) is refused with MAPAL_ERR_INVALID.
 * Runs on the calling thread's current device, enqueued on `stream` (a
 * cudaStream_t of that device, NULL = default stream; a stream of another
 * device is refused with MAPAL_ERR_INVALID); returns after enqueueing, so read
 * `out` (a device float) after synchronising the stream. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture. Host threads may call it
 * concurrently. The address is kept for the life of the process, so calls
 * after a cudaDeviceReset of that device are not supported. Calls share the
 * array: the counter is cleared on the stream before each launch, and calls
 * whose kernels overlap on the GPU race and give wrong results. */
int mapal_gpu_fold_sum_f32_noalloc(float seed, const float* x, uint64_t n, float* out, void* stream);

/* FIR / window site (benches/shapes/fir_1048576.mapal:10-12):
 * site must be rows=1, a = taps {ck=1, ci=0, clane=0}, b = signal {ck=1, clane=1,
 * ci=0}: out[t] = fold_k(acc + w[k]*x[t+k]) from seed, k ascending. Bit-exact. */
int mapal_gpu_fir_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* w,
                      const float* x, float* out);

/* 3x3 conv2d site (benches/shapes/conv2d_1024.mapal:11-15): a = 9 taps {ck=1},
 * b = image {ci=stride, clane=1, ck=0, ksplit={3, stride, 1}}. Bit-exact. */
int mapal_gpu_conv2d_3x3_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* w,
                             const float* img, float* out);

/* matmul site (benches/matmul/matmul1024_cap_f32.mapal:7-11): rows=M, c=N, k=K,
 * a = A {ci=lda, ck=1, clane=0}, b = B {ci=0, ck=ldb, clane=1}, out row-major M x N.
 * mode MAPAL_MATMUL_STRICT is bit-identical with the interpreter;
 * MAPAL_MATMUL_TF32X3 is within the bound stated at its definition. */
int mapal_gpu_matmul_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* A,
                         const float* B, float* C, int mode);

/* The same matmul site with A, B and C in HOST memory (the emitted program's
 * host<->device seam, one call instead of a blocking cudaMemcpy per array).
 * B is copied up first; A then goes up in row blocks on a copy stream while
 * earlier blocks multiply, and each finished block of C comes back on a
 * second copy stream, so with pinned (page-locked) host buffers the transfers
 * in both directions overlap the arithmetic; pageable buffers work, with
 * staged copies. Device memory is a staging buffer owned by the context
 * (grown on demand, freed with it). Results equal mapal_gpu_matmul_f32's in
 * the same mode. In async mode, C is complete once the context is
 * synchronised; A, B and C must stay valid and unmodified until then. */
int mapal_gpu_matmul_f32_host(MapalGpuCtx* ctx, const MapalTileSite* site, const float* A,
                              const float* B, float* C, int mode);

/* The host-array matmul site over the context's ranks: local device d owns
 * m[d] rows of A and C (A[d], C[d] point at the block's first row, in host
 * memory) and B[d] is a host copy of the whole B (the same pointer may serve
 * several local devices). In strict mode with K >= 512 each rank uploads only
 * its 1/nranks of every k-phase's B rows, and the ranks broadcast their slices
 * to one another over NVLink on a comm stream while the previous phase
 * multiplies; otherwise every rank runs mapal_gpu_matmul_f32_host on its block.
 * Collective: every rank calls it with the same site. Results equal the
 * one-device call's rows. */
int mapal_gpu_matmul_f32_host_sharded(MapalGpuCtx* ctx, const MapalTileSite* site,
                                      const float* const* A, const float* const* B, float* const* C,
                                      const uint64_t* m, int mode);

/* Any TileSite: dispatches to the matmul, FIR or conv2d kernel when the record
 * has that shape, else runs the generic one-thread-per-cell site kernel
 * (bit-exact, the rung-0 shape). mode applies to matmul-shaped sites. */
int mapal_gpu_tile_site_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* a,
                            const float* b, float* out, int mode);

/* ---- sharded sites (one pointer per local device, in local-device order) ----
 * Partitioning is contiguous and equal up to one unit (mapal_gpu_shard_range).
 * In a multi-process context each process passes arrays of length 1. */

/* Range [lo, hi) of `n` units owned by global rank r of `nranks`. */
int mapal_gpu_shard_range(uint64_t n, int nranks, int r, uint64_t* lo, uint64_t* hi);

/* saxpy over contiguous shards; n[d] elements on local device d. No collective. */
int mapal_gpu_saxpy_sharded(MapalGpuCtx* ctx, float a, const float* const* x,
                            const float* const* y0, float* const* y, const uint64_t* n);

/* Sum over contiguous shards: one f64 partial per rank; every local device
 * receives the f32 result seed + (sum of the partials) in out[d]. The
 * partials are combined inside the fold kernel over peer memory (each rank
 * stores its partial into every rank's exchange block; the sum is taken in
 * rank order, so every rank holds the same value); when some rank cannot map
 * its peers (or MAPAL_GPU_PEER_COMBINE=0), by an NCCL all-reduce instead. The
 * first call on a multi-rank context is collective setup (IPC handles
 * all-gathered over NCCL). A rank whose peers do not publish within 10 s
 * (MAPAL_GPU_PEER_WAIT_MS, read at that setup) returns MAPAL_ERR_TIMEOUT. Replaces the CUDA backend's one-thread fold
 * (crates/backends/cuda/src/kernel.rs:1484-1642) for a sharded array. */
int mapal_gpu_fold_sum_f32_sharded(MapalGpuCtx* ctx, float seed, const float* const* x,
                                   const uint64_t* n, float* const* out);

/* How the context's sharded sum combines partials: 0 = not decided yet (no
 * sharded sum called), 1 = over peer memory in the fold kernel, -1 = NCCL
 * all-reduce (one rank, or peers not mappable). */
int mapal_gpu_ctx_sum_combine(MapalGpuCtx* ctx, int* mode);

/* Broadcast n floats from global rank `root` into buf[d] on every device. */
int mapal_gpu_broadcast_f32(MapalGpuCtx* ctx, float* const* buf, uint64_t n, int root);

/* Gather with idx sharded and x replicated: x[d] holds n_x floats on every
 * device (replicate it first with mapal_gpu_broadcast_f32). */
int mapal_gpu_gather_sharded(MapalGpuCtx* ctx, const float* const* x, uint64_t n_x,
                             const int32_t* const* idx, float* const* out, const uint64_t* n);

/* Row-block matmul: device d holds its row block A[d] (m[d] rows x K) and a
 * full B buffer B[d]; B on global rank `root` is broadcast to all B[d] first
 * (NCCL), then each device computes C[d] = A[d] * B. site describes the full
 * problem (rows = total M). In strict mode over several ranks with K >= 512
 * the broadcast runs in k-ranges overlapped with the multiply of the previous
 * range; strict mode stays bit-exact, as each cell's k order is untouched by
 * the row split and the ranges. */
int mapal_gpu_matmul_f32_sharded(MapalGpuCtx* ctx, const MapalTileSite* site,
                                 const float* const* A, float* const* B, float* const* C,
                                 const uint64_t* m, int root, int mode);

/* ---- measurement --------------------------------------------------------------
 * No counterpart in the reference: the roofline of MAPAL_MATMUL_TF32X3.
 * Issues the 3xTF32 GEMM's own tensor-core instruction (tcgen05.mma M128 N256,
 * operands K-major with the 64-byte swizzle in shared memory, f32 accumulator
 * in tensor memory) back to back with no memory traffic: one CTA per SM,
 * `iters` rounds of 6 MMAs, one warm-up launch and one timed launch on local
 * device 0's stream. kind 0 = kind::tf32 (K8), kind 1 = kind::f16 with bf16
 * operands (K16), which checks the method against a bf16 GEMM's rate, kind 2
 * = kind::tf32 with B MN-major (the layout the GEMM reads B in place with).
 * *tflops receives the dense rate (2 flops per multiply-add). */
int mapal_gpu_probe_mma_peak(MapalGpuCtx* ctx, int kind, uint32_t iters, double* tflops);

/* No counterpart in the reference: the floor under the 2^20-element sites.
 * kind 0 launches an empty kernel; kind 1 reads x (n floats, n a multiple of
 * 4, 16-byte aligned) with the sum fold's own grid and loads but no combine
 * across blocks; kind 2 makes n independent 4-byte reads of x at hashed
 * positions in [0, n) (the gather's bound: random reads, no index array, no
 * output). `sink`, a device float, is written only to keep the loads.
 * Enqueued on local device 0's stream; time it as the sites are timed. */
int mapal_gpu_probe_launch_floor(MapalGpuCtx* ctx, int kind, const float* x, uint64_t n, float* sink);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MAPAL_GPU_H */
