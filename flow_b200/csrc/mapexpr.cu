// mapexpr.cu — the general map body: a per-element stack program.
//
// The reference generates a device function per map body (DevEmit,
// crates/backends/cuda/src/kernel.rs:1712-2936) and runs it one thread per
// element (kernel.rs:1156-1333). This library has fixed kernels, so a map body
// that is not one of the recognized site shapes arrives as a short program of
// scalar ops (include/mapal_gpu.h, MAPAL_X_*) and this kernel evaluates it for
// every element. The program sits in the kernel's parameter space, so every
// thread reads the same op from the constant cache; the value stack lives in
// registers / local memory. Arithmetic follows eval.rs:544-596: wrapping i32
// (div/rem by zero trap div_zero, MIN / -1 wraps), IEEE binary32 with every op
// rounded on its own (__fadd_rn & co. never contract), fmodf for f32 %.
#include <math.h>

#include "common.cuh"

namespace {

constexpr int kMaxStack = 16;

struct ExprProgram {
  MapalExprOp ops[MAPAL_X_MAX_OPS];
  const void* arrays[MAPAL_X_MAX_ARRAYS];
  uint64_t lens[MAPAL_X_MAX_ARRAYS];
  uint32_t nops;
};

__device__ __forceinline__ int32_t wrap_div(int32_t a, int32_t b) { return (a == INT32_MIN && b == -1) ? a : a / b; }
__device__ __forceinline__ int32_t wrap_rem(int32_t a, int32_t b) { return b == -1 ? 0 : a % b; }

__global__ void map_expr_kernel(const __grid_constant__ ExprProgram p, void* __restrict__ out, uint64_t n,
                                unsigned* trap) {
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t st[kMaxStack];
    int sp = 0;
    unsigned kind = 0;  // trap kind + 1
    for (uint32_t pc = 0; pc < p.nops && !kind; ++pc) {
      const MapalExprOp op = p.ops[pc];
      switch (op.code) {
        case MAPAL_X_T_I32: st[sp++] = (uint32_t)t; break;
        case MAPAL_X_CONST_I32: st[sp++] = (uint32_t)op.i; break;
        case MAPAL_X_CONST_F32: st[sp++] = __float_as_uint(op.f); break;
        case MAPAL_X_IN_I32:
        case MAPAL_X_IN_F32: st[sp++] = __ldg(static_cast<const uint32_t*>(p.arrays[op.slot]) + t); break;
        case MAPAL_X_LOAD_I32:
        case MAPAL_X_LOAD_F32: {
          const int64_t j = (int64_t)(int32_t)st[sp - 1];
          if (j < 0 || (uint64_t)j >= p.lens[op.slot]) {
            kind = 2;  // index_oob
            break;
          }
          st[sp - 1] = __ldg(static_cast<const uint32_t*>(p.arrays[op.slot]) + j);
          break;
        }
        case MAPAL_X_NEG_I32: st[sp - 1] = (uint32_t)(0u - st[sp - 1]); break;
        case MAPAL_X_NEG_F32: st[sp - 1] = __float_as_uint(-__uint_as_float(st[sp - 1])); break;
        case MAPAL_X_WIDEN_I32_F32: st[sp - 1] = __float_as_uint(__int2float_rn((int32_t)st[sp - 1])); break;
        case MAPAL_X_STORE_I32:
        case MAPAL_X_STORE_F32: static_cast<uint32_t*>(out)[t] = st[--sp]; break;
        default: {
          // binary ops: b on top, a below
          const uint32_t bb = st[--sp], aa = st[sp - 1];
          const int32_t ai = (int32_t)aa, bi = (int32_t)bb;
          const float af = __uint_as_float(aa), bf = __uint_as_float(bb);
          uint32_t r = 0;
          switch (op.code) {
            case MAPAL_X_ADD_I32: r = aa + bb; break;
            case MAPAL_X_SUB_I32: r = aa - bb; break;
            case MAPAL_X_MUL_I32: r = aa * bb; break;
            case MAPAL_X_DIV_I32:
              if (bi == 0) kind = 1; else r = (uint32_t)wrap_div(ai, bi);
              break;
            case MAPAL_X_REM_I32:
              if (bi == 0) kind = 1; else r = (uint32_t)wrap_rem(ai, bi);
              break;
            case MAPAL_X_ADD_F32: r = __float_as_uint(__fadd_rn(af, bf)); break;
            case MAPAL_X_SUB_F32: r = __float_as_uint(__fsub_rn(af, bf)); break;
            case MAPAL_X_MUL_F32: r = __float_as_uint(__fmul_rn(af, bf)); break;
            case MAPAL_X_DIV_F32: r = __float_as_uint(__fdiv_rn(af, bf)); break;
            case MAPAL_X_REM_F32: r = __float_as_uint(fmodf(af, bf)); break;
            default: kind = 3; break;  // unreachable: the host verified every code
          }
          st[sp - 1] = r;
          break;
        }
      }
    }
    if (kind) atomicMax(trap, kind);
  }
}

// Host check: every op known, operand types consistent, stack within bounds,
// slots in range, exactly one store and it is last. Types: 0 = i32, 1 = f32.
int verify(const MapalExprOp* prog, uint32_t nops, uint32_t narrays) {
  if (nops == 0 || nops > MAPAL_X_MAX_OPS) return set_error(MAPAL_ERR_INVALID, "program length out of range");
  int ty[kMaxStack];
  int sp = 0;
  auto bad = [](const char* m) { return set_error(MAPAL_ERR_INVALID, std::string("map program: ") + m); };
  for (uint32_t pc = 0; pc < nops; ++pc) {
    const MapalExprOp& op = prog[pc];
    const bool last = pc + 1 == nops;
    switch (op.code) {
      case MAPAL_X_T_I32:
      case MAPAL_X_CONST_I32:
      case MAPAL_X_CONST_F32:
      case MAPAL_X_IN_I32:
      case MAPAL_X_IN_F32:
        if ((op.code == MAPAL_X_IN_I32 || op.code == MAPAL_X_IN_F32) && op.slot >= narrays) return bad("slot");
        if (sp >= kMaxStack) return bad("stack overflow");
        ty[sp++] = (op.code == MAPAL_X_CONST_F32 || op.code == MAPAL_X_IN_F32) ? 1 : 0;
        break;
      case MAPAL_X_LOAD_I32:
      case MAPAL_X_LOAD_F32:
        if (op.slot >= narrays) return bad("slot");
        if (sp < 1 || ty[sp - 1] != 0) return bad("load index must be i32");
        ty[sp - 1] = op.code == MAPAL_X_LOAD_F32 ? 1 : 0;
        break;
      case MAPAL_X_NEG_I32:
      case MAPAL_X_NEG_F32:
        if (sp < 1 || ty[sp - 1] != (op.code == MAPAL_X_NEG_F32 ? 1 : 0)) return bad("neg type");
        break;
      case MAPAL_X_WIDEN_I32_F32:
        if (sp < 1 || ty[sp - 1] != 0) return bad("widen takes i32");
        ty[sp - 1] = 1;
        break;
      case MAPAL_X_ADD_I32: case MAPAL_X_SUB_I32: case MAPAL_X_MUL_I32: case MAPAL_X_DIV_I32:
      case MAPAL_X_REM_I32: case MAPAL_X_ADD_F32: case MAPAL_X_SUB_F32: case MAPAL_X_MUL_F32:
      case MAPAL_X_DIV_F32: case MAPAL_X_REM_F32: {
        const int want = op.code >= MAPAL_X_ADD_F32 ? 1 : 0;
        if (sp < 2 || ty[sp - 1] != want || ty[sp - 2] != want) return bad("binary operand types");
        --sp;
        break;
      }
      case MAPAL_X_STORE_I32:
      case MAPAL_X_STORE_F32:
        if (!last) return bad("store must be the last op");
        if (sp != 1 || ty[0] != (op.code == MAPAL_X_STORE_F32 ? 1 : 0)) return bad("store type or leftover stack");
        --sp;
        break;
      default: return bad("unknown op");
    }
    if (last && op.code != MAPAL_X_STORE_I32 && op.code != MAPAL_X_STORE_F32) return bad("missing store");
  }
  return 0;
}

}  // namespace

extern "C" int mapal_gpu_map_expr(MapalGpuCtx* ctx, const MapalExprOp* prog, uint32_t nops,
                                  const void* const* arrays, const uint64_t* lens, uint32_t narrays, void* out,
                                  uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (!prog) return set_error(MAPAL_ERR_INVALID, "program is null");
  if (narrays > MAPAL_X_MAX_ARRAYS || (narrays && (!arrays || !lens)))
    return set_error(MAPAL_ERR_INVALID, "bad array table");
  MAPAL_TRY(verify(prog, nops, narrays));
  if (n == 0) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  if (n > (1ull << 31)) return set_error(MAPAL_ERR_UNSUPPORTED, "index domain beyond i32");
  ExprProgram p{};
  for (uint32_t i = 0; i < nops; ++i) p.ops[i] = prog[i];
  p.nops = nops;
  for (uint32_t s = 0; s < narrays; ++s) {
    p.arrays[s] = arrays[s];
    p.lens[s] = lens[s];
    if (!arrays[s] && lens[s]) return set_error(MAPAL_ERR_INVALID, "null array");
  }
  // IN ops read arrays[s][t] for every t < n: each such array must hold n.
  for (uint32_t i = 0; i < nops; ++i)
    if ((prog[i].code == MAPAL_X_IN_I32 || prog[i].code == MAPAL_X_IN_F32) && lens[prog[i].slot] < n)
      return set_error(MAPAL_ERR_INVALID, "a mapped input is shorter than the domain");
  DeviceSlot& d = ctx->dev[0];
  map_expr_kernel<<<stream_grid(n, 256, d.prof.sm_count, 8), 256, 0, d.stream>>>(p, out, n, d.trap);
  count_launch();
  return finish(ctx, 0, true);
}
