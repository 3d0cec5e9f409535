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
constexpr int kE = 4;         // elements per thread, advanced together op by op
constexpr int kThreads = 256;
// Internal form: a constant immediately followed by a binary op is folded
// into the op (kImm + code, right operand in the op's immediate), so the
// common "x * 7 + 13" shapes never touch the value stack.
constexpr uint16_t kImm = 100;

struct ExprProgram {
  MapalExprOp ops[MAPAL_X_MAX_OPS];
  const void* arrays[MAPAL_X_MAX_ARRAYS];
  uint64_t lens[MAPAL_X_MAX_ARRAYS];
  uint32_t nops;
};

__device__ __forceinline__ int32_t wrap_div(int32_t a, int32_t b) { return (a == INT32_MIN && b == -1) ? a : a / b; }
__device__ __forceinline__ int32_t wrap_rem(int32_t a, int32_t b) { return b == -1 ? 0 : a % b; }

// a OP b for a binary op code; *kind gets 1 (div_zero + 1) on a zero divisor.
__device__ __forceinline__ uint32_t binop(uint16_t code, uint32_t aa, uint32_t bb, unsigned* kind) {
  const int32_t ai = (int32_t)aa, bi = (int32_t)bb;
  const float af = __uint_as_float(aa), bf = __uint_as_float(bb);
  switch (code) {
    case MAPAL_X_ADD_I32: return aa + bb;
    case MAPAL_X_SUB_I32: return aa - bb;
    case MAPAL_X_MUL_I32: return aa * bb;
    case MAPAL_X_DIV_I32:
      if (bi == 0) { *kind = 1; return 0u; }
      return (uint32_t)wrap_div(ai, bi);
    case MAPAL_X_REM_I32:
      if (bi == 0) { *kind = 1; return 0u; }
      return (uint32_t)wrap_rem(ai, bi);
    case MAPAL_X_ADD_F32: return __float_as_uint(__fadd_rn(af, bf));
    case MAPAL_X_SUB_F32: return __float_as_uint(__fsub_rn(af, bf));
    case MAPAL_X_MUL_F32: return __float_as_uint(__fmul_rn(af, bf));
    case MAPAL_X_DIV_F32: return __float_as_uint(__fdiv_rn(af, bf));
    default: return __float_as_uint(fmodf(af, bf));  // MAPAL_X_REM_F32 (the host verified every code)
  }
}

// Each thread advances kE elements, kThreads apart, through the program: the
// op decode is shared by the elements, the top of the stack lives in
// registers, and only deeper stack slots go to local memory. An element that
// traps keeps its first trap kind, skips its later loads and is not stored.
__global__ void __launch_bounds__(kThreads) map_expr_kernel(const __grid_constant__ ExprProgram p,
                                                           void* __restrict__ out, uint64_t n, unsigned* trap) {
  const uint64_t chunk = (uint64_t)kE * kThreads;
  unsigned worst = 0;
  for (uint64_t base = blockIdx.x * chunk; base < n; base += (uint64_t)gridDim.x * chunk) {
    uint64_t tt[kE];
    bool ok[kE];  // in the domain and not trapped
    unsigned kind[kE];
    uint32_t tos[kE];
    uint32_t st[kMaxStack][kE];
#pragma unroll
    for (int e = 0; e < kE; ++e) {
      tt[e] = base + (uint64_t)e * kThreads + threadIdx.x;
      ok[e] = tt[e] < n;
      kind[e] = 0;
      tos[e] = 0;
    }
    int depth = 0;  // values on the stack, the top one in tos
    for (uint32_t pc = 0; pc < p.nops; ++pc) {
      const MapalExprOp op = p.ops[pc];
      if (op.code <= MAPAL_X_IN_F32) {  // pushes
        if (depth > 0) {
#pragma unroll
          for (int e = 0; e < kE; ++e) st[depth - 1][e] = tos[e];
        }
        ++depth;
#pragma unroll
        for (int e = 0; e < kE; ++e) {
          switch (op.code) {
            case MAPAL_X_T_I32: tos[e] = (uint32_t)tt[e]; break;
            case MAPAL_X_CONST_I32: tos[e] = (uint32_t)op.i; break;
            case MAPAL_X_CONST_F32: tos[e] = __float_as_uint(op.f); break;
            default:  // IN: slot verified on the host, and the array holds >= n elements
              tos[e] = ok[e] ? __ldg(static_cast<const uint32_t*>(p.arrays[op.slot]) + tt[e]) : 0u;
              break;
          }
        }
        continue;
      }
      switch (op.code) {
        case MAPAL_X_LOAD_I32:
        case MAPAL_X_LOAD_F32: {
          const uint32_t* src = static_cast<const uint32_t*>(p.arrays[op.slot]);
          const uint64_t len = p.lens[op.slot];
#pragma unroll
          for (int e = 0; e < kE; ++e) {
            const int64_t j = (int64_t)(int32_t)tos[e];
            uint32_t v = 0;
            if (ok[e]) {
              if (j < 0 || (uint64_t)j >= len) {
                kind[e] = 2;  // index_oob
                ok[e] = false;
              } else {
                v = __ldg(src + j);
              }
            }
            tos[e] = v;
          }
          break;
        }
        case MAPAL_X_NEG_I32:
#pragma unroll
          for (int e = 0; e < kE; ++e) tos[e] = 0u - tos[e];
          break;
        case MAPAL_X_NEG_F32:
#pragma unroll
          for (int e = 0; e < kE; ++e) tos[e] ^= 0x80000000u;
          break;
        case MAPAL_X_WIDEN_I32_F32:
#pragma unroll
          for (int e = 0; e < kE; ++e) tos[e] = __float_as_uint(__int2float_rn((int32_t)tos[e]));
          break;
        case MAPAL_X_STORE_I32:
        case MAPAL_X_STORE_F32:
#pragma unroll
          for (int e = 0; e < kE; ++e)
            if (ok[e]) static_cast<uint32_t*>(out)[tt[e]] = tos[e];
          break;
        default:
          if (op.code >= kImm) {  // tos OP immediate
            const uint16_t code = op.code - kImm;
            const uint32_t imm = code >= MAPAL_X_ADD_F32 ? __float_as_uint(op.f) : (uint32_t)op.i;
#pragma unroll
            for (int e = 0; e < kE; ++e) {
              unsigned k = 0;
              tos[e] = binop(code, tos[e], imm, &k);
              if (k && ok[e]) {
                kind[e] = k;
                ok[e] = false;
              }
            }
          } else {  // st[depth-2] OP tos
            --depth;
#pragma unroll
            for (int e = 0; e < kE; ++e) {
              unsigned k = 0;
              tos[e] = binop(op.code, st[depth - 1][e], tos[e], &k);
              if (k && ok[e]) {
                kind[e] = k;
                ok[e] = false;
              }
            }
          }
          break;
      }
    }
#pragma unroll
    for (int e = 0; e < kE; ++e) worst = kind[e] > worst ? kind[e] : worst;
  }
  if (worst) atomicMax(trap, worst);
}

bool is_binary(uint16_t c) {
  return (c >= MAPAL_X_ADD_I32 && c <= MAPAL_X_REM_I32) || (c >= MAPAL_X_ADD_F32 && c <= MAPAL_X_REM_F32);
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
  uint32_t m = 0;
  for (uint32_t i = 0; i < nops; ++i) {
    const uint16_t c = prog[i].code;
    const bool is_const = c == MAPAL_X_CONST_I32 || c == MAPAL_X_CONST_F32;
    if (is_const && i + 1 < nops && is_binary(prog[i + 1].code)) {
      p.ops[m] = prog[i + 1];
      p.ops[m].code = (uint16_t)(kImm + prog[i + 1].code);
      p.ops[m].i = prog[i].i;
      p.ops[m].f = prog[i].f;
      ++m;
      ++i;
    } else {
      p.ops[m++] = prog[i];
    }
  }
  p.nops = m;
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
  map_expr_kernel<<<stream_grid((n + kE - 1) / kE, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(
      p, out, n, d.trap);
  count_launch();
  return finish(ctx, 0, true);
}
