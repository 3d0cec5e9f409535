// mapal_run.cpp — run a Mapal program's `main` with every bulk site on the GPU.
//
//   mapal-run [--device D] [--gpus N] [--plan] [--fast-fold] [--tf32x3] [--no-fuse] program.mapal
//
// The reference compiles a program to CUDA C++ (`emit`, crates/backends/cuda/
// src/lib.rs:72-111) and the emitted `main` launches one generated kernel per
// bulk site, prints through mapal-rt and exits 101 on a trap, 102 on an
// infrastructure failure (module.rs:61-95). This driver is the same contract on
// libmapal_gpu: it reads the bench subset of the language, evaluates `main`
// statement by statement, and hands every bulk site to the C ABI:
//
//   N -> iota                          an index domain (never materialised)
//   dom -> map { t -> body }           a recognised site (matmul / FIR / conv
//                                      tile sites, move sites, gather, saxpy,
//                                      the affine integer generator) or else
//                                      the general map body program
//   (x, y) -> zip -> map { p -> ... }  zipped inputs
//   (seed, xs) -> fold { acc, v -> acc + v }   the sum fold (f32 or i32)
//   a -> enumerate -> map { p -> ... }        index-element pairs
//   a[i] -> println, "text" -> print, () -> time, scalar arithmetic
//   (x, y) -> helper -> z              a counted-loop helper, lifted into a
//                                      map (and the fold helpers it calls)
//
// Scalars live on the host; arrays live on the device. Printing goes through
// mapal_print_* (Rust Display text, as mapal-rt/src/lib.rs:27-60), traps
// through mapal_trap (exit 101); infrastructure errors exit 102 and programs
// outside the subset are refused with exit 2 (EmitError::Unsupported).
// --plan reads the program and prints the site calls it would make, without a
// GPU (arrays are then shapes only). Top-level f32 sum folds run in the
// interpreter's order (bit-exact stdout); --fast-fold takes the bandwidth-bound
// reordered tree instead, whose result is within its stated tolerance.
// --gpus N partitions matmul sites across N devices (row blocks, B broadcast);
// every other site runs on the first device. --tf32x3 runs matmul-shaped
// sites on the tensor cores (3xTF32, within its stated tolerance) for programs
// whose precision contract allows it; the default stays strict.
// A general map body that cannot trap is deferred (elem_plan's `Apply`,
// crates/mapal-ir/src/algo.rs:451-475): a consumer map recomputes it in its own
// program, and its array is written only when something else reads it or a
// clock read comes while it is live. --no-fuse writes every map site's array.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <unistd.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cmath>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "../../include/mapal_gpu.h"
#include "../../include/mapal_rt.h"

namespace {

// ---- failure classes -------------------------------------------------------------

[[noreturn]] void unsupported(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  fflush(stdout);
  fprintf(stderr, "mapal-run: unsupported: ");
  vfprintf(stderr, fmt, ap);
  fprintf(stderr, "\n");
  va_end(ap);
  exit(2);
}

[[noreturn]] void infra(const std::string& what) {
  fflush(stdout);
  fprintf(stderr, "mapal-run infra error: %s\n", what.c_str());
  exit(102);
}

void check(int rc, const char* what) {
  if (rc == MAPAL_OK) return;
  if (rc == MAPAL_TRAP_DIV_ZERO) mapal_trap(0);
  if (rc == MAPAL_TRAP_INDEX_OOB) mapal_trap(1);
  infra(std::string(what) + ": " + mapal_gpu_last_error());
}

// While alive, anything written to stdout goes to stderr: NCCL prints its
// version banner on stdout at communicator set-up, and the program's stdout
// must hold exactly what the program prints.
struct StdoutToStderr {
  int saved;
  StdoutToStderr() {
    fflush(stdout);
    saved = dup(1);
    dup2(2, 1);
  }
  ~StdoutToStderr() {
    fflush(stdout);
    if (saved >= 0) {
      dup2(saved, 1);
      close(saved);
    }
  }
};

// ---- lexer -----------------------------------------------------------------------------

enum Tok { T_EOF, T_IDENT, T_INT, T_FLOAT, T_STR, T_ARROW, T_LBRACE, T_RBRACE, T_LPAREN, T_RPAREN, T_LBRACK,
           T_RBRACK, T_COMMA, T_SEMI, T_COLON, T_DOT, T_PLUS, T_MINUS, T_STAR, T_SLASH, T_PERCENT, T_LT, T_LARROW,
           T_OTHER };

struct Token {
  Tok k;
  std::string s;
  int line;
};

std::vector<Token> lex(const std::string& src) {
  std::vector<Token> out;
  size_t i = 0;
  int line = 1;
  while (i < src.size()) {
    char c = src[i];
    if (c == '\n') { ++line; ++i; continue; }
    if (isspace((unsigned char)c)) { ++i; continue; }
    if (c == '/' && i + 1 < src.size() && src[i + 1] == '/') {
      while (i < src.size() && src[i] != '\n') ++i;
      continue;
    }
    if (isalpha((unsigned char)c) || c == '_') {
      size_t j = i;
      while (j < src.size() && (isalnum((unsigned char)src[j]) || src[j] == '_')) ++j;
      out.push_back({T_IDENT, src.substr(i, j - i), line});
      i = j;
      continue;
    }
    if (isdigit((unsigned char)c)) {
      size_t j = i;
      bool fl = false;
      while (j < src.size() && isdigit((unsigned char)src[j])) ++j;
      // a '.' followed by a digit makes a float; `p.0` projections never start with a digit
      if (j + 1 < src.size() && src[j] == '.' && isdigit((unsigned char)src[j + 1])) {
        fl = true;
        ++j;
        while (j < src.size() && isdigit((unsigned char)src[j])) ++j;
      }
      out.push_back({fl ? T_FLOAT : T_INT, src.substr(i, j - i), line});
      i = j;
      continue;
    }
    if (c == '"') {
      size_t j = i + 1;
      std::string s;
      while (j < src.size() && src[j] != '"') {
        if (src[j] == '\\' && j + 1 < src.size()) {
          char e = src[j + 1];
          s += e == 'n' ? '\n' : e == 't' ? '\t' : e;
          j += 2;
        } else {
          s += src[j++];
        }
      }
      out.push_back({T_STR, s, line});
      i = j + 1;
      continue;
    }
    if (c == '-' && i + 1 < src.size() && src[i + 1] == '>') {
      out.push_back({T_ARROW, "->", line});
      i += 2;
      continue;
    }
    if (c == '<' && i + 1 < src.size() && src[i + 1] == '-') {
      out.push_back({T_LARROW, "<-", line});
      i += 2;
      continue;
    }
    Tok k = T_OTHER;
    switch (c) {
      case '{': k = T_LBRACE; break;
      case '}': k = T_RBRACE; break;
      case '(': k = T_LPAREN; break;
      case ')': k = T_RPAREN; break;
      case '[': k = T_LBRACK; break;
      case ']': k = T_RBRACK; break;
      case ',': k = T_COMMA; break;
      case ';': k = T_SEMI; break;
      case ':': k = T_COLON; break;
      case '.': k = T_DOT; break;
      case '+': k = T_PLUS; break;
      case '-': k = T_MINUS; break;
      case '*': k = T_STAR; break;
      case '/': k = T_SLASH; break;
      case '%': k = T_PERCENT; break;
      case '<': k = T_LT; break;
      default: break;
    }
    out.push_back({k, std::string(1, c), line});
    ++i;
  }
  out.push_back({T_EOF, "", line});
  return out;
}

// ---- syntax tree ------------------------------------------------------------------------

struct Chain;

struct Expr {
  enum K { INT, FLOAT, STR, NAME, UNIT, TUPLE, ARRAY, INDEX, PROJ, BIN, NEG } k;
  long long ival = 0;
  double fval = 0;
  std::string s;  // name / string / float text
  char op = 0;
  std::vector<std::shared_ptr<Expr>> kids;
};
using EP = std::shared_ptr<Expr>;

struct Lambda {
  std::vector<std::string> params;
  std::vector<Chain> stmts;  // the value is the last statement's
};

struct Stage {
  enum K { NAMED, MAP, FOLD } k;
  std::string name;  // builtin, function or binding name
  std::shared_ptr<Lambda> lam;
};

struct Chain {
  EP head;
  std::vector<Stage> stages;
  int line = 0;
};

// A helper function in the counted-loop form the reference lifts into a
// Fold or a Map (crates/mapal-rewrite/src/lift.rs:1-12):
//   mut CTR: i32 <- 0; mut X: T <- init;
//   loop { (CTR < K) -> { -true-> { stmts; CTR + 1 -> CTR; -> loop; } -false-> X -> ret; } }
struct LoopStmt {
  enum K { BIND, UPDATE } k;
  Chain chain;       // BIND: `expr [-> f] -> name`
  EP target, value;  // UPDATE: `target[idx] <- value` (target is the INDEX expression)
};

struct FnDef {
  std::string name;
  std::vector<std::string> params;
  struct Mut {
    std::string name;
    long long arr_len = -1;  // array length from the type, -1 for a scalar
    EP init;
  };
  std::vector<Mut> muts;
  EP cond_lhs, cond_rhs;        // (cond_lhs < cond_rhs)
  std::vector<LoopStmt> body;   // the true branch, without `-> loop`
  EP ret;                       // the false branch's value
  int line = 0;
};

struct Parser {
  std::vector<Token> t;
  size_t p = 0;
  std::map<std::string, FnDef> fns;

  const Token& cur() const { return t[p]; }
  bool at(Tok k) const { return t[p].k == k; }
  Token take(Tok k, const char* what) {
    if (!at(k)) unsupported("line %d: expected %s, found '%s'", cur().line, what, cur().s.c_str());
    return t[p++];
  }

  EP primary() {
    auto e = std::make_shared<Expr>();
    if (at(T_INT)) {
      e->k = Expr::INT;
      e->ival = atoll(t[p++].s.c_str());
    } else if (at(T_FLOAT)) {
      e->k = Expr::FLOAT;
      e->s = t[p].s;
      e->fval = atof(t[p++].s.c_str());
    } else if (at(T_STR)) {
      e->k = Expr::STR;
      e->s = t[p++].s;
    } else if (at(T_IDENT)) {
      e->k = Expr::NAME;
      e->s = t[p++].s;
    } else if (at(T_LPAREN)) {
      ++p;
      if (at(T_RPAREN)) {
        ++p;
        e->k = Expr::UNIT;
      } else {
        EP first = expr();
        if (at(T_COMMA)) {
          e->k = Expr::TUPLE;
          e->kids.push_back(first);
          while (at(T_COMMA)) {
            ++p;
            e->kids.push_back(expr());
          }
          take(T_RPAREN, "')'");
        } else {
          take(T_RPAREN, "')'");
          e = first;
        }
      }
    } else if (at(T_LBRACK)) {
      ++p;
      e->k = Expr::ARRAY;
      if (!at(T_RBRACK)) {
        e->kids.push_back(expr());
        while (at(T_COMMA)) {
          ++p;
          if (at(T_RBRACK)) break;
          e->kids.push_back(expr());
        }
      }
      take(T_RBRACK, "']'");
    } else {
      unsupported("line %d: unexpected '%s'", cur().line, cur().s.c_str());
    }
    // postfix: index and tuple projection
    for (;;) {
      if (at(T_LBRACK)) {
        ++p;
        auto ix = std::make_shared<Expr>();
        ix->k = Expr::INDEX;
        ix->kids = {e, expr()};
        take(T_RBRACK, "']'");
        e = ix;
      } else if (at(T_DOT) && t[p + 1].k == T_INT) {
        ++p;
        auto pr = std::make_shared<Expr>();
        pr->k = Expr::PROJ;
        pr->ival = atoll(t[p++].s.c_str());
        pr->kids = {e};
        e = pr;
      } else if (at(T_DOT) && t[p + 1].k == T_FLOAT) {
        // `p.0.1` lexes the suffix as a float: not in the subset
        unsupported("line %d: nested projection", cur().line);
      } else {
        break;
      }
    }
    return e;
  }

  EP unary() {
    if (at(T_MINUS)) {
      ++p;
      EP inner = unary();
      if (inner->k == Expr::INT) {  // a negative literal (reaches i32 MIN)
        inner->ival = -inner->ival;
        return inner;
      }
      auto e = std::make_shared<Expr>();
      e->k = Expr::NEG;
      e->kids = {inner};
      return e;
    }
    return primary();
  }

  EP mul() {
    EP e = unary();
    while (at(T_STAR) || at(T_SLASH) || at(T_PERCENT)) {
      auto b = std::make_shared<Expr>();
      b->k = Expr::BIN;
      b->op = t[p++].s[0];
      b->kids = {e, unary()};
      e = b;
    }
    return e;
  }

  EP expr() {
    EP e = mul();
    while (at(T_PLUS) || at(T_MINUS)) {
      auto b = std::make_shared<Expr>();
      b->k = Expr::BIN;
      b->op = t[p++].s[0];
      b->kids = {e, mul()};
      e = b;
    }
    return e;
  }

  void skip_type() {
    // `name: T` annotations: an identifier or a bracketed array type
    if (at(T_LBRACK)) {
      int depth = 0;
      do {
        if (at(T_LBRACK)) ++depth;
        if (at(T_RBRACK)) --depth;
        ++p;
      } while (depth > 0 && !at(T_EOF));
    } else if (at(T_LPAREN)) {
      int depth = 0;
      do {
        if (at(T_LPAREN)) ++depth;
        if (at(T_RPAREN)) --depth;
        ++p;
      } while (depth > 0 && !at(T_EOF));
    } else {
      take(T_IDENT, "type");
    }
  }

  std::shared_ptr<Lambda> lambda() {
    take(T_LBRACE, "'{'");
    auto L = std::make_shared<Lambda>();
    L->params.push_back(take(T_IDENT, "parameter").s);
    while (at(T_COMMA)) {
      ++p;
      L->params.push_back(take(T_IDENT, "parameter").s);
    }
    take(T_ARROW, "'->'");
    L->stmts.push_back(chain());
    while (at(T_SEMI)) {
      ++p;
      if (at(T_RBRACE)) break;
      L->stmts.push_back(chain());
    }
    take(T_RBRACE, "'}'");
    return L;
  }

  Chain chain() {
    Chain c;
    c.line = cur().line;
    c.head = expr();
    while (at(T_ARROW)) {
      ++p;
      Stage s;
      std::string name = take(T_IDENT, "stage").s;
      if (name == "map" || name == "fold") {
        s.k = name == "map" ? Stage::MAP : Stage::FOLD;
        s.lam = lambda();
      } else {
        s.k = Stage::NAMED;
        s.name = name;
        if (at(T_COLON)) {
          ++p;
          skip_type();
        }
      }
      c.stages.push_back(s);
    }
    return c;
  }

  // `name: T` with T a scalar type or `[T; N]`; returns N for arrays, else -1
  long long param_type() {
    if (at(T_LBRACK)) {
      ++p;
      take(T_IDENT, "element type");
      take(T_SEMI, "';'");
      const long long n = atoll(take(T_INT, "array length").s.c_str());
      take(T_RBRACK, "']'");
      return n;
    }
    take(T_IDENT, "type");
    return -1;
  }

  FnDef loop_fn(const std::string& name, int line) {
    FnDef f;
    f.name = name;
    f.line = line;
    take(T_LPAREN, "'('");
    while (!at(T_RPAREN)) {
      f.params.push_back(take(T_IDENT, "parameter").s);
      take(T_COLON, "':'");
      param_type();
      if (at(T_COMMA)) ++p;
    }
    take(T_RPAREN, "')'");
    if (at(T_ARROW)) {
      ++p;
      param_type();
    }
    take(T_LBRACE, "'{'");
    while (at(T_IDENT) && cur().s == "mut") {
      ++p;
      FnDef::Mut m;
      m.name = take(T_IDENT, "name").s;
      take(T_COLON, "':'");
      m.arr_len = param_type();
      take(T_LARROW, "'<-'");
      m.init = expr();
      take(T_SEMI, "';'");
      f.muts.push_back(m);
    }
    auto kw = [&](const char* w) {
      Token k = take(T_IDENT, w);
      if (k.s != w) unsupported("line %d: expected `%s`, found `%s`", k.line, w, k.s.c_str());
    };
    kw("loop");
    take(T_LBRACE, "'{'");
    take(T_LPAREN, "'('");
    f.cond_lhs = expr();
    take(T_LT, "'<' (only counted loops are lifted)");
    f.cond_rhs = expr();
    take(T_RPAREN, "')'");
    take(T_ARROW, "'->'");
    take(T_LBRACE, "'{'");
    take(T_MINUS, "'-true->'");
    kw("true");
    take(T_ARROW, "'->'");
    take(T_LBRACE, "'{'");
    bool cont = false;
    while (!at(T_RBRACE)) {
      if (at(T_ARROW)) {  // -> loop;
        ++p;
        kw("loop");
        take(T_SEMI, "';'");
        cont = true;
        continue;
      }
      if (cont) unsupported("line %d: statements after `-> loop`", cur().line);
      LoopStmt st;
      const size_t save = p;
      EP e = expr();
      if (at(T_LARROW)) {
        if (e->k != Expr::INDEX) unsupported("line %d: `<-` needs an element target", cur().line);
        ++p;
        st.k = LoopStmt::UPDATE;
        st.target = e;
        st.value = expr();
      } else {
        p = save;
        st.k = LoopStmt::BIND;
        st.chain = chain();
      }
      take(T_SEMI, "';'");
      f.body.push_back(st);
    }
    take(T_RBRACE, "'}'");
    if (!cont) unsupported("line %d: the loop's true branch must end with `-> loop`", f.line);
    take(T_MINUS, "'-false->'");
    kw("false");
    take(T_ARROW, "'->'");
    f.ret = expr();
    take(T_ARROW, "'->'");
    kw("ret");
    take(T_SEMI, "';'");
    take(T_RBRACE, "'}'");
    take(T_RBRACE, "'}'");
    take(T_RBRACE, "'}'");
    return f;
  }

  std::vector<Chain> main_body() {
    bool found = false;
    std::vector<Chain> body;
    while (!at(T_EOF)) {
      Token kw = take(T_IDENT, "'fn'");
      if (kw.s != "fn") unsupported("line %d: only `fn` items are in the subset", kw.line);
      std::string name = take(T_IDENT, "function name").s;
      if (name != "main") {
        if (fns.count(name)) unsupported("line %d: `%s` defined twice", kw.line, name.c_str());
        fns[name] = loop_fn(name, kw.line);
        continue;
      }
      take(T_LPAREN, "'('");
      take(T_RPAREN, "')'");
      take(T_LBRACE, "'{'");
      while (!at(T_RBRACE)) {
        body.push_back(chain());
        take(T_SEMI, "';'");
      }
      take(T_RBRACE, "'}'");
      found = true;
    }
    if (!found) unsupported("no fn main");
    return body;
  }

};

// ---- values ------------------------------------------------------------------------------

enum Ty { TY_I32, TY_F32, TY_F64, TY_STR, TY_UNIT, TY_TUPLE, TY_ARR, TY_IOTA, TY_ZIP };

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

struct Lazy;

struct Value {
  Ty ty = TY_UNIT;
  int32_t i = 0;
  float f = 0;
  double d = 0;
  std::string s;
  std::vector<Value> items;     // tuple parts / zip inputs
  Ty elem = TY_F32;             // array element type
  uint64_t n = 0;               // array / iota length
  uint64_t id = 0;              // array identity (also in plan mode)
  std::shared_ptr<DevBuf> buf;  // array storage (absent in plan mode)
  std::shared_ptr<Lazy> lazy;   // a deferred map: materialised on first ptr()
  void* ptr() const;
};

// A map site whose body is trap-free and effect-free, held as its element law
// instead of launched (elem_plan's `Apply`, crates/mapal-ir/src/algo.rs:
// 451-475 and the gate `body_is_classifiable`, :1531-1545). A consumer map
// splices `ops` into its own program and recomputes the element; the array is
// written only if something else reads it (a site that needs the pointer, an
// element read) or a clock read comes while it is still live.
struct Lazy {
  std::vector<MapalExprOp> ops;  // the body, without its store
  std::vector<Value> arrays;     // the body's slot table
  Ty out = TY_F32;
  uint64_t n = 0;
  bool consumed = false;  // spliced into a consumer at least once
  bool done = false;      // materialised into `mat`
  Value mat;
};

// ---- the runner ---------------------------------------------------------------------------

struct Runner {
  const std::map<std::string, FnDef>* fns = nullptr;  // the program's counted-loop helpers
  int gpus = 1;   // devices dev0 .. dev0 + gpus - 1; matmul sites are partitioned across them
  int mm_mode = MAPAL_MATMUL_STRICT;  // --tf32x3: matmul-shaped sites on the tensor cores
  int dev0 = 0;
  int synth = 0;                                       // counter for synthetic names
  bool plan = false;
  bool fast_fold = false;  // the reordered f64 tree instead of the interpreter's order
  MapalGpuCtx* ctx = nullptr;
  std::map<std::string, Value> env;

  uint64_t next_id = 1;

  Value make_array(Ty elem, uint64_t n) {
    Value v;
    v.ty = TY_ARR;
    v.elem = elem;
    v.n = n;
    v.id = next_id++;
    if (!plan && n) {
      v.buf = std::make_shared<DevBuf>();
      cudaError_t e = cudaMalloc(&v.buf->p, n * 4);
      if (e != cudaSuccess) infra(std::string("cudaMalloc: ") + cudaGetErrorString(e));
    }
    return v;
  }

  void say(const std::string& s) {
    if (plan) printf("%s\n", s.c_str());
  }

  // Sites are enqueued without waiting; every host-visible effect (a print,
  // an element read, a clock read) first drains the stream, so a trap in any
  // earlier site ends the program before that effect, as in the interpreter.
  void sync_point() {
    if (!plan) check(mapal_gpu_synchronize(ctx), "synchronize");
  }

  // -- scalar evaluation on the host (eval.rs:544-596 for the arithmetic) --

  static Value num_i32(int32_t x) { Value v; v.ty = TY_I32; v.i = x; return v; }
  static Value num_f32(float x) { Value v; v.ty = TY_F32; v.f = x; return v; }
  static Value num_f64(double x) { Value v; v.ty = TY_F64; v.d = x; return v; }

  static bool is_float_lit(const EP& e) { return e->k == Expr::FLOAT; }

  Value lit_as(const EP& e, Ty want) {
    // a float literal takes the float type its context asks for
    // an f32 literal is parsed directly as f32 (one rounding), as the reference's lowering does
    if (want == TY_F32) return num_f32(strtof(e->s.c_str(), nullptr));
    return num_f64(strtod(e->s.c_str(), nullptr));
  }

  Value scalar_bin(char op, Value a, Value b, int line) {
    if (a.ty != b.ty) unsupported("line %d: mixed operand types", line);
    if (a.ty == TY_I32) {
      uint32_t x = (uint32_t)a.i, y = (uint32_t)b.i;
      switch (op) {
        case '+': return num_i32((int32_t)(x + y));
        case '-': return num_i32((int32_t)(x - y));
        case '*': return num_i32((int32_t)(x * y));
        case '/':
          if (b.i == 0) mapal_trap(0);
          return num_i32(a.i == INT32_MIN && b.i == -1 ? a.i : a.i / b.i);
        case '%':
          if (b.i == 0) mapal_trap(0);
          return num_i32(b.i == -1 ? 0 : a.i % b.i);
      }
    }
    if (a.ty == TY_F32) {
      volatile float x = a.f, y = b.f, r = 0;
      switch (op) {
        case '+': r = x + y; break;
        case '-': r = x - y; break;
        case '*': r = x * y; break;
        case '/': r = x / y; break;
        case '%': r = fmodf(x, y); break;
      }
      return num_f32(r);
    }
    if (a.ty == TY_F64) {
      volatile double x = a.d, y = b.d, r = 0;
      switch (op) {
        case '+': r = x + y; break;
        case '-': r = x - y; break;
        case '*': r = x * y; break;
        case '/': r = x / y; break;
        case '%': r = fmod(x, y); break;
      }
      return num_f64(r);
    }
    unsupported("line %d: arithmetic on a non-number", line);
  }

  Value eval(const EP& e, int line, Ty float_ctx = TY_F64) {
    switch (e->k) {
      case Expr::INT:
        if (e->ival > INT32_MAX || e->ival < INT32_MIN) unsupported("line %d: integer literal beyond i32", line);
        return num_i32((int32_t)e->ival);
      case Expr::FLOAT: return lit_as(e, float_ctx);
      case Expr::STR: { Value v; v.ty = TY_STR; v.s = e->s; return v; }
      case Expr::UNIT: return Value{};
      case Expr::NAME: {
        auto it = env.find(e->s);
        if (it == env.end()) unsupported("line %d: unknown name `%s`", line, e->s.c_str());
        return it->second;
      }
      case Expr::TUPLE: {
        Value v;
        v.ty = TY_TUPLE;
        // float literals in a tuple take the type of the tuple's arrays (fold seeds)
        Ty ctx = float_ctx;
        for (auto& k : e->kids)
          if (k->k == Expr::NAME) {
            Value w = eval(k, line);
            if (w.ty == TY_ARR && w.elem == TY_F32) ctx = TY_F32;
          }
        for (auto& k : e->kids) v.items.push_back(eval(k, line, ctx));
        return v;
      }
      case Expr::ARRAY: return array_literal(e, line);
      case Expr::NEG: {
        Value a = eval(e->kids[0], line, float_ctx);
        if (a.ty == TY_I32) return num_i32((int32_t)(0u - (uint32_t)a.i));
        if (a.ty == TY_F32) return num_f32(-a.f);
        if (a.ty == TY_F64) return num_f64(-a.d);
        unsupported("line %d: negation of a non-number", line);
      }
      case Expr::BIN: {
        const EP &l = e->kids[0], &r = e->kids[1];
        Value a, b;
        if (is_float_lit(l) && !is_float_lit(r)) {
          b = eval(r, line, float_ctx);
          a = lit_as(l, b.ty == TY_F32 ? TY_F32 : TY_F64);
        } else if (is_float_lit(r) && !is_float_lit(l)) {
          a = eval(l, line, float_ctx);
          b = lit_as(r, a.ty == TY_F32 ? TY_F32 : TY_F64);
        } else {
          a = eval(l, line, float_ctx);
          b = eval(r, line, float_ctx);
        }
        return scalar_bin(e->op, a, b, line);
      }
      case Expr::INDEX: {
        Value a = eval(e->kids[0], line);
        Value ix = eval(e->kids[1], line);
        if (ix.ty != TY_I32) unsupported("line %d: index must be i32", line);
        return element(a, ix.i, line);
      }
      case Expr::PROJ: {
        Value a = eval(e->kids[0], line);
        if (a.ty != TY_TUPLE || e->ival >= (long long)a.items.size()) unsupported("line %d: bad projection", line);
        return a.items[e->ival];
      }
    }
    unsupported("line %d: expression", line);
  }

  // One element read, with the Index bounds rule (eval.rs:655-669).
  Value element(const Value& a, int32_t j, int line) {
    if (a.ty == TY_IOTA) {
      if (j < 0 || (uint64_t)j >= a.n) mapal_trap(1);
      return num_i32(j);
    }
    if (a.ty != TY_ARR) unsupported("line %d: indexing a non-array", line);
    if (j < 0 || (uint64_t)j >= a.n) mapal_trap(1);
    if (a.lazy) a.ptr();  // a deferred map is written before its element is read
    if (plan) {
      say("read element " + std::to_string(j));
      return a.elem == TY_I32 ? num_i32(0) : num_f32(0);
    }
    sync_point();
    uint32_t bits = 0;
    cudaError_t err = cudaMemcpy(&bits, (char*)a.ptr() + 4 * (uint64_t)j, 4, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) infra(std::string("cudaMemcpy: ") + cudaGetErrorString(err));
    if (a.elem == TY_I32) return num_i32((int32_t)bits);
    float f;
    memcpy(&f, &bits, 4);
    return num_f32(f);
  }

  Value array_literal(const EP& e, int line) {
    std::vector<Value> xs;
    bool any_float = false;
    for (auto& k : e->kids) {
      xs.push_back(eval(k, line, TY_F32));
      if (xs.back().ty != TY_I32) any_float = true;
    }
    Ty elem = any_float ? TY_F32 : TY_I32;
    Value v = make_array(elem, xs.size());
    std::vector<uint32_t> bits(xs.size());
    for (size_t i = 0; i < xs.size(); ++i) {
      if (elem == TY_F32) {
        float f = xs[i].ty == TY_F32 ? xs[i].f : xs[i].ty == TY_I32 ? (float)xs[i].i : (float)xs[i].d;
        memcpy(&bits[i], &f, 4);
      } else {
        bits[i] = (uint32_t)xs[i].i;
      }
    }
    if (!plan && !xs.empty()) {
      cudaError_t err = cudaMemcpy(v.ptr(), bits.data(), 4 * xs.size(), cudaMemcpyHostToDevice);
      if (err != cudaSuccess) infra(std::string("cudaMemcpy: ") + cudaGetErrorString(err));
    }
    return v;
  }

  // -- statements --

  // Every name a statement mentions (its expressions, stage names and lambda
  // bodies): a superset of the bindings it reads.
  static void names_in(const EP& e, std::set<std::string>& out) {
    if (!e) return;
    if (e->k == Expr::NAME) out.insert(e->s);
    for (auto& k : e->kids) names_in(k, out);
  }
  static void names_in(const Chain& c, std::set<std::string>& out) {
    names_in(c.head, out);
    for (auto& s : c.stages) {
      if (s.k == Stage::NAMED) out.insert(s.name);
      if (s.lam)
        for (auto& st : s.lam->stmts) names_in(st, out);
    }
  }

  // A site about to read an array: a deferred map is written first.
  void need(const Value& v) {
    if (v.lazy && !v.lazy->done) materialise(*v.lazy);
    for (auto& it : v.items) need(it);
  }

  void keep_bufs(const Value& v) {
    if (v.buf) kept.push_back(v.buf);
    if (v.lazy && v.lazy->mat.buf) kept.push_back(v.lazy->mat.buf);
    for (auto& it : v.items) keep_bufs(it);
  }

  // main's statements in order. After each one, the bindings no later
  // statement mentions are released (their device memory is kept until exit),
  // so a deferred map whose only reader recomputed it is never written.
  void run_main(const std::vector<Chain>& body) {
    std::map<std::string, size_t> last;
    for (size_t j = 0; j < body.size(); ++j) {
      std::set<std::string> ns;
      names_in(body[j], ns);
      for (auto& n : ns) last[n] = j;
    }
    for (size_t j = 0; j < body.size(); ++j) {
      run_chain(body[j]);
      for (auto it = env.begin(); it != env.end();) {
        auto l = last.find(it->first);
        if (l != last.end() && l->second > j) {
          ++it;
          continue;
        }
        keep_bufs(it->second);
        it = env.erase(it);
      }
      settle(false);
    }
  }

  void run(const std::vector<Chain>& body) {
    for (auto& c : body) run_chain(c);
  }

  Value run_chain(const Chain& c) {
    Value v = eval(c.head, c.line);
    for (auto& s : c.stages) v = stage(s, v, c.line, c);
    return v;
  }

  Value stage(const Stage& s, const Value& v, int line, const Chain& c) {
    if (s.k == Stage::MAP) return map_site(*s.lam, v, line);
    if (s.k == Stage::FOLD) return fold_site(*s.lam, v, line);
    const std::string& n = s.name;
    if (n == "iota") {
      if (v.ty != TY_I32 || v.i < 0) unsupported("line %d: iota takes a non-negative i32", line);
      Value r;
      r.ty = TY_IOTA;
      r.n = (uint64_t)v.i;
      return r;
    }
    if (n == "zip") {
      if (v.ty != TY_TUPLE || v.items.size() != 2) unsupported("line %d: zip takes a pair", line);
      for (auto& a : v.items)
        if (a.ty != TY_ARR && a.ty != TY_IOTA) unsupported("line %d: zip of non-arrays", line);
      if (v.items[0].n != v.items[1].n) unsupported("line %d: zip of arrays of different lengths", line);
      Value r;
      r.ty = TY_ZIP;
      r.items = v.items;
      r.n = v.items[0].n;
      return r;
    }
    if (n == "enumerate") {  // zip(iota n, a): pairs (index, element)
      if (v.ty != TY_ARR && v.ty != TY_IOTA) unsupported("line %d: enumerate of a non-array", line);
      Value idx;
      idx.ty = TY_IOTA;
      idx.n = v.n;
      Value r;
      r.ty = TY_ZIP;
      r.items = {idx, v};
      r.n = v.n;
      return r;
    }
    if (n == "widen_f32") {
      if (v.ty == TY_I32) return num_f32((float)v.i);
      unsupported("line %d: widen_f32 of a non-i32 scalar", line);
    }
    if (n == "widen_f64") {
      if (v.ty == TY_I32) return num_f64((double)v.i);
      if (v.ty == TY_F32) return num_f64((double)v.f);
      unsupported("line %d: widen_f64", line);
    }
    if (n == "println" || n == "print") {
      print(v, n == "println", line);
      return Value{};
    }
    if (n == "time") {
      // the clock reads after the device drains: the elapsed time between two
      // reads covers the sites launched between them
      settle(true);
      sync_point();
      return num_f64(mapal_time_ms());
    }
    if (fns && fns->count(n)) return call_fn(fns->at(n), v, line);
    // otherwise: a binding
    if (n == "map" || n == "fold") unsupported("line %d: %s without a body", line, n.c_str());
    (void)c;
    env[n] = v;
    return v;
  }

  void print(const Value& v, bool nl, int line) {
    if (plan) {
      say(std::string(nl ? "println" : "print"));
      return;
    }
    sync_point();
    switch (v.ty) {
      case TY_I32: mapal_print_i32(v.i, nl); break;
      case TY_F32: mapal_print_f32(v.f, nl); break;
      case TY_F64: mapal_print_f64(v.d, nl); break;
      case TY_STR: mapal_print_str((const uint8_t*)v.s.data(), v.s.size(), nl); break;
      default: unsupported("line %d: printing a non-scalar", line);
    }
  }

  // -- fold sites --

  Value fold_site(const Lambda& L, const Value& v, int line) {
    // (seed, xs) -> fold { acc, v -> acc + v }: the sum fold
    if (v.ty != TY_TUPLE || v.items.size() != 2) unsupported("line %d: fold takes (seed, array)", line);
    const Value &seed = v.items[0], &xs = v.items[1];
    if (L.params.size() != 2 || L.stmts.size() != 1 || !L.stmts[0].stages.empty())
      unsupported("line %d: fold body outside the subset", line);
    const EP& b = L.stmts[0].head;
    bool is_sum = b->k == Expr::BIN && b->op == '+' && b->kids[0]->k == Expr::NAME &&
                  b->kids[1]->k == Expr::NAME &&
                  ((b->kids[0]->s == L.params[0] && b->kids[1]->s == L.params[1]) ||
                   (b->kids[0]->s == L.params[1] && b->kids[1]->s == L.params[0]));
    if (is_sum && xs.ty == TY_ARR && xs.elem == TY_I32 && seed.ty == TY_I32) {
      // wrapping i32 addition is associative: the parallel fold is exact
      need(xs);
      say("fold_sum_i32 n=" + std::to_string(xs.n));
      if (plan) return num_i32(0);
      int32_t* out = nullptr;
      if (cudaMalloc(&out, 4) != cudaSuccess) infra("cudaMalloc");
      check(mapal_gpu_fold_sum_i32(ctx, seed.i, (const int32_t*)xs.ptr(), xs.n, out), "fold_sum_i32");
      sync_point();
      int32_t r = 0;
      if (cudaMemcpy(&r, out, 4, cudaMemcpyDeviceToHost) != cudaSuccess) infra("cudaMemcpy");
      cudaFree(out);
      return num_i32(r);
    }
    if (!is_sum || xs.ty != TY_ARR || xs.elem != TY_F32 || seed.ty != TY_F32)
      unsupported("line %d: only the f32 and i32 sum folds run at top level", line);
    need(xs);
    say(std::string(fast_fold ? "fold_sum_f32" : "fold_sum_f32_strict") + " n=" + std::to_string(xs.n));
    if (plan) return num_f32(0);
    float* out = nullptr;
    if (cudaMalloc(&out, 4) != cudaSuccess) infra("cudaMalloc");
    if (fast_fold)
      check(mapal_gpu_fold_sum_f32(ctx, seed.f, (const float*)xs.ptr(), xs.n, out), "fold_sum");
    else
      check(mapal_gpu_fold_sum_f32_strict(ctx, seed.f, (const float*)xs.ptr(), xs.n, out), "fold_sum");
    sync_point();
    float r = 0;
    if (cudaMemcpy(&r, out, 4, cudaMemcpyDeviceToHost) != cudaSuccess) infra("cudaMemcpy");
    cudaFree(out);
    return num_f32(r);
  }

  // -- map sites --

  // Substitute the lambda's local bindings (`expr -> name;`) into its final
  // expression; bodies are pure, so inlining keeps the meaning.
  EP inline_locals(const Lambda& L, size_t upto, const EP& e, std::map<std::string, EP>& locals) {
    (void)upto;
    if (e->k == Expr::NAME) {
      auto it = locals.find(e->s);
      if (it != locals.end()) return it->second;
      return e;
    }
    auto c = std::make_shared<Expr>(*e);
    for (auto& k : c->kids) k = inline_locals(L, upto, k, locals);
    return c;
  }

  Value map_site(const Lambda& L, const Value& dom, int line) {
    if (dom.ty != TY_IOTA && dom.ty != TY_ARR && dom.ty != TY_ZIP) unsupported("line %d: map over a non-array", line);
    if (L.params.size() != 1) unsupported("line %d: map takes one parameter", line);
    // local bindings, then the final statement
    std::map<std::string, EP> locals;
    for (size_t k = 0; k + 1 < L.stmts.size(); ++k) {
      const Chain& st = L.stmts[k];
      if (st.stages.size() != 1 || st.stages[0].k != Stage::NAMED) unsupported("line %d: map body statement", line);
      locals[st.stages[0].name] = inline_locals(L, k, st.head, locals);
    }
    const Chain& last = L.stmts.back();
    // tile site: (seed, krange) -> fold { acc, k -> acc + X[..] * Y[..] }
    if (last.stages.size() == 1 && last.stages[0].k == Stage::FOLD) return tile_site(L, dom, locals, last, line);
    EP body = inline_locals(L, 0, last.head, locals);
    bool widen = false;
    for (auto& s : last.stages) {
      if (s.k == Stage::NAMED && s.name == "widen_f32" && !widen) widen = true;
      else unsupported("line %d: map body stage", line);
    }
    // a deferred producer is recomputed inside the general map body rather than
    // written for a specialised kernel to read
    bool deferred_input = dom.lazy && !dom.lazy->done;
    for (auto& it : dom.items) deferred_input |= it.lazy && !it.lazy->done;
    if (!widen && !(fuse_maps && deferred_input)) {
      if (Value r; try_gather(L.params[0], body, dom, r, line)) return r;
      if (Value r; try_move(L.params[0], body, dom, r, line)) return r;
      if (Value r; try_saxpy(L.params[0], body, dom, r, line)) return r;
    } else {
      if (Value r; try_affine_gen(L.params[0], body, dom, r, line)) return r;
    }
    return general_map(L.params[0], body, widen, dom, line);
  }

  // t -> (t * A + B) % M - C -> widen_f32 over an index domain, integer
  // literals with M > 0: the benches' integer generators, one fused kernel.
  bool try_affine_gen(const std::string& prm, const EP& b, const Value& dom, Value& out, int line) {
    (void)line;
    if (dom.ty != TY_IOTA) return false;
    auto lit = [](const EP& e, long long& v) {
      if (e->k != Expr::INT || e->ival < INT32_MIN || e->ival > INT32_MAX) return false;
      v = e->ival;
      return true;
    };
    auto bin = [](const EP& e, char op) { return e->k == Expr::BIN && e->op == op; };
    long long A, B, M, C;
    if (!bin(b, '-') || !lit(b->kids[1], C)) return false;
    const EP& rem = b->kids[0];
    if (!bin(rem, '%') || !lit(rem->kids[1], M) || M <= 0) return false;
    const EP& add = rem->kids[0];
    if (!bin(add, '+') || !lit(add->kids[1], B)) return false;
    const EP& mul = add->kids[0];
    if (!bin(mul, '*')) return false;
    const EP &x = mul->kids[0], &y = mul->kids[1];
    const bool t_first = x->k == Expr::NAME && x->s == prm && lit(y, A);
    const bool t_second = y->k == Expr::NAME && y->s == prm && lit(x, A);
    if (!t_first && !t_second) return false;
    say("gen_affine n=" + std::to_string(dom.n) + " mul=" + std::to_string(A) + " add=" + std::to_string(B) +
        " mod=" + std::to_string(M) + " sub=" + std::to_string(C));
    out = make_array(TY_F32, dom.n);
    if (!plan)
      check(mapal_gpu_gen_affine_f32(ctx, (float*)out.ptr(), dom.n, 0, (int32_t)A, (int32_t)B, (int32_t)M,
                                     (int32_t)C),
            "gen_affine");
    return true;
  }

  // j -> x[j] over an i32 array
  bool try_gather(const std::string& prm, const EP& b, const Value& dom, Value& out, int line) {
    if (dom.ty != TY_ARR || dom.elem != TY_I32 || b->k != Expr::INDEX) return false;
    if (b->kids[0]->k != Expr::NAME || b->kids[1]->k != Expr::NAME || b->kids[1]->s != prm) return false;
    Value x = eval(b->kids[0], line);
    if (x.ty != TY_ARR || x.elem != TY_F32) return false;
    need(x);
    say("gather n=" + std::to_string(dom.n) + " n_x=" + std::to_string(x.n));
    out = make_array(TY_F32, dom.n);
    if (!plan) check(mapal_gpu_gather(ctx, (const float*)x.ptr(), x.n, (const int32_t*)dom.ptr(), (float*)out.ptr(), dom.n), "gather");
    return true;
  }

  // -- affine forms over the index atoms --------------------------------------------

  // atoms: "t", "t/C", "t%C", "k", "k/D", "k%D", "1"
  using Affine = std::map<std::string, long long>;

  static bool atom_of(const EP& e, const std::string& var, std::string& atom) {
    if (e->k == Expr::NAME && e->s == var) {
      atom = var;
      return true;
    }
    if (e->k == Expr::BIN && (e->op == '/' || e->op == '%') && e->kids[0]->k == Expr::NAME &&
        e->kids[0]->s == var && e->kids[1]->k == Expr::INT && e->kids[1]->ival > 0) {
      atom = var + std::string(1, e->op) + std::to_string(e->kids[1]->ival);
      return true;
    }
    return false;
  }

  bool affine(const EP& e, const std::vector<std::string>& vars, Affine& out) {
    std::string a;
    for (auto& v : vars)
      if (atom_of(e, v, a)) {
        out = {{a, 1}};
        return true;
      }
    if (e->k == Expr::INT) {
      out = {{"1", e->ival}};
      return true;
    }
    if (e->k == Expr::BIN && (e->op == '+' || e->op == '-')) {
      Affine x, y;
      if (!affine(e->kids[0], vars, x) || !affine(e->kids[1], vars, y)) return false;
      for (auto& [k, c] : y) x[k] += e->op == '+' ? c : -c;
      out = x;
      return true;
    }
    if (e->k == Expr::BIN && e->op == '*') {
      Affine x, y;
      if (!affine(e->kids[0], vars, x) || !affine(e->kids[1], vars, y)) return false;
      const Affine* cst = (x.size() == 1 && x.count("1")) ? &x : (y.size() == 1 && y.count("1")) ? &y : nullptr;
      if (!cst) return false;
      const Affine& other = cst == &x ? y : x;
      long long c = cst->at("1");
      out.clear();
      for (auto& [k, v] : other) out[k] = v * c;
      return true;
    }
    return false;
  }

  // -- tile sites: algo.rs:949-1079's record, recognised from the source form --

  Value tile_site(const Lambda& L, const Value& dom, std::map<std::string, EP>& locals, const Chain& fc, int line) {
    if (dom.ty != TY_IOTA) unsupported("line %d: tile sites map over an iota domain", line);
    const std::string& t = L.params[0];
    Value pair = eval(fc.head, line, TY_F32);
    if (pair.ty != TY_TUPLE || pair.items.size() != 2 || pair.items[1].ty != TY_IOTA)
      unsupported("line %d: fold over (seed, iota)", line);
    const Value seed = pair.items[0];
    if (seed.ty != TY_F32) unsupported("line %d: fold seed must be f32", line);
    const uint64_t K = pair.items[1].n;
    const Lambda& F = *fc.stages[0].lam;
    if (F.params.size() != 2 || F.stmts.size() != 1 || !F.stmts[0].stages.empty())
      unsupported("line %d: fold body outside the subset", line);
    const std::string &acc = F.params[0], &k = F.params[1];
    EP b = inline_locals(L, 0, F.stmts[0].head, locals);
    if (b->k != Expr::BIN || b->op != '+') unsupported("line %d: fold body must be acc + a * b", line);
    bool add_acc_first = b->kids[0]->k == Expr::NAME && b->kids[0]->s == acc;
    EP prod = add_acc_first ? b->kids[1] : b->kids[0];
    EP accn = add_acc_first ? b->kids[0] : b->kids[1];
    if (accn->k != Expr::NAME || accn->s != acc || prod->k != Expr::BIN || prod->op != '*' ||
        prod->kids[0]->k != Expr::INDEX || prod->kids[1]->k != Expr::INDEX)
      unsupported("line %d: fold body must be acc + X[..] * Y[..]", line);
    EP ra = prod->kids[0], rb = prod->kids[1];
    Value A = eval(ra->kids[0], line), B = eval(rb->kids[0], line);
    if (A.ty != TY_ARR || B.ty != TY_ARR || A.elem != TY_F32 || B.elem != TY_F32)
      unsupported("line %d: tile-site reads must be f32 arrays", line);
    Affine fa, fbb;
    if (!affine(ra->kids[1], {t, k}, fa) || !affine(rb->kids[1], {t, k}, fbb))
      unsupported("line %d: tile-site addresses must be affine in the indices", line);
    // the cell split t = i*c + lane: the divisor the body uses, else a single row
    long long c = 0;
    long long D = 0;
    for (const Affine* f : {&fa, &fbb})
      for (auto& [atom, coef] : *f) {
        (void)coef;
        if (atom.rfind(t + "/", 0) == 0 || atom.rfind(t + "%", 0) == 0) {
          long long C = atoll(atom.c_str() + t.size() + 1);
          if (c && c != C) unsupported("line %d: two cell widths", line);
          c = C;
        }
        if (atom.rfind(k + "/", 0) == 0 || atom.rfind(k + "%", 0) == 0) {
          long long d = atoll(atom.c_str() + k.size() + 1);
          if (D && D != d) unsupported("line %d: two k splits", line);
          D = d;
        }
      }
    const uint64_t n = dom.n;
    uint64_t rows, cw;
    if (c) {
      if (n % (uint64_t)c) unsupported("line %d: domain not a whole number of rows", line);
      rows = n / c;
      cw = c;
    } else {
      rows = 1;
      cw = n;
    }
    MapalTileSite s{};
    s.rows = rows;
    s.c = cw;
    s.k = K;
    s.seed = seed.f;
    s.mul_a_first = 1;
    s.add_acc_first = add_acc_first ? 1 : 0;
    auto fill = [&](const Affine& f, MapalTileRead& r, uint64_t len) {
      long long base = 0, ci = 0, clane = 0, ck = 0, cq = 0, cr = 0;
      for (auto& [atom, coef] : f) {
        if (atom == "1") base += coef;
        else if (atom == t) {  // t = i*c + lane
          ci += coef * (long long)cw;
          clane += coef;
        } else if (atom == t + "/" + std::to_string(c)) ci += coef;
        else if (atom == t + "%" + std::to_string(c)) clane += coef;
        else if (atom == k) ck += coef;
        else if (atom == k + "/" + std::to_string(D)) cq += coef;
        else if (atom == k + "%" + std::to_string(D)) cr += coef;
        else unsupported("line %d: address atom %s", line, atom.c_str());
      }
      if (rows == 1) ci = 0;
      if (base < 0 || ci < 0 || clane < 0 || ck < 0 || cq < 0 || cr < 0)
        unsupported("line %d: negative address coefficient", line);
      r.base = base;
      r.ci = ci;
      r.clane = clane;
      r.ck = ck;
      r.ksplit.div = (cq || cr) ? D : 0;
      r.ksplit.cq = cq;
      r.ksplit.cr = cr;
      r.len = len;
    };
    fill(fa, s.a, A.n);
    fill(fbb, s.b, B.n);
    need(A);
    need(B);
    say(describe(s));
    if (nt_shaped(s)) return matmul_nt(s, A, B, line);
    return run_tile(s, A, B);
  }

  static std::string describe(const MapalTileSite& s) {
    char desc[512];
    snprintf(desc, sizeof desc,
             "tile_site rows=%llu c=%llu k=%llu a{base=%llu ci=%llu ck=%llu clane=%llu ks=%llu/%llu/%llu} "
             "b{base=%llu ci=%llu ck=%llu clane=%llu ks=%llu/%llu/%llu}",
             (unsigned long long)s.rows, (unsigned long long)s.c, (unsigned long long)s.k,
             (unsigned long long)s.a.base, (unsigned long long)s.a.ci, (unsigned long long)s.a.ck,
             (unsigned long long)s.a.clane, (unsigned long long)s.a.ksplit.div, (unsigned long long)s.a.ksplit.cq,
             (unsigned long long)s.a.ksplit.cr, (unsigned long long)s.b.base, (unsigned long long)s.b.ci,
             (unsigned long long)s.b.ck, (unsigned long long)s.b.clane, (unsigned long long)s.b.ksplit.div,
             (unsigned long long)s.b.ksplit.cq, (unsigned long long)s.b.ksplit.cr);
    return desc;
  }

  Value run_tile(const MapalTileSite& s, const Value& A, const Value& B) {
    if (mm_mode == MAPAL_MATMUL_TF32X3 && matmul_shaped(s)) say("matmul mode tf32x3");
    if (gpus > 1 && matmul_shaped(s) && s.rows >= (uint64_t)gpus) return matmul_partitioned(s, A, B);
    Value out = make_array(TY_F32, s.rows * s.c);
    if (!plan)
      check(mapal_gpu_tile_site_f32(ctx, &s, (const float*)A.ptr(), (const float*)B.ptr(), (float*)out.ptr(),
                                    mm_mode),
            "tile_site");
    return out;
  }

  // A * B^T: b reads B[base + k + lane * ldb] (B holds the right operand's
  // columns as rows, e.g. benches/shapes/attn_256_rowmajor.mapal).
  static bool nt_shaped(const MapalTileSite& s) {
    return s.k > 0 && s.a.ksplit.div == 0 && s.b.ksplit.div == 0 && s.a.ck == 1 && s.a.clane == 0 &&
           s.a.ci >= s.k && s.b.ci == 0 && s.b.ck == 1 && s.b.clane >= s.k && s.c > 1;
  }

  // Relayout first, then the plain matmul site: a move site writes the K x N
  // operand (T[k*N + n] = B[base + n*ldb + k]), and the matmul reads it row-major.
  // Every cell keeps its k order, so the result is the same bit for bit.
  Value matmul_nt(const MapalTileSite& s, const Value& A, const Value& B, int line) {
    const uint64_t K = s.k, N = s.c, ldb = s.b.clane;
    const unsigned __int128 b_max = (unsigned __int128)s.b.base + (unsigned __int128)(N - 1) * ldb + (K - 1);
    if (b_max >= B.n) mapal_trap(1);  // the Index rule, as the site itself would apply it
    MapalMoveSite mv{N, K, 1, ldb, B.n - s.b.base};
    say("move_site width=" + std::to_string(N) + " rows=" + std::to_string(K) + " cq=1 cr=" + std::to_string(ldb) +
        " (B^T -> K x N)");
    Value T = make_array(TY_F32, K * N);
    if (!plan) check(mapal_gpu_transpose(ctx, &mv, (const float*)B.ptr() + s.b.base, (float*)T.ptr()), "move_site");
    MapalTileSite m = s;
    m.b.base = 0;
    m.b.ck = N;
    m.b.clane = 1;
    m.b.len = K * N;
    (void)line;
    say(describe(m));
    return run_tile(m, A, T);
  }

  static bool matmul_shaped(const MapalTileSite& s) {
    return s.k > 0 && s.a.ksplit.div == 0 && s.b.ksplit.div == 0 && s.a.ck == 1 && s.a.clane == 0 &&
           s.b.ci == 0 && s.b.clane == 1 && s.a.ci >= s.k && s.b.ck >= s.c;
  }

  // The partitioner's matmul rule (row blocks of A and C per device, B
  // replicated by the sharded entry point's NCCL broadcast): arrays live on
  // the first device, so each other device receives its A rows by a peer copy
  // and returns its C rows the same way. Strict results are bit-identical to
  // the one-device site: no cell's k order changes.
  Value matmul_partitioned(const MapalTileSite& s, const Value& A, const Value& B) {
    std::vector<uint64_t> lo(gpus), hi(gpus), m(gpus);
    std::string rows;
    for (int d = 0; d < gpus; ++d) {
      mapal_gpu_shard_range(s.rows, gpus, d, &lo[d], &hi[d]);
      m[d] = hi[d] - lo[d];
      rows += (d ? "," : "") + std::to_string(m[d]);
    }
    say("matmul_f32_sharded gpus=" + std::to_string(gpus) + " rows=" + rows);
    // the Index rule before any copy: a read outside an operand traps
    const unsigned __int128 a_max = (unsigned __int128)s.a.base + (unsigned __int128)(s.rows - 1) * s.a.ci + (s.k - 1);
    const unsigned __int128 b_max = (unsigned __int128)s.b.base + (unsigned __int128)(s.k - 1) * s.b.ck + (s.c - 1);
    if (a_max >= A.n || b_max >= B.n) mapal_trap(1);
    Value out = make_array(TY_F32, s.rows * s.c);
    if (plan) return out;
    sync_point();  // A and B are final on the first device
    const uint64_t lda = s.a.ci, K = s.k, N = s.c;
    const float* abase = (const float*)A.ptr() + s.a.base;
    std::vector<const float*> ap(gpus);
    std::vector<float*> bp(gpus), cp(gpus);
    auto cuda = [](cudaError_t e, const char* what) {
      if (e != cudaSuccess) infra(std::string(what) + ": " + cudaGetErrorString(e));
    };
    for (int d = 0; d < gpus; ++d) {
      if (d == 0) {
        ap[0] = abase + lo[0] * lda;
        bp[0] = (float*)B.ptr();
        cp[0] = (float*)out.ptr() + lo[0] * N;
        continue;
      }
      const uint64_t a_elems = m[d] ? (m[d] - 1) * lda + K : 0;
      float *a_d = nullptr, *b_d = nullptr, *c_d = nullptr;
      cuda(cudaSetDevice(dev0 + d), "cudaSetDevice");
      cuda(cudaMalloc(&a_d, (a_elems ? a_elems : 1) * 4), "cudaMalloc");
      cuda(cudaMalloc(&b_d, (s.b.len ? s.b.len : 1) * 4), "cudaMalloc");
      cuda(cudaMalloc(&c_d, (m[d] * N ? m[d] * N : 1) * 4), "cudaMalloc");
      if (a_elems) cuda(cudaMemcpyPeer(a_d, dev0 + d, abase + lo[d] * lda, dev0, a_elems * 4), "cudaMemcpyPeer");
      ap[d] = a_d;
      bp[d] = b_d;
      cp[d] = c_d;
    }
    cuda(cudaSetDevice(dev0), "cudaSetDevice");
    {
      StdoutToStderr quiet;
      check(mapal_gpu_matmul_f32_sharded(ctx, &s, ap.data(), bp.data(), cp.data(), m.data(), 0, mm_mode),
            "matmul_f32_sharded");
      check(mapal_gpu_synchronize(ctx), "synchronize");
    }
    for (int d = 1; d < gpus; ++d) {
      if (m[d]) cuda(cudaMemcpyPeer(cp[0] - lo[0] * N + lo[d] * N, dev0, cp[d], dev0 + d, m[d] * N * 4), "cudaMemcpyPeer");
      cuda(cudaSetDevice(dev0 + d), "cudaSetDevice");
      cudaFree((void*)ap[d]);
      cudaFree(bp[d]);
      cudaFree(cp[d]);
    }
    cuda(cudaSetDevice(dev0), "cudaSetDevice");
    return out;
  }

  // t -> a[cq*(t/W) + cr*(t%W)] over an iota domain: a move site
  bool try_move(const std::string& prm, const EP& b, const Value& dom, Value& out, int line) {
    if (dom.ty != TY_IOTA || b->k != Expr::INDEX || b->kids[0]->k != Expr::NAME) return false;
    Value a = eval(b->kids[0], line);
    if (a.ty != TY_ARR || a.elem != TY_F32) return false;
    Affine f;
    if (!affine(b->kids[1], {prm}, f)) return false;
    long long W = 0, cq = 0, cr = 0;
    for (auto& [atom, coef] : f) {
      if (atom == "1") {
        if (coef) return false;
      } else if (atom == prm) {
        return false;  // plain t reads are not a move site; the general map handles them
      } else {
        long long C = atoll(atom.c_str() + prm.size() + 1);
        if (W && W != C) return false;
        W = C;
        (atom[prm.size()] == '/' ? cq : cr) += coef;
      }
    }
    if (!W || cq < 0 || cr < 0 || dom.n % (uint64_t)W) return false;
    MapalMoveSite s{(uint64_t)W, dom.n / W, (uint64_t)cq, (uint64_t)cr, a.n};
    need(a);
    say("move_site width=" + std::to_string(W) + " rows=" + std::to_string(s.rows) + " cq=" + std::to_string(cq) +
        " cr=" + std::to_string(cr));
    out = make_array(TY_F32, dom.n);
    if (!plan) check(mapal_gpu_transpose(ctx, &s, (const float*)a.ptr(), (float*)out.ptr()), "move_site");
    return true;
  }

  // (x, y) -> zip -> map { p -> a * p.0 + p.1 }
  bool try_saxpy(const std::string& prm, const EP& b, const Value& dom, Value& out, int line) {
    if (dom.ty != TY_ZIP || b->k != Expr::BIN || b->op != '+') return false;
    const EP &l = b->kids[0], &r = b->kids[1];
    auto proj = [&](const EP& e, long long idx) {
      return e->k == Expr::PROJ && e->ival == idx && e->kids[0]->k == Expr::NAME && e->kids[0]->s == prm;
    };
    if (l->k != Expr::BIN || l->op != '*' || !proj(r, 1)) return false;
    EP lit = l->kids[0], x = l->kids[1];
    if (!(lit->k == Expr::FLOAT || lit->k == Expr::NAME) || !proj(x, 0)) return false;
    const Value &X = dom.items[0], &Y = dom.items[1];
    if (X.ty != TY_ARR || Y.ty != TY_ARR || X.elem != TY_F32 || Y.elem != TY_F32) return false;
    Value a = eval(lit, line, TY_F32);
    if (a.ty != TY_F32) return false;
    say("saxpy n=" + std::to_string(dom.n));
    out = make_array(TY_F32, dom.n);
    if (!plan)
      check(mapal_gpu_map_saxpy(ctx, a.f, (const float*)X.ptr(), (const float*)Y.ptr(), (float*)out.ptr(), dom.n),
            "saxpy");
    return true;
  }

  // -- counted-loop helpers, lifted into the cap form ---------------------------------
  //
  // The reference rewrites canonical counted loops into a captured Fold or
  // Map before any backend sees them (crates/mapal-rewrite/src/lift.rs:1-12,
  // R-LF / R-LM): `(counter, acc)` loops with counter 0..K and a pure
  // accumulator become `(seed, K -> iota) -> fold`, and `(counter, out)` loops
  // whose one update is `out[counter] <- value` with len(out) == K become
  // `K -> iota -> map`. A call of a Map-form helper runs as that map site, with
  // Fold-form helpers it calls inlined as the cell's fold: the matmul loop form
  // (examples/matmul4_loop.mapal, benches/matmul/matmul16.mapal) becomes the
  // matmul tile site.

  static EP subst(const EP& e, const std::map<std::string, EP>& m) {
    if (e->k == Expr::NAME) {
      auto it = m.find(e->s);
      return it == m.end() ? e : it->second;
    }
    auto c = std::make_shared<Expr>(*e);
    for (auto& k : c->kids) k = subst(k, m);
    return c;
  }

  static bool is_name(const EP& e, const std::string& n) { return e->k == Expr::NAME && e->s == n; }
  static bool is_int(const EP& e, long long v) { return e->k == Expr::INT && e->ival == v; }

  // `ctr + 1 -> ctr`
  static bool is_step(const LoopStmt& st, const std::string& ctr) {
    if (st.k != LoopStmt::BIND || st.chain.stages.size() != 1 || st.chain.stages[0].k != Stage::NAMED ||
        st.chain.stages[0].name != ctr)
      return false;
    const EP& h = st.chain.head;
    return h->k == Expr::BIN && h->op == '+' && is_name(h->kids[0], ctr) && is_int(h->kids[1], 1);
  }

  // The loop's counter: `mut ctr: i32 <- 0` compared against an integer literal K.
  static bool counter(const FnDef& f, std::string& ctr, long long& K) {
    if (f.cond_lhs->k != Expr::NAME || f.cond_rhs->k != Expr::INT || f.cond_rhs->ival < 1) return false;
    ctr = f.cond_lhs->s;
    K = f.cond_rhs->ival;
    for (auto& m : f.muts)
      if (m.name == ctr) return m.arr_len < 0 && is_int(m.init, 0);
    return false;
  }

  struct FoldForm {
    std::string ctr, acc;
    long long K;
    EP seed, body;
  };

  static bool fold_form(const FnDef& f, FoldForm& ff) {
    if (f.muts.size() != 2 || !counter(f, ff.ctr, ff.K) || f.body.size() != 2) return false;
    const FnDef::Mut& m = f.muts[0].name == ff.ctr ? f.muts[1] : f.muts[0];
    if (m.arr_len >= 0 || !is_name(f.ret, m.name)) return false;
    ff.acc = m.name;
    ff.seed = m.init;
    const LoopStmt& upd = f.body[0];
    if (upd.k != LoopStmt::BIND || upd.chain.stages.size() != 1 || upd.chain.stages[0].k != Stage::NAMED ||
        upd.chain.stages[0].name != ff.acc || !is_step(f.body[1], ff.ctr))
      return false;
    ff.body = upd.chain.head;
    return true;
  }

  // `(seed', iota K) -> fold { acc, ctr -> body' }` for a call of a Fold-form helper
  Chain inline_fold(const FnDef& g, const EP& args, int line) {
    FoldForm ff;
    if (!fold_form(g, ff)) unsupported("line %d: `%s` is not a counted fold loop", line, g.name.c_str());
    std::map<std::string, EP> m;
    std::vector<EP> av = args->k == Expr::TUPLE ? args->kids : std::vector<EP>{args};
    if (av.size() != g.params.size()) unsupported("line %d: `%s` takes %zu arguments", line, g.name.c_str(), g.params.size());
    for (size_t i = 0; i < av.size(); ++i) m[g.params[i]] = av[i];
    if (m.count(ff.acc) || m.count(ff.ctr)) unsupported("line %d: loop variable shadows a parameter", line);
    const std::string iota_name = "__iota" + std::to_string(synth++);
    Value iv;
    iv.ty = TY_IOTA;
    iv.n = (uint64_t)ff.K;
    env[iota_name] = iv;
    Chain c;
    c.line = line;
    c.head = std::make_shared<Expr>();
    c.head->k = Expr::TUPLE;
    auto nm = std::make_shared<Expr>();
    nm->k = Expr::NAME;
    nm->s = iota_name;
    c.head->kids = {subst(ff.seed, m), nm};
    Stage st;
    st.k = Stage::FOLD;
    st.lam = std::make_shared<Lambda>();
    st.lam->params = {ff.acc, ff.ctr};
    Chain b;
    b.line = line;
    b.head = subst(ff.body, m);
    st.lam->stmts.push_back(b);
    c.stages.push_back(st);
    return c;
  }

  Value call_fn(const FnDef& f, const Value& args, int line) {
    // arguments become synthetic bindings the lifted body refers to
    std::vector<Value> av = args.ty == TY_TUPLE ? args.items : std::vector<Value>{args};
    if (av.size() != f.params.size())
      unsupported("line %d: `%s` takes %zu arguments", line, f.name.c_str(), f.params.size());
    std::map<std::string, EP> m;
    for (size_t i = 0; i < av.size(); ++i) {
      const std::string nm = "__arg" + std::to_string(synth++);
      env[nm] = av[i];
      auto e = std::make_shared<Expr>();
      e->k = Expr::NAME;
      e->s = nm;
      m[f.params[i]] = e;
    }
    std::string ctr;
    long long K = 0;
    if (f.muts.size() != 2 || !counter(f, ctr, K) || f.body.size() < 2 || !is_step(f.body.back(), ctr))
      unsupported("line %d: `%s` is not a counted map loop", line, f.name.c_str());
    const FnDef::Mut& out = f.muts[0].name == ctr ? f.muts[1] : f.muts[0];
    const LoopStmt& upd = f.body[f.body.size() - 2];
    if (out.arr_len != K || !is_name(f.ret, out.name) || upd.k != LoopStmt::UPDATE ||
        !is_name(upd.target->kids[0], out.name) || !is_name(upd.target->kids[1], ctr))
      unsupported("line %d: `%s` must write every element out[%s] of a length-%lld array", line, f.name.c_str(),
                  ctr.c_str(), K);
    if (m.count(ctr)) unsupported("line %d: loop variable shadows a parameter", line);
    auto L = std::make_shared<Lambda>();
    L->params = {ctr};
    std::string call_result;
    Chain call_chain;
    for (size_t i = 0; i + 2 < f.body.size(); ++i) {
      const LoopStmt& st = f.body[i];
      if (st.k != LoopStmt::BIND) unsupported("line %d: only out[%s] may be updated", line, ctr.c_str());
      const Chain& c = st.chain;
      if (c.stages.size() == 2 && c.stages[0].k == Stage::NAMED && fns->count(c.stages[0].name) &&
          c.stages[1].k == Stage::NAMED) {
        if (!call_result.empty()) unsupported("line %d: more than one helper call in a map loop", line);
        call_result = c.stages[1].name;
        call_chain = inline_fold(fns->at(c.stages[0].name), subst(c.head, m), line);
        continue;
      }
      if (c.stages.size() != 1 || c.stages[0].k != Stage::NAMED) unsupported("line %d: map loop statement", line);
      Chain b = c;
      b.head = subst(c.head, m);
      L->stmts.push_back(b);
    }
    if (!call_result.empty()) {
      if (!is_name(upd.value, call_result)) unsupported("line %d: the helper's result must be the stored value", line);
      L->stmts.push_back(call_chain);
    } else {
      Chain b;
      b.line = line;
      b.head = subst(upd.value, m);
      L->stmts.push_back(b);
    }
    Value dom;
    dom.ty = TY_IOTA;
    dom.n = (uint64_t)K;
    say("lift " + f.name + ": counted loop over " + std::to_string(K) + " -> map");
    return map_site(*L, dom, line);
  }

  // -- the general map body -> MAPAL_X_* program --

  struct Compiler {
    Runner& R;
    std::string prm;
    const Value& dom;
    int line;
    bool fuse = false;  // splice deferred producers instead of reading their arrays
    std::vector<MapalExprOp> ops;
    std::vector<Value> arrays;  // slot table
    std::vector<std::shared_ptr<Lazy>> spliced;
    bool overflow = false;  // a fused program outgrew the op or slot table

    int slot_of(const Value& a) {
      for (size_t s = 0; s < arrays.size(); ++s)
        if (arrays[s].id == a.id) return (int)s;
      if (arrays.size() >= MAPAL_X_MAX_ARRAYS) {
        if (!fuse) unsupported("line %d: more than 8 arrays in one map body", line);
        overflow = true;
        return 0;
      }
      arrays.push_back(a);
      return (int)arrays.size() - 1;
    }
    void emit(uint16_t code, uint16_t slot = 0, int32_t i = 0, float f = 0) {
      if (ops.size() >= MAPAL_X_MAX_OPS - 1) {
        if (!fuse) unsupported("line %d: map body too long", line);
        overflow = true;
        return;
      }
      ops.push_back(MapalExprOp{code, slot, i, f});
    }
    // the producer's element law in place of a load of its element
    Ty splice(const std::shared_ptr<Lazy>& z) {
      for (MapalExprOp op : z->ops) {
        const bool slotted = op.code == MAPAL_X_IN_I32 || op.code == MAPAL_X_IN_F32 ||
                             op.code == MAPAL_X_LOAD_I32 || op.code == MAPAL_X_LOAD_F32;
        if (slotted) op.slot = (uint16_t)slot_of(z->arrays[op.slot]);
        emit(op.code, op.slot, op.i, op.f);
      }
      spliced.push_back(z);
      return z->out;
    }
    // the element (or zip projection) pushes
    Ty push_elem(int which) {
      const Value* src = nullptr;
      if (dom.ty == TY_IOTA) {
        if (which >= 0) unsupported("line %d: projection of an index", line);
        emit(MAPAL_X_T_I32);
        return TY_I32;
      }
      if (dom.ty == TY_ARR) {
        if (which >= 0) unsupported("line %d: projection of an array element", line);
        src = &dom;
      } else {
        if (which < 0 || which > 1) unsupported("line %d: a zip element is used as p.0 / p.1", line);
        src = &dom.items[which];
      }
      if (src->ty == TY_IOTA) {
        emit(MAPAL_X_T_I32);
        return TY_I32;
      }
      if (fuse && src->lazy && !src->lazy->done) return splice(src->lazy);
      int s = slot_of(*src);
      emit(src->elem == TY_F32 ? MAPAL_X_IN_F32 : MAPAL_X_IN_I32, (uint16_t)s);
      return src->elem;
    }
    Ty gen(const EP& e, Ty float_ctx) {
      switch (e->k) {
        case Expr::INT:
          emit(MAPAL_X_CONST_I32, 0, (int32_t)e->ival);
          return TY_I32;
        case Expr::FLOAT:
          emit(MAPAL_X_CONST_F32, 0, 0, strtof(e->s.c_str(), nullptr));
          return TY_F32;
        case Expr::NAME: {
          if (e->s == prm) return push_elem(-1);
          Value v = R.eval(e, line);
          if (v.ty == TY_I32) { emit(MAPAL_X_CONST_I32, 0, v.i); return TY_I32; }
          if (v.ty == TY_F32) { emit(MAPAL_X_CONST_F32, 0, 0, v.f); return TY_F32; }
          unsupported("line %d: capture `%s` is not an i32/f32 scalar", line, e->s.c_str());
        }
        case Expr::PROJ:
          if (e->kids[0]->k != Expr::NAME || e->kids[0]->s != prm) unsupported("line %d: projection", line);
          return push_elem((int)e->ival);
        case Expr::NEG: {
          Ty t = gen(e->kids[0], float_ctx);
          emit(t == TY_F32 ? MAPAL_X_NEG_F32 : MAPAL_X_NEG_I32);
          return t;
        }
        case Expr::INDEX: {
          if (e->kids[0]->k != Expr::NAME) unsupported("line %d: indexing an expression", line);
          Value a = R.eval(e->kids[0], line);
          if (a.ty == TY_IOTA) {  // iota[j] is j, with the bounds rule
            unsupported("line %d: indexing an iota inside a map body", line);
          }
          if (a.ty != TY_ARR) unsupported("line %d: indexing a non-array", line);
          if (gen(e->kids[1], TY_F32) != TY_I32) unsupported("line %d: index must be i32", line);
          int s = slot_of(a);
          emit(a.elem == TY_F32 ? MAPAL_X_LOAD_F32 : MAPAL_X_LOAD_I32, (uint16_t)s);
          return a.elem;
        }
        case Expr::BIN: {
          // a float literal takes its partner's type
          Ty tl, tr;
          const EP &l = e->kids[0], &r = e->kids[1];
          if (l->k == Expr::FLOAT && r->k != Expr::FLOAT) {
            size_t mark = ops.size();
            tr = gen(r, float_ctx);
            std::vector<MapalExprOp> rhs(ops.begin() + mark, ops.end());
            ops.resize(mark);
            tl = gen(l, float_ctx);
            ops.insert(ops.end(), rhs.begin(), rhs.end());
          } else {
            tl = gen(l, float_ctx);
            tr = gen(r, float_ctx);
          }
          if (tl != tr) unsupported("line %d: mixed operand types in a map body", line);
          const bool f = tl == TY_F32;
          uint16_t code = 0;
          switch (e->op) {
            case '+': code = f ? MAPAL_X_ADD_F32 : MAPAL_X_ADD_I32; break;
            case '-': code = f ? MAPAL_X_SUB_F32 : MAPAL_X_SUB_I32; break;
            case '*': code = f ? MAPAL_X_MUL_F32 : MAPAL_X_MUL_I32; break;
            case '/': code = f ? MAPAL_X_DIV_F32 : MAPAL_X_DIV_I32; break;
            case '%': code = f ? MAPAL_X_REM_F32 : MAPAL_X_REM_I32; break;
          }
          emit(code);
          return tl;
        }
        default: unsupported("line %d: expression kind in a map body", line);
      }
    }
  };

  // Deepest stack a program reaches (the map_expr kernel holds 16 values).
  static int stack_depth(const std::vector<MapalExprOp>& ops) {
    int sp = 0, top = 0;
    for (const MapalExprOp& op : ops) {
      switch (op.code) {
        case MAPAL_X_T_I32: case MAPAL_X_CONST_I32: case MAPAL_X_CONST_F32:
        case MAPAL_X_IN_I32: case MAPAL_X_IN_F32:
          ++sp;
          break;
        case MAPAL_X_LOAD_I32: case MAPAL_X_LOAD_F32: case MAPAL_X_NEG_I32: case MAPAL_X_NEG_F32:
        case MAPAL_X_WIDEN_I32_F32:
          break;
        default:  // the binary ops and the store pop one
          --sp;
      }
      if (sp > top) top = sp;
    }
    return top;
  }

  // Whether consumers may recompute a body in place of loading its result: no
  // Index read (it could trap index_oob) and no i32 division or remainder by
  // anything but a nonzero literal (div_zero). Float arithmetic never traps,
  // and a body holds no print, clock or loop, so it is also effect-free.
  static bool trap_free(const std::vector<MapalExprOp>& ops) {
    for (size_t k = 0; k < ops.size(); ++k) {
      const uint16_t c = ops[k].code;
      if (c == MAPAL_X_LOAD_I32 || c == MAPAL_X_LOAD_F32) return false;
      if ((c == MAPAL_X_DIV_I32 || c == MAPAL_X_REM_I32) &&
          !(k > 0 && ops[k - 1].code == MAPAL_X_CONST_I32 && ops[k - 1].i != 0))
        return false;
    }
    return true;
  }

  static constexpr int kMapStack = 16;
  bool fuse_maps = true;                        // --no-fuse: every map site writes its array
  std::vector<std::shared_ptr<Lazy>> pending;  // deferred maps not yet written
  std::vector<std::shared_ptr<DevBuf>> kept;   // dead arrays, freed at exit (cudaFree waits for the device)

  // Launch a deferred map: its body plus the store, into a new array.
  void materialise(Lazy& z) {
    if (z.done) return;
    z.done = true;
    for (auto& a : z.arrays) need(a);
    std::vector<MapalExprOp> prog = z.ops;
    prog.push_back(MapalExprOp{(uint16_t)(z.out == TY_F32 ? MAPAL_X_STORE_F32 : MAPAL_X_STORE_I32), 0, 0, 0});
    say("map_expr n=" + std::to_string(z.n) + " ops=" + std::to_string(prog.size()) +
        " arrays=" + std::to_string(z.arrays.size()));
    Value out = make_array(z.out, z.n);
    if (!plan) {
      std::vector<const void*> ptrs;
      std::vector<uint64_t> lens;
      for (auto& a : z.arrays) {
        ptrs.push_back(a.ptr());
        lens.push_back(a.n);
      }
      check(mapal_gpu_map_expr(ctx, prog.data(), (uint32_t)prog.size(), ptrs.data(), lens.data(),
                               (uint32_t)z.arrays.size(), out.ptr(), z.n),
            "map_expr");
    }
    z.mat = out;
  }

  // After a statement (clock = false) or before a clock read (clock = true).
  // A deferred map that nothing holds any more is dropped when a consumer
  // recomputed it and written otherwise, so its work still runs where the
  // program put it; before a clock read every live one is written, so the
  // time between two reads covers the sites issued between them.
  void settle(bool clock) {
    std::vector<std::shared_ptr<Lazy>> keep;
    for (auto& z : pending) {
      const bool dead = z.use_count() == 1;
      if (!z->done && !(dead && z->consumed) && (dead || clock)) materialise(*z);
      if (z->done) {
        if (z->mat.buf) kept.push_back(z->mat.buf);
      } else if (!dead) {
        keep.push_back(z);
      }
    }
    pending.swap(keep);
  }

  Value general_map(const std::string& prm, const EP& body, bool widen, const Value& dom, int line) {
    for (int pass = 0;; ++pass) {
      // pass 0 splices deferred producers; pass 1 (if the fused program is too
      // long, too deep or has too many arrays) reads their arrays instead
      Compiler C{*this, prm, dom, line};
      C.fuse = fuse_maps && pass == 0;
      Ty t = C.gen(body, TY_F32);
      if (widen) {
        if (t != TY_I32) unsupported("line %d: widen_f32 of a non-i32 body", line);
        C.emit(MAPAL_X_WIDEN_I32_F32);
        t = TY_F32;
      }
      if (t != TY_I32 && t != TY_F32) unsupported("line %d: map body result type", line);
      if (C.fuse && (C.overflow || stack_depth(C.ops) > kMapStack)) continue;
      for (auto& z : C.spliced) z->consumed = true;
      const std::string fused = C.spliced.empty() ? "" : " fused=" + std::to_string(C.spliced.size());
      if (fuse_maps && dom.n > 0 && dom.n <= (1ull << 31) && trap_free(C.ops)) {
        auto z = std::make_shared<Lazy>();
        z->ops = C.ops;
        z->arrays = C.arrays;
        z->out = t;
        z->n = dom.n;
        say("map_expr n=" + std::to_string(dom.n) + " ops=" + std::to_string(C.ops.size() + 1) +
            " arrays=" + std::to_string(C.arrays.size()) + fused + " deferred");
        pending.push_back(z);
        Value v;
        v.ty = TY_ARR;
        v.elem = t;
        v.n = dom.n;
        v.id = next_id++;
        v.lazy = z;
        return v;
      }
      for (auto& a : C.arrays) need(a);
      C.ops.push_back(MapalExprOp{(uint16_t)(t == TY_F32 ? MAPAL_X_STORE_F32 : MAPAL_X_STORE_I32), 0, 0, 0});
      say("map_expr n=" + std::to_string(dom.n) + " ops=" + std::to_string(C.ops.size()) +
          " arrays=" + std::to_string(C.arrays.size()) + fused);
      Value out = make_array(t, dom.n);
      if (!plan) {
        std::vector<const void*> ptrs;
        std::vector<uint64_t> lens;
        for (auto& a : C.arrays) {
          ptrs.push_back(a.ptr());
          lens.push_back(a.n);
        }
        check(mapal_gpu_map_expr(ctx, C.ops.data(), (uint32_t)C.ops.size(), ptrs.data(), lens.data(),
                                 (uint32_t)C.arrays.size(), out.ptr(), dom.n),
              "map_expr");
      }
      return out;
    }
  }
};

Runner* g_runner = nullptr;

void* Value::ptr() const {
  if (lazy) {
    if (!lazy->done) g_runner->materialise(*lazy);
    return lazy->mat.buf ? lazy->mat.buf->p : nullptr;
  }
  return buf ? buf->p : nullptr;
}

}  // namespace

int main(int argc, char** argv) {
  bool plan = false, fast_fold = false, tf32x3 = false, no_fuse = false;
  int device = 0, gpus = 1;
  const char* path = nullptr;
  for (int a = 1; a < argc; ++a) {
    if (!strcmp(argv[a], "--plan")) plan = true;
    else if (!strcmp(argv[a], "--fast-fold")) fast_fold = true;
    else if (!strcmp(argv[a], "--tf32x3")) tf32x3 = true;
    else if (!strcmp(argv[a], "--no-fuse")) no_fuse = true;
    else if (!strcmp(argv[a], "--device") && a + 1 < argc) device = atoi(argv[++a]);
    else if (!strcmp(argv[a], "--gpus") && a + 1 < argc) gpus = atoi(argv[++a]);
    else path = argv[a];
  }
  if (!path) {
    fprintf(stderr, "usage: mapal-run [--device D] [--gpus N] [--plan] [--fast-fold] [--tf32x3] [--no-fuse] program.mapal\n");
    return 2;
  }
  if (gpus < 1 || device < 0 || device + gpus > 32) {
    fprintf(stderr, "mapal-run: bad --device / --gpus\n");
    return 2;
  }
  FILE* f = fopen(path, "rb");
  if (!f) {
    fprintf(stderr, "mapal-run: cannot open %s\n", path);
    return 2;
  }
  std::string src;
  char buf[65536];
  size_t got;
  while ((got = fread(buf, 1, sizeof buf, f)) > 0) src.append(buf, got);
  fclose(f);

  Parser P{lex(src)};
  std::vector<Chain> body = P.main_body();
  Runner R;
  R.fns = &P.fns;
  R.gpus = gpus;
  R.mm_mode = tf32x3 ? MAPAL_MATMUL_TF32X3 : MAPAL_MATMUL_STRICT;
  R.dev0 = device;
  R.plan = plan;
  R.fast_fold = fast_fold;
  R.fuse_maps = !no_fuse;
  g_runner = &R;
  mapal_time_ms();  // start the process clock, as the reference's runtime does on first use
  if (!plan) {
    int have = 0;
    check(mapal_gpu_device_count(&have), "device_count");
    if (device + gpus > have) infra("fewer devices than --device + --gpus");
    if (cudaSetDevice(device) != cudaSuccess) infra("cudaSetDevice");
    {
      StdoutToStderr quiet;  // a multi-device context sets up NCCL communicators
      check(mapal_gpu_ctx_create(((1u << gpus) - 1) << device, &R.ctx), "ctx_create");
    }
    // the legacy default stream orders the sites with this driver's own copies
    check(mapal_gpu_set_stream(R.ctx, 0, nullptr), "set_stream");
    check(mapal_gpu_set_sync(R.ctx, 0), "set_sync");
  }
  R.run_main(body);
  if (R.ctx) {
    check(mapal_gpu_synchronize(R.ctx), "synchronize");
    R.env.clear();
    R.pending.clear();
    R.kept.clear();
    mapal_gpu_ctx_destroy(R.ctx);
  }
  fflush(stdout);
  return 0;
}
