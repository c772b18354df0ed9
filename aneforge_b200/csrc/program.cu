// The CUDA invoker: a "program" is a lowered plan of fused sm_100a kernel launches over named
// device buffers (ports, resident state, weights, activations, scratch), replayed as one CUDA graph
// with programmatic dependent launch between kernels. It replaces the reference's e5rt program
// (aneforge/_lib/ane_e5rt_dispatch.mm): same port model (named fp16 ports, zero-initialised,
// zero-copy buffer pointers, output->input aliasing for resident state, synchronous execute whose
// first call finalises the program), with device memory instead of shared ANE buffers.
//
// Plan text (one statement per line, '#' comments):
//   AFPLAN 1
//   buf <name> <bytes> <role>          role: in | out | state | tmp | weight | scratch
//   wfile <name> <offset>              load a weight buffer from <plan dir>/weights.bin
//   op <kind> key=value ...            buffer refs are `name`, `name@byte_offset`, or `-` (null)
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "af_common.cuh"
#include "af_kernels.h"
#include "../../include/af_cuda.h"

namespace af {

static thread_local std::string g_last_error;

static void set_error(const std::string& msg) {
  g_last_error = msg;
  fprintf(stderr, "[aneforge_b200] %s\n", msg.c_str());
}

void set_error_public(const std::string& msg) { set_error(msg); }

enum Role { R_IN, R_OUT, R_STATE, R_TMP, R_WEIGHT, R_SCRATCH };

struct Buffer {
  std::string name;
  size_t bytes = 0;
  Role role = R_TMP;
  void* dev = nullptr;
  bool owned = false;
  bool ready = false;          // weights: uploaded/bound/loaded
  long long file_off = -1;
  int alias_of = -1;           // share_buffer: this input reads buffer `alias_of`
};

struct Op {
  std::string kind;
  std::map<std::string, std::string> kv;
  int line = 0;
};

struct Program {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<Buffer> bufs;
  std::map<std::string, int> idx;
  std::vector<Op> ops;
  std::string dir;
  bool finalized = false;
  bool use_graph = true;
  bool use_pdl = true;
  cudaGraphExec_t exec = nullptr;
  int* d_err = nullptr;
  void* comm = nullptr;        // tensor-parallel communicator (af_program_set_comm), not owned
};

// ------------------------------------------------------------------------------------ helpers

static bool parse_role(const std::string& s, Role& r) {
  if (s == "in") r = R_IN;
  else if (s == "out") r = R_OUT;
  else if (s == "state") r = R_STATE;
  else if (s == "tmp") r = R_TMP;
  else if (s == "weight") r = R_WEIGHT;
  else if (s == "scratch") r = R_SCRATCH;
  else return false;
  return true;
}

static int find_buf(Program& p, const std::string& name) {
  auto it = p.idx.find(name);
  return it == p.idx.end() ? -1 : it->second;
}

struct OpCtx {
  Program& p;
  const Op& op;
  std::string err;
  bool has(const char* k) const { return op.kv.count(k) && op.kv.at(k) != "-"; }
  const std::string* raw(const char* k) {
    auto it = op.kv.find(k);
    if (it == op.kv.end()) { err = std::string("missing key '") + k + "'"; return nullptr; }
    return &it->second;
  }
  long long i(const char* k, long long dflt = LLONG_MIN) {
    auto it = op.kv.find(k);
    if (it == op.kv.end()) {
      if (dflt == LLONG_MIN) err = std::string("missing int '") + k + "'";
      return dflt == LLONG_MIN ? 0 : dflt;
    }
    return strtoll(it->second.c_str(), nullptr, 10);
  }
  double f(const char* k, double dflt = NAN) {
    auto it = op.kv.find(k);
    if (it == op.kv.end()) {
      if (std::isnan(dflt)) err = std::string("missing float '") + k + "'";
      return std::isnan(dflt) ? 0.0 : dflt;
    }
    return strtod(it->second.c_str(), nullptr);
  }
  // buffer reference with optional byte offset; `need` bytes must fit
  void* ptr(const char* k, size_t need = 0, bool optional = false) {
    auto it = op.kv.find(k);
    if (it == op.kv.end() || it->second == "-") {
      if (!optional) err = std::string("missing buffer '") + k + "'";
      return nullptr;
    }
    std::string s = it->second;
    size_t off = 0;
    auto at = s.find('@');
    if (at != std::string::npos) {
      off = strtoull(s.c_str() + at + 1, nullptr, 10);
      s = s.substr(0, at);
    }
    int bi = find_buf(p, s);
    if (bi < 0) { err = "unknown buffer '" + s + "'"; return nullptr; }
    int root = bi;
    while (p.bufs[root].alias_of >= 0) root = p.bufs[root].alias_of;
    if (off + need > p.bufs[root].bytes) {
      err = "buffer '" + s + "' too small for key '" + k + "' (" + std::to_string(off + need) + " > " +
            std::to_string(p.bufs[root].bytes) + ")";
      return nullptr;
    }
    return static_cast<char*>(p.bufs[root].dev) + off;
  }
  // a buffer by its plan name (per-layer names derived by the op)
  void* named(const std::string& s, size_t need, bool optional = false) {
    int bi = find_buf(p, s);
    if (bi < 0) {
      if (!optional) err = "unknown buffer '" + s + "'";
      return nullptr;
    }
    int root = bi;
    while (p.bufs[root].alias_of >= 0) root = p.bufs[root].alias_of;
    if (need > p.bufs[root].bytes) {
      err = "buffer '" + s + "' too small (" + std::to_string(need) + " > " + std::to_string(p.bufs[root].bytes) + ")";
      return nullptr;
    }
    return p.bufs[root].dev;
  }
  // comma-separated integers (graph shapes and strides); empty when the key is absent or "-"
  std::vector<long long> ints(const char* k) {
    std::vector<long long> v;
    auto it = op.kv.find(k);
    if (it == op.kv.end() || it->second == "-") return v;
    std::stringstream ss(it->second);
    std::string item;
    while (std::getline(ss, item, ',')) v.push_back(strtoll(item.c_str(), nullptr, 10));
    return v;
  }
  std::vector<double> list(const char* k, size_t n) {
    std::vector<double> v;
    auto it = op.kv.find(k);
    if (it == op.kv.end()) { err = std::string("missing list '") + k + "'"; return v; }
    std::stringstream ss(it->second);
    std::string item;
    while (std::getline(ss, item, ',')) v.push_back(strtod(item.c_str(), nullptr));
    if (v.size() != n) err = std::string("list '") + k + "' needs " + std::to_string(n) + " values";
    return v;
  }
};

// Optional L2 prefetch keys of an op: pf=<buffer> (a later kernel's weights), pfs=<bytes of that
// region>, pfn=<bytes to prefetch>, pfg=<CTAs of the kernel that reads them>. The region splits
// into pfg equal pieces (that kernel's CTAs read consecutive equal ranges in order) and the first
// pfn/pfs of each piece is fetched, so every CTA starts on lines already in L2.
static L2Pf parse_pf(OpCtx& c) {
  L2Pf f;
  const long long total = c.i("pfs", 0), want = c.i("pfn", 0), parts = c.i("pfg", 1);
  if (total <= 0 || want <= 0 || parts < 1 || !c.has("pf")) return f;
  f.base = static_cast<const char*>(c.ptr("pf", (size_t)total));
  if (!f.base) return L2Pf();
  f.bytes = (size_t)total;
  f.stride = ((size_t)total / (size_t)parts) & ~(size_t)15;
  if (f.stride < 16) return L2Pf();
  const double frac = want < total ? (double)want / (double)total : 1.0;
  f.piece = ((size_t)(frac * (double)f.stride) + 15) & ~(size_t)15;
  if (f.piece > f.stride) f.piece = f.stride;
  if (f.piece == f.stride) {                     // the whole region: 16 KB pieces back to back
    f.piece = f.stride = 16384;
  }
  f.keep = (int)c.i("pfk", 0);
  return f;
}

static int wf_of(const std::string& s) {
  if (s == "i8") return W_I8;
  if (s == "f16") return W_F16;
  if (s == "i4") return W_I4G32;
  if (s == "l4") return W_LUT4;
  if (s == "i8g") return W_I8G;
  if (s == "sp") return W_SPARSE;
  return -1;
}
static int epi_of(const std::string& s) {
  if (s == "f32") return EPI_F32;
  if (s == "f16") return EPI_F16;
  if (s == "resid") return EPI_RESID;
  if (s == "swiglu") return EPI_SWIGLU;
  if (s == "argmax") return EPI_ARGMAX;
  return -1;
}

// ------------------------------------------------------------------------------------ graph ops

// elements an N-d view spans: 1 + sum over axes of (extent - 1) * stride (strides >= 0)
static size_t view_span(const std::vector<long long>& shape, const std::vector<long long>& stride) {
  long long hi = 0;
  for (size_t d = 0; d < shape.size(); ++d) {
    if (shape[d] <= 0) return 0;
    hi += (shape[d] - 1) * stride[d];
  }
  return (size_t)hi + 1;
}

static bool fill_nd(const std::vector<long long>& v, long long (&out)[GRAPH_MAX_RANK]) {
  if (v.size() > (size_t)GRAPH_MAX_RANK) return false;
  for (size_t d = 0; d < v.size(); ++d) out[d] = v[d];
  return true;
}

static long long numel_of(const std::vector<long long>& shape) {
  long long n = 1;
  for (long long d : shape) n *= d;
  return n;
}

// The generic graph ops (`g_*`, graph_ops.cu). Every operand size is checked against its buffer
// before anything launches, so a plan with a bad shape fails at compile time.
static bool graph_op(OpCtx& c, const Op& op, bool dry, cudaStream_t st, cudaError_t& e, std::string& why) {
  auto bad = [&](const std::string& m) { why = m; return false; };
  auto rank_ok = [&](const std::vector<long long>& sh, const std::vector<long long>& st1) {
    return !sh.empty() && sh.size() <= (size_t)GRAPH_MAX_RANK && st1.size() == sh.size();
  };
  if (op.kind == "g_ew") {
    GraphEwArgs a;
    const auto shape = c.ints("shape"), sa = c.ints("sa"), sb = c.ints("sb"), sc = c.ints("sc");
    a.op = (int)c.i("op");
    if (!rank_ok(shape, sa)) return bad("g_ew: bad shape / sa");
    a.rank = (int)shape.size();
    a.n = numel_of(shape);
    fill_nd(shape, a.shape); fill_nd(sa, a.sa);
    a.a = (const float*)c.ptr("a", 4 * view_span(shape, sa));
    if (c.has("b")) {
      if (sb.size() != shape.size()) return bad("g_ew: bad sb");
      fill_nd(sb, a.sb);
      a.b = (const float*)c.ptr("b", 4 * view_span(shape, sb));
    }
    if (a.op == G_SELECT) {
      if (sc.size() != shape.size() || !c.has("b")) return bad("g_ew select: needs b and c with strides");
      fill_nd(sc, a.sc);
      a.c = (const float*)c.ptr("c", 4 * view_span(shape, sc));
    } else if (a.op < 0 || a.op > G_NE) {
      return bad("g_ew: unknown op");
    }
    a.y = (float*)c.ptr("y", 4 * (size_t)a.n);
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_ew_launch(a, st);
  } else if (op.kind == "g_un") {
    const long long n = c.i("n");
    const int u = (int)c.i("op");
    const float k = (float)c.f("k", 0.0), k2 = (float)c.f("k2", 0.0);
    const float* x = (const float*)c.ptr("x", 4 * (size_t)n);
    float* y = (float*)c.ptr("y", 4 * (size_t)n);
    if (u < 0 || u > U_SOFTPLUS) return bad("g_un: unknown op");
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_unary_launch(x, y, n, u, k, k2, st);
  } else if (op.kind == "g_copy") {
    GraphCopyArgs a;
    const auto shape = c.ints("shape"), sx = c.ints("sx"), sy = c.ints("sy");
    if (!rank_ok(shape, sx) || sy.size() != shape.size()) return bad("g_copy: bad shape / strides");
    a.rank = (int)shape.size();
    a.n = numel_of(shape);
    fill_nd(shape, a.shape); fill_nd(sx, a.sx); fill_nd(sy, a.sy);
    a.x = (const float*)c.ptr("x", 4 * view_span(shape, sx));
    a.y = (float*)c.ptr("y", 4 * view_span(shape, sy));
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_copy_launch(a, st);
  } else if (op.kind == "g_reduce") {
    GraphReduceArgs a;
    const auto shape = c.ints("shape");
    if (shape.empty() || shape.size() > (size_t)GRAPH_MAX_RANK) return bad("g_reduce: bad shape");
    a.rank = (int)shape.size();
    fill_nd(shape, a.shape);
    a.op = (int)c.i("op");
    a.mask = (int)c.i("mask");
    if (a.op < 0 || a.op > RD_L1) return bad("g_reduce: unknown op");
    long long nout = 1;
    for (int d = 0; d < a.rank; ++d) nout *= ((a.mask >> d) & 1) ? 1 : shape[d];
    a.n_out = nout;
    a.x = (const float*)c.ptr("x", 4 * (size_t)numel_of(shape));
    a.y = (float*)c.ptr("y", 4 * (size_t)nout);
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_reduce_launch(a, st);
  } else if (op.kind == "g_softmax") {
    const long long outer = c.i("outer"), n = c.i("n"), inner = c.i("inner");
    const size_t total = 4 * (size_t)(outer * n * inner);
    const float* x = (const float*)c.ptr("x", total);
    float* y = (float*)c.ptr("y", total);
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_softmax_launch(x, y, outer, n, inner, st);
  } else if (op.kind == "g_rms" || op.kind == "g_ln") {
    const long long rows = c.i("rows");
    const int d = (int)c.i("d");
    const float* x = (const float*)c.ptr("x", 4 * (size_t)(rows * d));
    float* y = (float*)c.ptr("y", 4 * (size_t)(rows * d));
    const __half* g = (const __half*)c.ptr("g", 2 * (size_t)d);
    if (op.kind == "g_rms") {
      const float floor = (float)c.f("floor");
      if (!c.err.empty()) return bad(c.err);
      if (!dry) e = graph_rms_launch(x, y, g, floor, rows, d, st);
    } else {
      const __half* b = (const __half*)c.ptr("b", 2 * (size_t)d, true);
      const float eps = (float)c.f("eps");
      if (!c.err.empty()) return bad(c.err);
      if (!dry) e = graph_layernorm_launch(x, y, g, b, eps, rows, d, st);
    }
  } else if (op.kind == "g_linear") {
    GraphLinearArgs a;
    a.rows = c.i("rows"); a.N = c.i("n"); a.K = c.i("k");
    a.ldx = c.i("ldx", a.K); a.ldy = c.i("ldy", a.N);
    a.int8 = (int)c.i("i8", 0);
    if (a.rows < 1 || a.N < 1 || a.K < 1 || a.ldx < a.K || a.ldy < a.N) return bad("g_linear: bad dimensions");
    a.x = (const float*)c.ptr("x", 4 * (size_t)((a.rows - 1) * a.ldx + a.K));
    a.w = c.ptr("w", (size_t)(a.N * a.K) * (a.int8 ? 1 : 2));
    a.scale = (const __half*)c.ptr("s", 2 * (size_t)a.N, !a.int8);
    a.bias = (const __half*)c.ptr("bias", 2 * (size_t)a.N, true);
    a.y = (float*)c.ptr("y", 4 * (size_t)((a.rows - 1) * a.ldy + a.N));
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_linear_launch(a, st);
  } else if (op.kind == "g_bmm") {
    GraphBmmArgs a;
    const auto bshape = c.ints("bshape"), sa = c.ints("sa"), sb = c.ints("sb");
    a.M = c.i("m"); a.N = c.i("n"); a.K = c.i("k");
    a.sam = c.i("sam"); a.sak = c.i("sak"); a.sbk = c.i("sbk"); a.sbn = c.i("sbn");
    a.round_b = (int)c.i("rb", 1);
    if (bshape.size() > (size_t)GRAPH_MAX_RANK || sa.size() != bshape.size() || sb.size() != bshape.size())
      return bad("g_bmm: bad batch shape / strides");
    if (a.M < 1 || a.N < 1 || a.K < 1) return bad("g_bmm: bad dimensions");
    a.brank = (int)bshape.size();
    fill_nd(bshape, a.bshape); fill_nd(sa, a.sa); fill_nd(sb, a.sb);
    a.batch = numel_of(bshape);
    std::vector<long long> ash(bshape), ast(sa), bsh(bshape), bst(sb);
    ash.push_back(a.M); ast.push_back(a.sam); ash.push_back(a.K); ast.push_back(a.sak);
    bsh.push_back(a.K); bst.push_back(a.sbk); bsh.push_back(a.N); bst.push_back(a.sbn);
    a.a = (const float*)c.ptr("a", 4 * view_span(ash, ast));
    a.b = (const float*)c.ptr("b", 4 * view_span(bsh, bst));
    a.y = (float*)c.ptr("y", 4 * (size_t)(a.batch * a.M * a.N));
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_bmm_launch(a, st);
  } else if (op.kind == "g_decode_ctx") {
    const int M = (int)c.i("m"), dh = (int)c.i("dh");
    const int* pos = (const int*)c.ptr("pos", 4);
    const __half* cos_t = (const __half*)c.ptr("cos", 2 * (size_t)M * dh, true);
    const __half* sin_t = (const __half*)c.ptr("sin", 2 * (size_t)M * dh, true);
    float* oh = (float*)c.ptr("oh", 4 * (size_t)M);
    float* inv = (float*)c.ptr("inv", 4 * (size_t)M);
    float* mask = (float*)c.ptr("mask", 4 * (size_t)M);
    float* cosp = (float*)c.ptr("cosp", 4 * (size_t)dh);
    float* sinp = (float*)c.ptr("sinp", 4 * (size_t)dh);
    if (M < 1 || dh < 1) return bad("g_decode_ctx: bad dimensions");
    if (!c.err.empty()) return bad(c.err);
    if (!dry) e = graph_decode_ctx_launch(pos, cos_t, sin_t, M, dh, oh, inv, mask, cosp, sinp, st);
  } else {
    return bad("unknown op kind '" + op.kind + "'");
  }
  return true;
}

// ------------------------------------------------------------------------------------ op launchers

static cudaError_t run_op(Program& p, const Op& op, bool dry, std::string& why) {
  OpCtx c{p, op, {}};
  cudaStream_t st = p.stream;
  const bool pdl = p.use_pdl;
  cudaError_t e = cudaSuccess;
  if (op.kind == "embed") {
    const int nb = c.i("nb"), d = c.i("d"), vocab = c.i("vocab"), ldh = c.i("ldh", d);
    const int* tok = (const int*)c.ptr("tok", 4 * (size_t)nb);
    const __half* table = (const __half*)c.ptr("table", 2 * (size_t)vocab * d);
    float* h = (float*)c.ptr("h", 4 * ((size_t)(nb - 1) * ldh + d));
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = embed_launch(tok, table, vocab, h, ldh, nb, d, p.d_err, st, pdl);
  } else if (op.kind == "layernorm") {
    const int nb = c.i("nb"), d = c.i("d");
    const int ldx = c.i("ldx", d), ldo = c.i("ldo", d);
    const float* x = (const float*)c.ptr("x", 4 * ((size_t)(nb - 1) * ldx + d));
    const __half* g = (const __half*)c.ptr("g", 2 * (size_t)d);
    const __half* b = (const __half*)c.ptr("b", 2 * (size_t)d, true);
    __half* out = (__half*)c.ptr("out", 2 * ((size_t)(nb - 1) * ldo + d));
    const float eps = (float)c.f("eps");
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = layernorm_launch(x, ldx, g, b, eps, out, ldo, nb, d, st, pdl);
  } else if (op.kind == "add_pos") {
    const int nb = c.i("nb"), d = c.i("d"), npos = c.i("npos");
    const int ldh = c.i("ldh", d);
    float* h = (float*)c.ptr("h", 4 * ((size_t)(nb - 1) * ldh + d));
    const __half* table = (const __half*)c.ptr("table", 2 * (size_t)npos * d);
    const int* pos = (const int*)c.ptr("pos", 4 * (size_t)nb, true);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = add_pos_launch(h, ldh, table, npos, pos, nb, d, p.d_err, st, pdl);
  } else if (op.kind == "rmsnorm") {
    const int nb = c.i("nb"), d = c.i("d"), xf16 = c.i("xf16", 0);
    const int ldx = c.i("ldx", d), ldo = c.i("ldo", d);
    const void* x = c.ptr("x", (xf16 ? 2 : 4) * ((size_t)(nb - 1) * ldx + d));
    const __half* g = (const __half*)c.ptr("g", 2 * (size_t)d);
    __half* out = (__half*)c.ptr("out", 2 * ((size_t)(nb - 1) * ldo + d));
    const float floor = (float)c.f("floor");
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    const L2Pf pf = parse_pf(c);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = rmsnorm_launch(x, xf16, ldx, g, floor, out, ldo, nb, d, st, pdl, pf);
  } else if (op.kind == "gemv" && c.has("wf") && (op.kv.at("wf") == "i8t" || op.kv.at("wf") == "i4t")) {
    GemvTcArgs a;
    const bool i4 = op.kv.at("wf") == "i4t";
    a.wf = i4 ? W_I4G32 : W_I8;
    const std::string* eps = c.raw("epi");
    if (!eps) { why = c.err; return cudaErrorInvalidValue; }
    a.epi = epi_of(*eps);
    if (a.epi < 0 || a.epi == EPI_ARGMAX) { why = "bad epi for a tiled gemv"; return cudaErrorInvalidValue; }
    a.NB = c.i("nb"); a.N = c.i("n"); a.K = c.i("k");
    a.ldx = c.i("ldx", a.K);
    const int out_cols = a.epi == EPI_SWIGLU ? a.N / 2 : a.N;
    a.ldy = c.i("ldy", out_cols);
    // a routed launch gathers x rows / scatters y rows among xrows / yrows rows (default nb)
    const int xrows = (int)c.i("xrows", a.NB), yrows = (int)c.i("yrows", a.NB);
    a.x = (const __half*)c.ptr("x", 2 * ((size_t)(xrows - 1) * a.ldx + a.K));
    // experts (MoE): E experts' tiles back to back, expert from `sel[slot]` or `fixe`
    const int nexp = (int)c.i("experts", 1);
    const size_t tile_bytes = i4 ? pack_i4_tiles_bytes(a.N, a.K) : pack_i8_tiles_bytes(a.N, a.K);
    a.w = c.ptr("w", tile_bytes * nexp);
    if (!i4) a.scale = (const __half*)c.ptr("s", 2 * (size_t)a.N * nexp);
    if (nexp > 1) {
      a.w_stride = (long long)tile_bytes;
      a.s_stride = i4 ? 0 : a.N;
      a.sel = (const int*)c.ptr("sel", 4 * ((size_t)c.i("slot", 0) + 1), true);
      a.slot = (int)c.i("slot", 0);
      a.fixed_e = (int)c.i("fixe", 0);
      if (a.fixed_e < 0 || a.fixed_e >= nexp) c.err = "fixe out of range";
      a.e_base = (int)c.i("ebase", 0);
      a.n_exp = nexp;
      if (a.e_base < 0) c.err = "ebase < 0";
    }
    // routed batch (moe_route lists): rows=, rcnt= over eg global experts, rld= rows per list,
    // r0= this launch's first list entry, route= 1 gather x / 2 scatter y
    a.route = (int)c.i("route", 0);
    if (a.route) {
      const int eg = (int)c.i("eg", a.e_base + nexp);
      a.rld = (int)c.i("rld");
      a.r0 = (int)c.i("r0", 0);
      a.rows = (const int*)c.ptr("rows", 4 * (size_t)eg * a.rld);
      a.rcnt = (const int*)c.ptr("rcnt", 4 * (size_t)eg);
      if (nexp <= 1 || a.sel) c.err = "route needs experts and fixe";
      if (a.route < 0 || a.route > 3 || a.NB > 16 || a.r0 < 0 || a.e_base + nexp > eg) c.err = "bad route";
      if (((a.route & 1) && xrows < a.rld) || ((a.route & 2) && yrows < a.rld)) c.err = "route rows exceed x / y";
    }
    a.rw_e = (int)c.i("rwe", 0);
    a.rw = (const float*)c.ptr("rw", 4 * (size_t)yrows * (a.rw_e > 0 ? a.rw_e : 1), true);
    if (a.rw && a.epi != EPI_RESID) c.err = "rw needs epi=resid";
    a.bias = (const __half*)c.ptr("bias", 2 * (size_t)a.N, true);
    const size_t esz = (a.epi == EPI_F16 || a.epi == EPI_SWIGLU) ? 2 : 4;
    a.y = c.ptr("y", esz * ((size_t)(yrows - 1) * a.ldy + out_cols));
    const bool want_gemm = c.i("gemm", 0) != 0;
    a.scratch_bytes = want_gemm ? 0 : gemv_tc_scratch_bytes(a.N, a.K, a.NB);
    if (a.scratch_bytes) a.scratch = c.ptr("scr", a.scratch_bytes);
    a.pf = parse_pf(c);
    a.err = p.d_err;
    static const int evict_first = env_int("AF_L2_EVICT_FIRST", 1);
    a.evict_first = (int)c.i("ef", evict_first);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    // prompt-sized row counts (prefill) run as a tensor-core GEMM unless the op asks for the GEMV
    const bool gemm = want_gemm && nexp == 1;
    if (!dry) e = gemm ? gemm_tc_launch(a, st, pdl) : gemv_tc_launch(a, st, pdl);
  } else if (op.kind == "gemv_chain") {
    // jobs=n nb= wf=i8t|i4t scr= and per job j: j<j>.{w,s,b,x,ldx,y,ldy,n,k,epi} plus an optional
    // norm run after the job: j<j>.{nx,ldnx,ng,nf,nout,ldno,nd}
    GemvChainArgs a;
    const std::string* wfs = c.raw("wf");
    if (!wfs || (*wfs != "i8t" && *wfs != "i4t")) { why = "gemv_chain: wf must be i8t or i4t"; return cudaErrorInvalidValue; }
    const bool i4 = *wfs == "i4t";
    a.wf = i4 ? W_I4G32 : W_I8;
    a.NB = (int)c.i("nb");
    a.njobs = (int)c.i("jobs");
    if (a.njobs < 1 || a.njobs > CHAIN_MAX_JOBS || a.NB < 1 || a.NB > 16) { why = "gemv_chain: bad jobs / nb"; return cudaErrorInvalidValue; }
    for (int j = 0; j < a.njobs && c.err.empty(); ++j) {
      ChainJob& J = a.job[j];
      const std::string p = "j" + std::to_string(j) + ".";
      auto K = [&](const char* s) { return p + s; };
      J.N = (int)c.i(K("n").c_str());
      J.K = (int)c.i(K("k").c_str());
      const std::string* es = c.raw(K("epi").c_str());
      if (!es) break;
      J.epi = epi_of(*es);
      if (J.epi < 0 || J.epi == EPI_ARGMAX) { c.err = "gemv_chain: bad epi"; break; }
      J.ldx = (int)c.i(K("ldx").c_str(), J.K);
      const int out_cols = J.epi == EPI_SWIGLU ? J.N / 2 : J.N;
      J.ldy = (int)c.i(K("ldy").c_str(), out_cols);
      J.x = (const __half*)c.ptr(K("x").c_str(), 2 * ((size_t)(a.NB - 1) * J.ldx + J.K));
      J.w = c.ptr(K("w").c_str(), i4 ? pack_i4_tiles_bytes(J.N, J.K) : pack_i8_tiles_bytes(J.N, J.K));
      if (!i4) J.scale = (const __half*)c.ptr(K("s").c_str(), 2 * (size_t)J.N);
      J.bias = (const __half*)c.ptr(K("b").c_str(), 2 * (size_t)J.N, true);
      const size_t esz = (J.epi == EPI_F16 || J.epi == EPI_SWIGLU) ? 2 : 4;
      J.y = c.ptr(K("y").c_str(), esz * ((size_t)(a.NB - 1) * J.ldy + out_cols));
      if (c.has(K("nx").c_str())) {
        J.nd = (int)c.i(K("nd").c_str());
        J.ldnx = (int)c.i(K("ldnx").c_str(), J.nd);
        J.ldno = (int)c.i(K("ldno").c_str(), J.nd);
        J.nx = (const float*)c.ptr(K("nx").c_str(), 4 * ((size_t)(a.NB - 1) * J.ldnx + J.nd));
        J.ng = (const __half*)c.ptr(K("ng").c_str(), 2 * (size_t)J.nd);
        J.nfloor = (float)c.f(K("nf").c_str());
        J.nout = (__half*)c.ptr(K("nout").c_str(), 2 * ((size_t)(a.NB - 1) * J.ldno + J.nd));
      }
    }
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    a.scratch_bytes = gemv_chain_scratch_bytes(a);
    a.scratch = c.ptr("scr", a.scratch_bytes);
    a.err = p.d_err;
    static const int evict_first = env_int("AF_L2_EVICT_FIRST", 1);
    a.evict_first = (int)c.i("ef", evict_first);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = gemv_chain_launch(a, st, pdl);
  } else if (op.kind == "gemv") {
    GemvArgs a;
    const std::string* wfs = c.raw("wf");
    const std::string* eps = c.raw("epi");
    if (!wfs || !eps) { why = c.err; return cudaErrorInvalidValue; }
    a.wf = wf_of(*wfs);
    a.epi = epi_of(*eps);
    if (a.wf < 0 || a.epi < 0) { why = "bad wf/epi"; return cudaErrorInvalidValue; }
    a.NB = c.i("nb"); a.N = c.i("n"); a.K = c.i("k");
    a.ldx = c.i("ldx", a.K);
    const int out_cols = a.epi == EPI_SWIGLU ? a.N / 2 : a.N;
    a.ldy = c.i("ldy", out_cols);
    a.x = (const __half*)c.ptr("x", 2 * ((size_t)(a.NB - 1) * a.ldx + a.K));
    const size_t wbytes = (a.wf == W_I8 || a.wf == W_I8G) ? (size_t)a.N * a.K
                          : a.wf == W_F16 ? (size_t)a.N * a.K * 2
                          : a.wf == W_SPARSE ? (size_t)a.N * (a.K / 32) * 4 : (size_t)a.N * a.K / 2;
    a.w = c.ptr("w", wbytes);
    if (a.wf == W_I8) a.scale = (const __half*)c.ptr("s", 2 * (size_t)a.N);
    if (a.wf == W_I4G32) a.gscale = (const __half*)c.ptr("gs", 2 * (size_t)a.N * (a.K / 32));
    if (a.wf == W_LUT4) a.gscale = (const __half*)c.ptr("gs", 2 * (size_t)a.N * 16);
    if (a.wf == W_I8G) {
      a.group = (int)c.i("grp", 32);
      if (a.group < 16 || a.group % 16 || a.K % a.group) c.err = "grp must be a multiple of 16 dividing k";
      else a.gscale = (const __half*)c.ptr("gs", 2 * (size_t)a.N * (a.K / a.group));
    }
    if (a.wf == W_SPARSE) {
      if (a.K % 32 || a.epi == EPI_ARGMAX) c.err = "sparse weights need k % 32 == 0 and no argmax epilogue";
      a.gscale = (const __half*)c.ptr("gs", 2 * (size_t)c.i("nnz"));
      a.rowoff = (const int*)c.ptr("ro", 4 * ((size_t)a.N + 1));
    }
    a.bias = (const __half*)c.ptr("bias", 2 * (size_t)a.N, true);
    const size_t esz = (a.epi == EPI_F16 || a.epi == EPI_SWIGLU) ? 2 : 4;
    a.y = c.ptr("y", esz * ((size_t)(a.NB - 1) * a.ldy + out_cols), a.epi == EPI_ARGMAX);
    if (a.epi == EPI_ARGMAX) {
      size_t slots = 0, counters = 0;
      gemv_argmax_scratch(a.wf, a.N, a.K, a.NB, &slots, &counters);
      a.am_val = (float*)c.ptr("amv", 4 * slots);
      a.am_idx = (int*)c.ptr("ami", 4 * slots);
      a.am_count = (int*)c.ptr("amc", 4 * counters);
      const int ctas = gemv_argmax_ctas(a.wf, a.N, a.K, a.NB);
      a.tok_out = (int*)c.ptr("tok", 4 * (size_t)a.NB);
      a.pos_adv = (int*)c.ptr("pos", 4 * (size_t)a.NB, true);
      a.hist_ld = (int)c.i("histld", 0);
      a.hist = (int*)c.ptr("hist", 4 * (size_t)a.NB * a.hist_ld, true);
      if (a.hist && !a.pos_adv) c.err = "hist needs pos";
      a.val_out = (float*)c.ptr("val", 4 * (size_t)a.NB, true);
      a.idx_base = (int)c.i("ibase", 0);
      a.am_grid_cap = ctas;
    }
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = gemv_launch(a, st, pdl);
  } else if (op.kind == "attn_decode" || op.kind == "kv_append") {
    AttnDecodeArgs a;
    a.NB = c.i("nb"); a.H = c.i("h"); a.KV = c.i("kv"); a.dh = c.i("dh"); a.M = c.i("m");
    a.n_split = c.i("nsplit", 1);
    a.ld_qkv = c.i("ldqkv", (a.H + 2 * a.KV) * a.dh);
    a.ld_out = c.i("ldo", a.H * a.dh);
    // seqrows: cache rows between sequences (absent: KV * M each; 0: all rows query one shared cache)
    a.kv_seq_rows = (int)c.i("seqrows", -1);
    a.write_kv = (int)c.i("wkv", 1);
    const size_t rows = a.kv_seq_rows < 0 ? (size_t)a.NB * a.KV * a.M
                                          : (size_t)(a.NB - 1) * a.kv_seq_rows + (size_t)a.KV * a.M;
    const size_t cache = 2 * rows * a.dh;
    if (op.kind == "kv_append") {
      a.qkv = (const float*)c.ptr("qkv", 4 * ((size_t)(a.NB - 1) * a.ld_qkv + (a.H + 2 * a.KV) * a.dh));
      a.kc = (__half*)c.ptr("kc", cache);
      a.vc = (__half*)c.ptr("vc", cache);
      a.pos = (const int*)c.ptr("pos", 4 * (size_t)a.NB);
      a.cos_t = (const __half*)c.ptr("cos", 2 * (size_t)a.M * a.dh, true);
      a.sin_t = (const __half*)c.ptr("sin", 2 * (size_t)a.M * a.dh, true);
      a.kn_g = (const __half*)c.ptr("kn", 2 * (size_t)a.dh, true);
      a.kn_floor = (float)c.f("knf", 0.0);
      a.err = p.d_err;
      if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
      if (!dry) e = kv_append_launch(a, st, pdl);
      if (e != cudaSuccess) why = std::string("launch failed: ") + cudaGetErrorString(e);
      return e;
    }
    a.qkv = (const float*)c.ptr("qkv", 4 * ((size_t)(a.NB - 1) * a.ld_qkv + (a.H + 2 * a.KV) * a.dh));
    a.kc = (__half*)c.ptr("kc", cache);
    a.vc = (__half*)c.ptr("vc", cache);
    a.pos = (const int*)c.ptr("pos", 4 * (size_t)a.NB);
    a.cos_t = (const __half*)c.ptr("cos", 2 * (size_t)a.M * a.dh, true);
    a.sin_t = (const __half*)c.ptr("sin", 2 * (size_t)a.M * a.dh, true);
    a.qn_g = (const __half*)c.ptr("qn", 2 * (size_t)a.dh, true);
    a.kn_g = (const __half*)c.ptr("kn", 2 * (size_t)a.dh, true);
    a.qn_floor = (float)c.f("qnf", 0.0);
    a.kn_floor = (float)c.f("knf", 0.0);
    a.out = (__half*)c.ptr("out", 2 * ((size_t)(a.NB - 1) * a.ld_out + a.H * a.dh));
    if (a.n_split > 1) {
      a.part = (float*)c.ptr("part", 4 * attn_decode_scratch_floats(a.NB, a.KV, a.n_split, a.H / a.KV, a.dh));
      a.counters = (int*)c.ptr("cnt", 4 * (size_t)a.NB * a.KV);
    }
    a.scale = (float)c.f("scale");
    a.kv_c = (float)c.f("kvc", 1.0);
    a.expand = c.i("expand", 0);
    a.prefetch = (int)c.i("prefetch", 0);
    // rows of a shared cache are written by the kv_append launch just before: none may be staged
    // before the launch wait
    if (a.kv_seq_rows == 0 && a.prefetch) c.err = "prefetch needs one cache per sequence";
    a.pf = parse_pf(c);
    a.err = p.d_err;
    if ((a.cos_t == nullptr) != (a.sin_t == nullptr)) c.err = "cos/sin must both be given";
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = attn_decode_launch(a, st, pdl);
  } else if (op.kind == "attn_prefill") {
    AttnPrefillArgs a;
    a.S = c.i("s"); a.H = c.i("h"); a.KV = c.i("kv"); a.dh = c.i("dh");
    a.ldm = c.i("ldm", a.S);
    a.ld_qkv = c.i("ldqkv", (a.H + 2 * a.KV) * a.dh);
    a.qkv = (const float*)c.ptr("qkv", 4 * ((size_t)(a.S - 1) * a.ld_qkv + (a.H + 2 * a.KV) * a.dh));
    a.kc = (__half*)c.ptr("kc", 2 * (size_t)a.KV * a.ldm * a.dh);
    a.vc = (__half*)c.ptr("vc", 2 * (size_t)a.KV * a.ldm * a.dh);
    a.cos_t = (const __half*)c.ptr("cos", 2 * (size_t)a.S * a.dh, true);
    a.sin_t = (const __half*)c.ptr("sin", 2 * (size_t)a.S * a.dh, true);
    a.qn_g = (const __half*)c.ptr("qn", 2 * (size_t)a.dh, true);
    a.kn_g = (const __half*)c.ptr("kn", 2 * (size_t)a.dh, true);
    a.qn_floor = (float)c.f("qnf", 0.0);
    a.kn_floor = (float)c.f("knf", 0.0);
    a.out = (__half*)c.ptr("out", 2 * (size_t)a.S * a.H * a.dh);
    __half* qbuf = (__half*)c.ptr("qbuf", 2 * (size_t)a.H * a.S * a.dh);
    a.scale = (float)c.f("scale");
    a.kv_c = (float)c.f("kvc", 1.0);
    a.expand = c.i("expand", 0);
    a.kvx = (__half*)c.ptr("kvx", 2 * 2 * (size_t)a.KV * a.S * a.dh, true);
    a.err = p.d_err;
    if (a.ldm < a.S) c.err = "ldm < s";
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) {
      e = rope_kv_prefill_launch(a, qbuf, st);
      if (e == cudaSuccess) e = attn_prefill_with_q(a, qbuf, st);
    }
  } else if (op.kind.compare(0, 2, "g_") == 0) {
    if (!graph_op(c, op, dry, st, e, why)) return cudaErrorInvalidValue;
  } else if (op.kind == "moe_gate") {
    const int nb = (int)c.i("nb"), E = (int)c.i("e"), k = (int)c.i("k"), ld = (int)c.i("ld", E);
    const float* lg = (const float*)c.ptr("logits", 4 * ((size_t)(nb - 1) * ld + E));
    float* gw = (float*)c.ptr("gw", 4 * (size_t)nb * E);
    int* sel = (int*)c.ptr("sel", 4 * (size_t)nb * k);
    const int renorm = (int)c.i("renorm", 1);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = moe_gate_launch(lg, ld, nb, E, k, renorm, gw, sel, st, pdl);
  } else if (op.kind == "moe_route") {
    // per-expert row lists of the batch: rows [e][rld], cnt [e]
    const int nb = (int)c.i("nb"), E = (int)c.i("e"), k = (int)c.i("k"), rld = (int)c.i("rld", nb);
    const int* sel = (const int*)c.ptr("sel", 4 * (size_t)nb * k);
    int* rows = (int*)c.ptr("rows", 4 * (size_t)E * rld);
    int* cnt = (int*)c.ptr("cnt", 4 * (size_t)E);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = moe_route_launch(sel, nb, k, E, rld, rows, cnt, st, pdl);
  } else if (op.kind == "allreduce" || op.kind == "allgather") {
    // fp32 sum over the ranks / int32 gather of n elements per rank, on the program's communicator
    const size_t n = (size_t)c.i("n");
    const int T = comm_size(p.comm);
    const bool red = op.kind == "allreduce";
    void* src = c.ptr("src", 4 * n);
    void* dst = c.ptr("dst", 4 * n * (red ? 1 : (size_t)c.i("ranks")));
    float* addto = red ? (float*)c.ptr("addto", 4 * n, true) : nullptr;     // allreduce: y += sum
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) {
      if (!p.comm) { why = op.kind + " needs a communicator (af_program_set_comm)"; return cudaErrorInvalidValue; }
      if (!red && c.i("ranks") != T) { why = "allgather: ranks does not match the communicator"; return cudaErrorInvalidValue; }
      e = red ? comm_all_reduce_f32(p.comm, (const float*)src, (float*)dst, n, st, why, p.d_err, addto, pdl)
              : comm_all_gather_i32(p.comm, (const int*)src, (int*)dst, n, st, why);
      if (e != cudaSuccess) return e;
    }
  } else if (op.kind == "allreduce_rms") {
    // tensor parallel: h += sum over the ranks of src, then out = rmsnorm(h) (one fused launch on
    // the peer-memory path; all-reduce + norm otherwise)
    const int nb = (int)c.i("nb"), d = (int)c.i("d");
    const size_t n = (size_t)nb * d;
    const float* src = (const float*)c.ptr("src", 4 * n);
    float* tmp = (float*)c.ptr("dst", 4 * n);
    float* h = (float*)c.ptr("h", 4 * n);
    const __half* g = (const __half*)c.ptr("g", 2 * (size_t)d);
    __half* out = (__half*)c.ptr("out", 2 * n);
    const float floor = (float)c.f("floor");
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) {
      if (!p.comm) { why = "allreduce_rms needs a communicator (af_program_set_comm)"; return cudaErrorInvalidValue; }
      e = comm_all_reduce_rms_f32(p.comm, src, tmp, h, nb, d, g, floor, out, st, why, p.d_err, pdl);
      if (e != cudaSuccess) return e;
    }
  } else if (op.kind == "tp_argmax") {
    const int T = (int)c.i("ranks"), nb = (int)c.i("nb");
    const int* g = (const int*)c.ptr("src", 4 * (size_t)T * 2 * nb);
    int* tok = (int*)c.ptr("tok", 4 * (size_t)nb);
    int* pos = (int*)c.ptr("pos", 4 * (size_t)nb, true);
    const int hist_ld = (int)c.i("histld", 0);
    int* hist = (int*)c.ptr("hist", 4 * (size_t)nb * hist_ld, true);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = tp_argmax_launch(g, T, nb, tok, pos, hist, hist_ld, st);
  } else if (op.kind == "add") {
    const size_t n = (size_t)c.i("n");
    float* y = (float*)c.ptr("y", 4 * n);
    const float* x = (const float*)c.ptr("x", 4 * n);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = add_f32_launch(y, x, n, st);
  } else if (op.kind == "cast") {
    const size_t n = (size_t)c.i("n");
    const int mode = (int)c.i("mode");
    const void* src = c.ptr("src", n * (mode == 0 ? 2 : 4));
    void* dst = c.ptr("dst", n * (mode == 0 ? 4 : 2));
    if (mode != 0 && mode != 1) c.err = "cast mode must be 0 or 1";
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = cast_launch(src, dst, n, mode, st, pdl);
  } else if (op.kind == "copy") {
    const size_t bytes = (size_t)c.i("bytes");
    void* dst = c.ptr("dst", bytes);
    const void* src = c.ptr("src", bytes);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st);
  } else if (op.kind == "fill") {
    const size_t bytes = (size_t)c.i("bytes");
    void* dst = c.ptr("dst", bytes);
    if (!c.err.empty()) { why = c.err; return cudaErrorInvalidValue; }
    if (!dry) e = cudaMemsetAsync(dst, (int)c.i("value", 0), bytes, st);
  } else {
    why = "unknown op kind '" + op.kind + "'";
    return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) {
    why = std::string("launch failed: ") + cudaGetErrorString(e) + " [";
    for (const auto& kv : op.kv) why += " " + kv.first + "=" + kv.second;
    why += " ]";
  }
  return e;
}

// ------------------------------------------------------------------------------------ parsing

static bool parse_plan(Program& p, const std::string& text, std::string& err) {
  std::istringstream in(text);
  std::string line;
  int ln = 0;
  bool header = false;
  while (std::getline(in, line)) {
    ++ln;
    auto hash = line.find('#');
    if (hash != std::string::npos) line = line.substr(0, hash);
    std::istringstream ls(line);
    std::string kw;
    if (!(ls >> kw)) continue;
    if (!header) {
      int ver = 0;
      if (kw != "AFPLAN" || !(ls >> ver) || ver != 1) { err = "plan must start with 'AFPLAN 1'"; return false; }
      header = true;
      continue;
    }
    if (kw == "buf") {
      Buffer b;
      std::string role;
      if (!(ls >> b.name >> b.bytes >> role) || !parse_role(role, b.role)) {
        err = "line " + std::to_string(ln) + ": bad buf statement";
        return false;
      }
      if (p.idx.count(b.name)) { err = "line " + std::to_string(ln) + ": duplicate buffer " + b.name; return false; }
      p.idx[b.name] = (int)p.bufs.size();
      p.bufs.push_back(b);
    } else if (kw == "wfile") {
      std::string name;
      long long off;
      if (!(ls >> name >> off) || find_buf(p, name) < 0) { err = "line " + std::to_string(ln) + ": bad wfile"; return false; }
      p.bufs[find_buf(p, name)].file_off = off;
    } else if (kw == "op") {
      Op op;
      op.line = ln;
      if (!(ls >> op.kind)) { err = "line " + std::to_string(ln) + ": op without kind"; return false; }
      std::string tok;
      while (ls >> tok) {
        auto eq = tok.find('=');
        if (eq == std::string::npos) { err = "line " + std::to_string(ln) + ": expected key=value, got " + tok; return false; }
        op.kv[tok.substr(0, eq)] = tok.substr(eq + 1);
      }
      p.ops.push_back(op);
    } else {
      err = "line " + std::to_string(ln) + ": unknown statement " + kw;
      return false;
    }
  }
  if (!header) { err = "empty plan"; return false; }
  return true;
}

static bool alloc_buffers(Program& p, std::string& err) {
  for (auto& b : p.bufs) {
    const size_t bytes = ((b.bytes + 255) / 256) * 256;
    if (bytes == 0) continue;
    cudaError_t e = cudaMalloc(&b.dev, bytes);
    if (e != cudaSuccess) { err = "cudaMalloc(" + b.name + ", " + std::to_string(bytes) + ") failed: " + cudaGetErrorString(e); return false; }
    b.owned = true;
    if (b.role != R_WEIGHT) {
      cudaMemset(b.dev, 0, bytes);   // ports and state start zeroed, like the e5rt ports
      b.ready = true;
    }
  }
  cudaError_t e = cudaMalloc(&p.d_err, 256);
  if (e != cudaSuccess) { err = "cudaMalloc(err) failed"; return false; }
  cudaMemset(p.d_err, 0, 256);
  return true;
}

static bool load_weight_file(Program& p, std::string& err) {
  bool any = false;
  for (auto& b : p.bufs) any |= b.file_off >= 0;
  if (!any) return true;
  std::ifstream f(p.dir + "/weights.bin", std::ios::binary);
  if (!f) { err = "cannot open " + p.dir + "/weights.bin"; return false; }
  std::vector<char> tmp;
  for (auto& b : p.bufs) {
    if (b.file_off < 0) continue;
    tmp.resize(b.bytes);
    f.seekg(b.file_off);
    f.read(tmp.data(), (std::streamsize)b.bytes);
    if (!f) { err = "short read of weight " + b.name; return false; }
    cudaError_t e = cudaMemcpy(b.dev, tmp.data(), b.bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { err = "upload of " + b.name + " failed"; return false; }
    b.ready = true;
  }
  return true;
}

static void free_program(Program* p) {
  if (!p) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  if (p->stream) cudaStreamSynchronize(p->stream);
  if (p->exec) cudaGraphExecDestroy(p->exec);
  for (auto& b : p->bufs)
    if (b.owned && b.dev) cudaFree(b.dev);
  if (p->d_err) cudaFree(p->d_err);
  if (p->stream) cudaStreamDestroy(p->stream);
  cudaSetDevice(prev);
  delete p;
}

static int device_from_mask(uint64_t mask) {
  if (mask == 0) {
    int d = 0;
    cudaGetDevice(&d);
    return d;
  }
  for (int i = 0; i < 64; ++i)
    if (mask & (1ull << i)) return i;
  return 0;
}

struct DeviceGuard {
  int prev = 0;
  explicit DeviceGuard(int d) { cudaGetDevice(&prev); cudaSetDevice(d); }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

static Program* build_program(const std::string& text, const std::string& dir, uint64_t mask) {
  Program* p = new Program();
  p->dir = dir;
  p->device = device_from_mask(mask);
  std::string err;
  if (!parse_plan(*p, text, err)) { set_error("plan parse: " + err); delete p; return nullptr; }
  // validate every op against the declared buffers before touching the device
  for (auto& op : p->ops) {
    std::string why;
    // dry validation needs buffer sizes only; device pointers are still null
    if (run_op(*p, op, true, why) != cudaSuccess) {
      set_error("plan line " + std::to_string(op.line) + " (" + op.kind + "): " + why);
      delete p;
      return nullptr;
    }
  }
  DeviceGuard g(p->device);
  if (cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("cudaStreamCreate failed");
    delete p;
    return nullptr;
  }
  if (!alloc_buffers(*p, err) || !load_weight_file(*p, err)) { set_error(err); free_program(p); return nullptr; }
  if (getenv("AF_CUDA_NO_GRAPH")) p->use_graph = false;
  if (getenv("AF_CUDA_NO_PDL")) p->use_pdl = false;
  return p;
}

static int launch_all(Program& p) {
  for (auto& op : p.ops) {
    std::string why;
    if (run_op(p, op, false, why) != cudaSuccess) {
      set_error("op line " + std::to_string(op.line) + " (" + op.kind + "): " + why);
      return -1;
    }
  }
  return 0;
}

static int finalize(Program& p) {
  for (auto& b : p.bufs)
    if (b.role == R_WEIGHT && !b.ready && b.alias_of < 0) {
      set_error("weight buffer '" + b.name + "' was never uploaded or bound");
      return -1;
    }
  if (p.use_graph) {
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(p.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      set_error("stream capture failed to start");
      return -1;
    }
    const int rc = launch_all(p);
    cudaError_t e = cudaStreamEndCapture(p.stream, &graph);
    if (rc != 0 || e != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      if (rc == 0) set_error(std::string("stream capture failed: ") + cudaGetErrorString(e));
      cudaGetLastError();
      return -1;
    }
    e = cudaGraphInstantiate(&p.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) { set_error(std::string("graph instantiate failed: ") + cudaGetErrorString(e)); return -1; }
  }
  p.finalized = true;
  return 0;
}

static int check_err(Program& p) {
  int h = 0;
  if (cudaMemcpyAsync(&h, p.d_err, 4, cudaMemcpyDeviceToHost, p.stream) != cudaSuccess ||
      cudaStreamSynchronize(p.stream) != cudaSuccess) {
    set_error(std::string("device failure: ") + cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  if (h != 0) {
    static const char* names[] = {"ok", "token id out of range", "decode position out of range", "bounded wait timed out"};
    set_error(std::string("kernel reported error ") + std::to_string(h) + " (" + (h > 0 && h < 4 ? names[h] : "?") + ")");
    cudaMemsetAsync(p.d_err, 0, 4, p.stream);
    cudaStreamSynchronize(p.stream);
    return -2;
  }
  return 0;
}

static int execute(Program& p, bool sync) {
  DeviceGuard g(p.device);
  if (!p.finalized && finalize(p) != 0) return -1;
  cudaError_t e;
  if (p.use_graph) {
    e = cudaGraphLaunch(p.exec, p.stream);
    if (e != cudaSuccess) { set_error(std::string("graph launch failed: ") + cudaGetErrorString(e)); return -1; }
  } else if (launch_all(p) != 0) {
    return -1;
  }
  return sync ? check_err(p) : 0;
}

static Buffer* port(Program& p, const char* name, bool input) {
  int i = find_buf(p, name);
  if (i < 0) return nullptr;
  Buffer& b = p.bufs[i];
  if (input && !(b.role == R_IN || b.role == R_STATE)) return nullptr;
  if (!input && b.role != R_OUT) return nullptr;
  return &b;
}

static Buffer& root(Program& p, Buffer& b) {
  int i = (int)(&b - p.bufs.data());
  while (p.bufs[i].alias_of >= 0) i = p.bufs[i].alias_of;
  return p.bufs[i];
}

}  // namespace af

using namespace af;

// ============================================================================= C ABI

extern "C" {

const char* af_last_error(void) { return g_last_error.c_str(); }

int af_abi_version(void) { return AF_CUDA_ABI_VERSION; }

void* af_program_compile(const char* program_path, const char* cache_dir, uint64_t device_mask,
                         const char* const* in_names, const size_t* in_bytes, size_t n_in,
                         const char* const* out_names, const size_t* out_bytes, size_t n_out) {
  (void)cache_dir;
  if (!program_path) { set_error("null program path"); return nullptr; }
  std::string dir(program_path);
  std::ifstream f(dir + "/plan.txt");
  if (!f) { set_error("cannot open " + dir + "/plan.txt"); return nullptr; }
  std::stringstream ss;
  ss << f.rdbuf();
  Program* p = build_program(ss.str(), dir, device_mask);
  if (!p) return nullptr;
  // the declared ports must match the plan's (names, roles, sizes)
  for (size_t i = 0; i < n_in; ++i) {
    Buffer* b = port(*p, in_names[i], true);
    if (!b || b->bytes < in_bytes[i]) {
      set_error(std::string("input port '") + in_names[i] + "' missing or smaller than declared");
      free_program(p);
      return nullptr;
    }
  }
  for (size_t i = 0; i < n_out; ++i) {
    Buffer* b = port(*p, out_names[i], false);
    if (!b || b->bytes < out_bytes[i]) {
      set_error(std::string("output port '") + out_names[i] + "' missing or smaller than declared");
      free_program(p);
      return nullptr;
    }
  }
  return p;
}

void* af_program_compile_text(const char* plan_text, const char* weights_dir, uint64_t device_mask) {
  if (!plan_text) { set_error("null plan"); return nullptr; }
  return build_program(plan_text, weights_dir ? weights_dir : ".", device_mask);
}

int af_compile_check(const char* program_path, const char* cache_dir, uint64_t device_mask,
                     const char* custom_options) {
  (void)cache_dir; (void)device_mask; (void)custom_options;
  std::ifstream f(std::string(program_path ? program_path : "") + "/plan.txt");
  if (!f) { set_error("cannot open plan"); return -1; }
  std::stringstream ss;
  ss << f.rdbuf();
  Program p;
  std::string err;
  if (!parse_plan(p, ss.str(), err)) { set_error(err); return -1; }
  for (auto& op : p.ops) {
    std::string why;
    if (run_op(p, op, true, why) != cudaSuccess) { set_error(why); return -1; }
  }
  return 0;
}

static int copy_in(void* h, const char* name, const void* src, size_t nbytes, bool any_buffer, size_t off) {
  if (!h || !name || (!src && nbytes)) return -1;
  Program& p = *static_cast<Program*>(h);
  Buffer* b = nullptr;
  if (any_buffer) {
    int i = find_buf(p, name);
    b = i < 0 ? nullptr : &p.bufs[i];
  } else {
    b = port(p, name, true);
  }
  if (!b) { set_error(std::string("unknown input port '") + name + "'"); return -1; }
  Buffer& r = root(p, *b);
  if (off + nbytes > r.bytes) { set_error(std::string("copy into '") + name + "' exceeds its size"); return -1; }
  DeviceGuard g(p.device);
  if (cudaMemcpyAsync(static_cast<char*>(r.dev) + off, src, nbytes, cudaMemcpyHostToDevice, p.stream) != cudaSuccess ||
      cudaStreamSynchronize(p.stream) != cudaSuccess) {
    set_error(std::string("upload to '") + name + "' failed");
    return -1;
  }
  r.ready = true;
  return 0;
}

int af_program_set_input_fp16(void* h, const char* port_name, const uint16_t* src, size_t n_elems) {
  return copy_in(h, port_name, src, 2 * n_elems, false, 0);
}

int af_program_set_input_bytes(void* h, const char* port_name, const void* src, size_t nbytes) {
  return copy_in(h, port_name, src, nbytes, false, 0);
}

int af_program_upload(void* h, const char* name, const void* src, size_t nbytes, size_t offset) {
  return copy_in(h, name, src, nbytes, true, offset);
}

static int copy_out(void* h, const char* name, void* dst, size_t nbytes, bool any_buffer) {
  if (!h || !name || !dst) return -1;
  Program& p = *static_cast<Program*>(h);
  Buffer* b = nullptr;
  if (any_buffer) {
    int i = find_buf(p, name);
    b = i < 0 ? nullptr : &p.bufs[i];
  } else {
    b = port(p, name, false);
  }
  if (!b) { set_error(std::string("unknown output port '") + name + "'"); return -1; }
  Buffer& r = root(p, *b);
  const size_t n = nbytes < r.bytes ? nbytes : r.bytes;
  DeviceGuard g(p.device);
  if (cudaMemcpyAsync(dst, r.dev, n, cudaMemcpyDeviceToHost, p.stream) != cudaSuccess ||
      cudaStreamSynchronize(p.stream) != cudaSuccess) {
    set_error(std::string("download of '") + name + "' failed");
    return -1;
  }
  return 0;
}

int af_program_get_output_fp16(void* h, const char* port_name, uint16_t* dst, size_t n_elems) {
  return copy_out(h, port_name, dst, 2 * n_elems, false);
}

int af_program_get_output_bytes(void* h, const char* port_name, void* dst, size_t nbytes) {
  return copy_out(h, port_name, dst, nbytes, false);
}

int af_program_download(void* h, const char* name, void* dst, size_t nbytes) {
  return copy_out(h, name, dst, nbytes, true);
}

static int buffer_of(void* h, const char* name, void** ptr, size_t* bytes, int want) {
  if (!h || !name || !ptr || !bytes) return -1;
  Program& p = *static_cast<Program*>(h);
  Buffer* b = nullptr;
  if (want == 0) b = port(p, name, true);
  else if (want == 1) b = port(p, name, false);
  else {
    int i = find_buf(p, name);
    b = i < 0 ? nullptr : &p.bufs[i];
  }
  if (!b) { set_error(std::string("unknown buffer '") + name + "'"); return -1; }
  Buffer& r = root(p, *b);
  *ptr = r.dev;
  *bytes = r.bytes;
  return 0;
}

int af_program_input_buffer(void* h, const char* port_name, void** ptr, size_t* bytes) {
  return buffer_of(h, port_name, ptr, bytes, 0);
}

int af_program_output_buffer(void* h, const char* port_name, void** ptr, size_t* bytes) {
  return buffer_of(h, port_name, ptr, bytes, 1);
}

int af_program_buffer(void* h, const char* name, void** ptr, size_t* bytes) {
  return buffer_of(h, name, ptr, bytes, 2);
}

int af_program_bind_buffer(void* h, const char* name, void* dev, size_t bytes) {
  if (!h || !name || !dev) return -1;
  Program& p = *static_cast<Program*>(h);
  if (p.finalized) { set_error("bind_buffer after the first execute"); return -1; }
  int i = find_buf(p, name);
  if (i < 0) { set_error(std::string("unknown buffer '") + name + "'"); return -1; }
  Buffer& b = p.bufs[i];
  if (bytes < b.bytes) { set_error(std::string("bound memory smaller than buffer '") + name + "'"); return -1; }
  if ((reinterpret_cast<uintptr_t>(dev) & 15) != 0) { set_error("bound memory must be 16-byte aligned"); return -1; }
  DeviceGuard g(p.device);
  if (b.owned && b.dev) cudaFree(b.dev);
  b.dev = dev;
  b.owned = false;
  b.ready = true;
  return 0;
}

int af_program_execute(void* h) {
  if (!h) return -1;
  return execute(*static_cast<Program*>(h), true);
}

int af_program_execute_async(void* h) {
  if (!h) return -1;
  return execute(*static_cast<Program*>(h), false);
}

int af_program_sync(void* h) {
  if (!h) return -1;
  Program& p = *static_cast<Program*>(h);
  DeviceGuard g(p.device);
  return check_err(p);
}

int af_program_stream(void* h, void** stream) {
  if (!h || !stream) return -1;
  *stream = static_cast<Program*>(h)->stream;
  return 0;
}

int af_program_set_comm(void* h, void* comm) {
  if (!h) return -1;
  Program& p = *static_cast<Program*>(h);
  if (p.finalized) { set_error("set_comm after the first execute"); return -1; }
  p.comm = comm;
  return 0;
}

int af_program_set_options(void* h, int use_graph, int use_pdl) {
  if (!h) return -1;
  Program& p = *static_cast<Program*>(h);
  if (p.finalized) { set_error("set_options after the first execute"); return -1; }
  p.use_graph = use_graph != 0;
  p.use_pdl = use_pdl != 0;
  return 0;
}

int af_program_share_buffer(void* h, size_t src_op, const char* src_out, size_t dst_op, const char* dst_in) {
  if (!h || !src_out || !dst_in) return -1;
  Program& p = *static_cast<Program*>(h);
  if (src_op != 0 || dst_op != 0) { set_error("share_buffer: a program has one op index (0)"); return -1; }
  if (p.finalized) { set_error("share_buffer after the first execute"); return -1; }
  Buffer* o = port(p, src_out, false);
  Buffer* in = port(p, dst_in, true);
  if (!o || !in) { set_error("share_buffer: unknown port"); return -1; }
  Buffer& ro = root(p, *o);
  if (ro.bytes < in->bytes) { set_error("share_buffer: source smaller than destination"); return -1; }
  DeviceGuard g(p.device);
  if (in->owned && in->dev) cudaFree(in->dev);   // the destination's own buffer is freed exactly once
  in->dev = nullptr;
  in->owned = false;
  in->alias_of = (int)(&ro - p.bufs.data());
  return 0;
}

void af_program_release(void* h) { free_program(static_cast<Program*>(h)); }

}  // extern "C"
