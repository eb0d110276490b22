// Device-resident graph executor (tysor_cuda_graph_* in include/tysor_cuda.h).
//
// One executor object holds one lowered graph.  Planning walks the graph
// once on the host, exactly in the order of the reference interpreters
// (runtime/graph_executor.rs:249-356 for --run, training/backward.rs:145-380
// for --backward, training/executor.rs:252-816 for --train): it evaluates
// constants and layer constructors, infers every tensor shape, reports the
// reference's errors, and records a list of device steps.  All tensors live
// in one device arena laid out after planning; reshape and flatten_heads are
// views.  Executing a plan only enqueues kernels on the context stream; a
// train step (forward, backward, optional gradient all-reduce, SGD) is
// captured once as a CUDA graph and replayed.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/tysor_cuda.h"
#include "context.cuh"
#include "ops.cuh"

namespace tysor {
namespace {

enum VKind { kVTensor, kVInt, kVFloat, kVBool, kVCallable };
enum NKind { kNConst, kNBinary, kNPrimitive, kNCall, kNCtor, kNApply };
enum Mode { kModeRun = 0, kModeBackward = 1, kModeTrain = 2 };

struct GValue {
  int id = 0;
  VKind kind = kVTensor;
  bool is_param = false;
  std::string name;
};

struct GNode {
  NKind kind = kNConst;
  int output = 0;
  std::string op;
  char binop = '+';
  int ckind = 0;  // const: 0 int, 1 float, 2 bool
  int64_t ival = 0;
  double fval = 0;
  std::vector<int> inputs;
};

// A region of the device arena.  Views point into their base.
struct Slot {
  size_t n = 0;
  Slot* base = nullptr;
  size_t offset = 0;
  float* p = nullptr;
};

struct HVal {
  enum T { None, Int, Float, Bool, Tensor, Linear, Embedding, Act, RmsNorm } t = None;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::vector<int64_t> shape;
  Slot* slot = nullptr;
  // closures
  int64_t in_features = -1, out_features = 0;
  bool with_bias = true;
  int64_t num = 0, dim = 0, hidden = 0;
  std::string act;
  double prob = 0, eps = 1e-5;
  int ctor_id = -1;
};

// A causal softmax's per-row masked probabilities (launch_masked_softmax's
// `leak`) for a GEMM that skips masked entries: the terms of rows where they
// are not zero are added back after it (launch_causal_leak_fix).
struct LeakFix {
  Slot* leak = nullptr;
  int64_t rows = 0;  // softmax rows per batch item
  int mode = 0;      // 2: O = P.V; 3: dV = P^T.dO
};

struct Param {
  std::vector<int64_t> shape;
  Slot* value = nullptr;
  Slot* grad = nullptr;
  bool grad_written = false;
  // Backward items that must run before the gradient is final (the index
  // just past the last item that writes it).
  size_t grad_ready = 0;
  // initialiser: 0 linear weight, 1 linear bias, 2 embedding weight, 3 ones
  int init = 0;
};

using StepFn = std::function<void(cudaStream_t)>;

// A step list whose items carry the label of the graph node being planned
// when they were added (for the traced step's per-op report).
struct StepList {
  std::vector<StepFn> fns;
  std::vector<std::string> labels;
  const std::string* cur = nullptr;
  void push_back(StepFn f) {
    fns.push_back(std::move(f));
    labels.push_back(cur ? *cur : std::string());
  }
  void clear() {
    fns.clear();
    labels.clear();
  }
  size_t size() const { return fns.size(); }
  std::vector<StepFn>::const_iterator begin() const { return fns.begin(); }
  std::vector<StepFn>::const_iterator end() const { return fns.end(); }
};

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); ++i) o << (i ? ", " : "") << s[i];
  o << "]";
  return o.str();
}

[[noreturn]] void fail(const std::string& m) { throw CudaError(m); }

struct Executor {
  Context* ctx = nullptr;
  std::vector<GValue> values;
  std::vector<GNode> nodes;
  std::vector<int> outputs;
  int objective = -1;
  std::map<std::string, std::vector<int64_t>> shapes;
  std::map<std::string, std::vector<float>> inputs;
  std::map<std::string, std::vector<float>> param_init;

  // plan
  int mode = -1;
  bool dirty = true;
  std::deque<Slot> slots;
  std::vector<HVal> hv;
  std::vector<StepFn> setup;      // once per plan: constant weights, parameter init
  std::vector<std::pair<std::string, StepFn>> upload;  // once per call: graph inputs
  std::set<std::string> device_inputs;  // inputs last written by upload_input
  std::string cur_label;         // node being planned (labels step items)
  StepList forward{{}, {}, &cur_label};   // every step
  StepList backward{{}, {}, &cur_label};  // every step
  StepList update{{}, {}, &cur_label};    // every train step
  std::map<int, Slot*> vgrad;
  std::map<std::string, Param> params;
  std::vector<std::string> param_order;
  Slot* loss = nullptr;           // one float per step
  Slot* grad_block = nullptr;     // all parameter gradients + loss, contiguous
  Slot* param_block = nullptr;    // the trained parameters, laid out like their gradients
  size_t param_block_n = 0;       // floats of param_block (its padding included)
  size_t scratch_floats = 0;
  Slot* scratch = nullptr;
  void* arena = nullptr;
  bool setup_done = false;
  bool stepped = false;  // a train step of this plan has run eagerly
  bool capture = true;
  bool allreduce = false;
  cudaGraphExec_t exec = nullptr;
  int64_t last_launches = 0;
  int64_t step_launches = 0;   // kernels of one train step (forward, backward, update)
  std::vector<std::string> trace_labels;  // item labels of the last traced step
  float* loss_hist = nullptr;  // per-step losses of one train call (device)
  int loss_hist_cap = 0;

  // Prefetched inputs: two device staging buffers per input, filled from
  // host memory on a copy stream while earlier steps compute, and copied
  // into the input's buffer (a kernel on the compute stream) at the start of
  // the next run / backward / train call.
  struct Staging {
    float* buf = nullptr;
    size_t n = 0;
    cudaEvent_t copied = nullptr;    // the host-to-device copy landed
    cudaEvent_t consumed = nullptr;  // the compute stream has copied it out
    bool used = false;               // `consumed` has been recorded
  };
  struct PrefetchQueue {
    Staging st[2];
    int next = 0;            // buffer the next prefetch fills
    std::deque<int> ready;   // filled buffers, oldest first
  };
  std::map<std::string, PrefetchQueue> prefetch;
  cudaStream_t copy_stream = nullptr;

  void prefetch_input(const std::string& name, Slot* s, const float* data, size_t count) {
    PrefetchQueue& pq = prefetch[name];
    if (pq.ready.size() >= 2) throw CudaError("input '" + name + "' already has two prefetched values waiting");
    if (!copy_stream) TYSOR_CUDA(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking));
    const int k = pq.next;
    Staging& b = pq.st[k];
    if (b.n != count) {
      if (b.buf) {
        TYSOR_CUDA(cudaStreamSynchronize(copy_stream));
        TYSOR_CUDA(cudaStreamSynchronize(ctx->stream));
        TYSOR_CUDA(cudaFree(b.buf));
      }
      b.buf = nullptr;
      b.used = false;
      TYSOR_CUDA(cudaMalloc(&b.buf, sizeof(float) * (count ? count : 1)));
      b.n = count;
    }
    if (!b.copied) TYSOR_CUDA(cudaEventCreateWithFlags(&b.copied, cudaEventDisableTiming));
    if (!b.consumed) TYSOR_CUDA(cudaEventCreateWithFlags(&b.consumed, cudaEventDisableTiming));
    // The buffer's previous value must have been copied out first.
    if (b.used) TYSOR_CUDA(cudaStreamWaitEvent(copy_stream, b.consumed, 0));
    TYSOR_CUDA(cudaMemcpyAsync(b.buf, data, sizeof(float) * count, cudaMemcpyHostToDevice, copy_stream));
    TYSOR_CUDA(cudaEventRecord(b.copied, copy_stream));
    pq.ready.push_back(k);
    pq.next = 1 - k;
    (void)s;
  }

  // Stored inputs (pattern or set_input values) unless a device value was
  // uploaded, then the oldest prefetched value of each input.
  void run_uploads() {
    for (auto& [name, fn] : upload)
      if (!device_inputs.count(name)) fn(ctx->stream);
    for (auto& [name, pq] : prefetch) {
      if (pq.ready.empty()) continue;
      Staging& b = pq.st[pq.ready.front()];
      pq.ready.pop_front();
      Slot* dst = input_slot(name);
      if (!dst || dst->n != b.n) throw CudaError("prefetched input '" + name + "' no longer matches its buffer");
      TYSOR_CUDA(cudaStreamWaitEvent(ctx->stream, b.copied, 0));
      launch_unary(kUnaryCopy, b.buf, dst->p, (int64_t)b.n, 0.0f, ctx->stream);
      TYSOR_CUDA(cudaEventRecord(b.consumed, ctx->stream));
      b.used = true;
    }
  }

  // The device buffer of graph input `name` (null if there is none).
  Slot* input_slot(const std::string& name) {
    for (const GValue& v : values)
      if (v.is_param && v.name == name) return v.id < (int)hv.size() ? hv[v.id].slot : nullptr;
    return nullptr;
  }

  ~Executor() {
    release();
    if (loss_hist) cudaFree(loss_hist);
    if (copy_stream) cudaStreamSynchronize(copy_stream);
    for (auto& [name, pq] : prefetch)
      for (Staging& b : pq.st) {
        if (b.buf) cudaFree(b.buf);
        if (b.copied) cudaEventDestroy(b.copied);
        if (b.consumed) cudaEventDestroy(b.consumed);
      }
    if (copy_stream) cudaStreamDestroy(copy_stream);
    for (Bucket& b : buckets)
      if (b.ready_ev) cudaEventDestroy(b.ready_ev);
    if (comm_stream) {
      cudaStreamSynchronize(comm_stream);
      cudaStreamDestroy(comm_stream);
    }
    if (comm_done) cudaEventDestroy(comm_done);
  }

  void release() {
    if (exec) cudaGraphExecDestroy(exec);
    exec = nullptr;
    if (arena) cudaFree(arena);
    arena = nullptr;
    slots.clear();
    hv.clear();
    setup.clear();
    upload.clear();
    forward.clear();
    backward.clear();
    update.clear();
    vgrad.clear();
    params.clear();
    param_order.clear();
    prep_cache.clear();
    pack_cache.clear();
    lazy_lo.clear();
    deferred_matmul.clear();
    folded_scale.clear();
    masked_input.clear();
    fused_silu.clear();
    residual_sum.clear();
    residual_lin.clear();
    seqmajor_transpose.clear();
    causal_scores.clear();
    causal_probs.clear();
    causal_leak.clear();
    folded_transpose.clear();
    grad_alias.clear();
    loss = grad_block = scratch = param_block = nullptr;
    param_block_n = 0;
    scratch_floats = 0;
    setup_done = false;
    stepped = false;
    // The input buffers are new: every input comes from its host copy again
    // until upload_input writes it.
    device_inputs.clear();
  }

  Slot* alloc(size_t n) {
    slots.push_back(Slot{n, nullptr, 0, nullptr});
    return &slots.back();
  }
  Slot* view(Slot* base, size_t offset, size_t n) {
    while (base->base) {
      offset += base->offset;
      base = base->base;
    }
    slots.push_back(Slot{n, base, offset, nullptr});
    return &slots.back();
  }
  void need_scratch(size_t floats) {
    if (floats > scratch_floats) scratch_floats = floats;
  }

  // ---- parsing ------------------------------------------------------------
  void parse(const char* text) {
    std::istringstream in(text);
    std::string line;
    while (std::getline(in, line)) {
      std::istringstream ls(line);
      std::string tag;
      if (!(ls >> tag)) continue;
      if (tag == "graph") continue;
      if (tag == "end") break;
      if (tag == "value") {
        GValue v;
        std::string kind, name;
        int param;
        ls >> v.id >> kind >> param >> name;
        if (kind == "tensor") v.kind = kVTensor;
        else if (kind == "int") v.kind = kVInt;
        else if (kind == "float") v.kind = kVFloat;
        else if (kind == "bool") v.kind = kVBool;
        else v.kind = kVCallable;
        v.is_param = param != 0;
        v.name = name == "-" ? "" : name;
        if (v.id != (int)values.size()) fail("graph text: value ids must be dense and ordered");
        values.push_back(v);
      } else if (tag == "node") {
        GNode n;
        std::string kind;
        ls >> kind >> n.output;
        if (kind == "const") {
          std::string ck;
          ls >> ck;
          if (ck == "int") {
            n.ckind = 0;
            ls >> n.ival;
          } else if (ck == "float") {
            n.ckind = 1;
            std::string s;
            ls >> s;
            n.fval = strtod(s.c_str(), nullptr);
          } else {
            n.ckind = 2;
            ls >> n.ival;
          }
          n.kind = kNConst;
        } else if (kind == "binary") {
          std::string op;
          ls >> op;
          n.binop = op[0];
          n.kind = kNBinary;
        } else if (kind == "apply") {
          n.kind = kNApply;
        } else {
          ls >> n.op;
          n.kind = kind == "primitive" ? kNPrimitive : kind == "call" ? kNCall : kNCtor;
        }
        int x;
        while (ls >> x) n.inputs.push_back(x);
        for (int i : n.inputs)
          if (i < 0 || i >= (int)values.size()) fail("graph text: input id out of range");
        if (n.output < 0 || n.output >= (int)values.size()) fail("graph text: output id out of range");
        nodes.push_back(n);
      } else if (tag == "output") {
        int o;
        ls >> o;
        outputs.push_back(o);
      } else if (tag == "objective") {
        ls >> objective;
      }
    }
    if (values.empty()) fail("graph text: no values");
  }

  // ---- helpers over planning values ----------------------------------------
  const HVal& val(int id) const { return hv.at(id); }
  const HVal& tensor(int id, const char* /*what*/) const {
    const HVal& h = hv.at(id);
    if (h.t != HVal::Tensor) fail("Graph executor expected tensor value");
    return h;
  }
  static double number(const HVal& h) {
    switch (h.t) {
      case HVal::Int: return (double)h.i;
      case HVal::Float: return h.f;
      case HVal::Bool: return h.b ? 1.0 : 0.0;
      default: fail("Graph executor expected scalar value");
    }
  }
  static int64_t integer(const HVal& h) {
    if (h.t != HVal::Int) fail("Graph executor expected integer value");
    return h.i;
  }
  static bool boolean(const HVal& h) {
    if (h.t != HVal::Bool) fail("Graph executor expected bool value");
    return h.b;
  }

  HVal new_tensor(std::vector<int64_t> shape) {
    HVal h;
    h.t = HVal::Tensor;
    h.shape = std::move(shape);
    h.slot = alloc((size_t)numel(h.shape));
    return h;
  }

  // ---- parameters ---------------------------------------------------------------
  Param& ensure_param(const std::string& name, std::vector<int64_t> shape, int init) {
    auto it = params.find(name);
    if (it != params.end()) return it->second;
    Param p;
    p.shape = shape;
    p.value = alloc((size_t)numel(shape));
    p.init = init;
    params[name] = p;
    param_order.push_back(name);
    Param& ref = params[name];
    Slot* s = ref.value;
    const int64_t n = numel(shape);
    auto explicit_it = param_init.find(name);
    if (explicit_it != param_init.end()) {
      if ((int64_t)explicit_it->second.size() != n)
        fail("initial value of '" + name + "' has " + std::to_string(explicit_it->second.size()) +
             " values, expected " + std::to_string(n));
      const std::vector<float>* host = &explicit_it->second;
      setup.push_back([s, host, n](cudaStream_t st) {
        TYSOR_CUDA(cudaMemcpyAsync(s->p, host->data(), sizeof(float) * n, cudaMemcpyHostToDevice, st));
      });
    } else {
      setup.push_back([s, n, init](cudaStream_t st) { fill_pattern(s->p, n, init, st); });
    }
    return ref;
  }

  static void fill_pattern(float* p, int64_t n, int init, cudaStream_t st) {
    switch (init) {
      case 0: launch_pattern(p, n, 13, 1.0f, 16.0f, st); break;   // layers.rs:39-51
      case 1: launch_pattern(p, n, 7, 1.0f, 32.0f, st); break;    // layers.rs:53-63
      case 2: launch_pattern(p, n, 17, 1.0f, 8.0f, st); break;    // layers.rs:65-75
      case 3: launch_fill(p, n, 1.0f, st); break;                 // RMSNorm gain
      case 4: launch_pattern(p, n, 11, -5.0f, 16.0f, st); break;  // backward.rs:225-235
      default: launch_pattern(p, n, 17, 1.0f, 8.0f, st); break;   // tensor.rs:24-34
    }
  }

  // A constant (non-trainable) pattern tensor for --run / --backward.
  Slot* const_pattern(std::vector<int64_t> shape, int init) {
    Slot* s = alloc((size_t)numel(shape));
    const int64_t n = numel(shape);
    setup.push_back([s, n, init](cudaStream_t st) { fill_pattern(s->p, n, init, st); });
    return s;
  }

  // ---- GEMM step --------------------------------------------------------------
  // A matmul operand as the tensor-core kernel will read it: `hi` holds the
  // values (possibly a transposed copy), `lo` (strict mode) their low parts
  // in the same layout.
  struct Prepared {
    Slot* hi = nullptr;
    Slot* lo = nullptr;
    bool trans = false;
    int64_t ld = 0, bs = 0;
  };
  using PrepKey = std::tuple<Slot*, bool, int64_t, int64_t, int64_t, int64_t, int64_t>;
  std::map<PrepKey, std::pair<Slot*, Slot*>> prep_cache;
  // Split-fp16 packings (kGemmStrict16), keyed by operand, K contiguous or
  // not, rows, K and row pitch.
  std::map<std::tuple<Slot*, bool, int64_t, int64_t, int64_t>, Slot*> pack_cache;
  // Low parts that the kernel producing a value can write as it goes (the
  // fused causal softmax, forward and backward), keyed like prep_cache.  The
  // buffer is made, and the producer told to fill it, only when a GEMM's
  // preparation asks for it: GEMMs that make A's low part in shared memory
  // do not.
  struct LazyLo {
    Slot* slot = nullptr;
    size_t n = 0;
  };
  std::map<PrepKey, std::shared_ptr<LazyLo>> lazy_lo;
  std::shared_ptr<LazyLo> offer_lo(const PrepKey& key, size_t n) {
    auto lo = std::make_shared<LazyLo>();
    lo->n = n;
    lazy_lo[key] = lo;
    return lo;
  }
  int plan_matmul_mode = kGemmStrict;
  int plan_accum_chunk = 0;  // the context's accumulation chunk when planned

  static bool tma_aligned(int64_t ld, int64_t bs, int batch) {
    return (ld % 4) == 0 && (batch == 1 || (bs % 4) == 0);
  }

  // Prepares operand X (A if is_a, else B) of a GEMM once per step: the
  // low-part split for strict mode, and for an M/N-contiguous operand that
  // is small next to the GEMM's work, a transposed copy so the kernel reads
  // both operands K-major (its fastest form).  Values are immutable within
  // a step once produced, so one preparation serves every later GEMM that
  // reads the same operand the same way.
  Prepared prepare(StepList& out, Slot* x, bool is_a, bool trans, int64_t ld, int64_t bs,
                   int batch, int64_t M, int64_t N, int64_t K, int gmode, bool need_lo = true) {
    const int64_t R = is_a ? (trans ? K : M) : (trans ? N : K);
    const int64_t C = is_a ? (trans ? M : K) : (trans ? K : N);
    const bool mn_major = is_a ? trans : !trans;
    const bool contiguous = ld == C && (batch == 1 || bs == R * C);
    const double flops = 2.0 * batch * (double)M * N * K;
    const bool transpose = mn_major && contiguous && (double)batch * R * C * 2000.0 <= flops;
    const bool strict = gmode == kGemmStrict;
    Prepared p;
    p.hi = x;
    p.trans = trans;
    p.ld = ld;
    p.bs = bs;
    if (!transpose && !(strict && need_lo)) return p;
    // The cache holds memory objects (a copy of the stored [R][C] matrix,
    // transposed or not, and its low part); how a GEMM reads them (its
    // trans flag) is rebuilt for each caller.
    auto key = std::make_tuple(x, transpose, R, C, ld, bs, (int64_t)batch);
    auto it = prep_cache.find(key);
    std::pair<Slot*, Slot*> mem;
    auto lz = lazy_lo.find(key);
    if (it != prep_cache.end()) {
      mem = it->second;
      if (strict && need_lo && mem.second == nullptr) {
        // An earlier GEMM took this transposed copy without its low part
        // (it made A's low part itself): split the copy now.
        const int64_t n = (int64_t)batch * R * C;
        Slot *hi = mem.first, *lo = alloc((size_t)n);
        out.push_back([=](cudaStream_t st) { launch_split_lo(hi->p, lo->p, n, st); });
        mem.second = lo;
        it->second = mem;
      }
    } else if (lz != lazy_lo.end()) {
      // The producer writes the low part: claim its buffer.
      lz->second->slot = alloc(lz->second->n);
      mem = {x, lz->second->slot};
      prep_cache[key] = mem;
    } else if (transpose) {
      const int64_t n = (int64_t)batch * R * C;
      mem = {alloc((size_t)n), strict && need_lo ? alloc((size_t)n) : nullptr};
      Slot *src = x, *hi = mem.first, *lo = mem.second;
      out.push_back([=](cudaStream_t st) {
        launch_split_transpose(src->p, hi->p, lo ? lo->p : nullptr, batch, R, C, st);
      });
      prep_cache[key] = mem;
    } else {
      const int64_t span = (int64_t)(batch - 1) * bs + (R - 1) * ld + C;
      mem = {x, alloc((size_t)span)};
      Slot *src = x, *lo = mem.second;
      out.push_back([=](cudaStream_t st) { launch_split_lo(src->p, lo->p, span, st); });
      prep_cache[key] = mem;
    }
    p.hi = mem.first;
    p.lo = mem.second;
    if (transpose) {  // the copy is stored [C][R]
      p.trans = !trans;
      p.ld = R;
      p.bs = R * C;
    }
    return p;
  }

  // The split-fp16 packing of GEMM operand x with `rows` rows (M of A, N of
  // B), once per step (launch_pack16); returns the packed buffer.
  Slot* pack16(StepList& out, Slot* x, bool k_contiguous, int64_t rows, int64_t K, int64_t ld) {
    auto key = std::make_tuple(x, k_contiguous, rows, K, ld);
    if (auto it = pack_cache.find(key); it != pack_cache.end()) return it->second;
    Slot* packed = alloc((size_t)gemm_pack16_elems(rows, K));
    out.push_back([=](cudaStream_t st) { launch_pack16(x->p, k_contiguous, rows, K, ld, packed->p, st); });
    pack_cache[key] = packed;
    return packed;
  }

  // The mode this GEMM runs in (kGemmStrict16 covers only some shapes).
  int gemm_mode_for(int batch, int64_t M, int64_t N, int64_t K, int tri, bool smx, int64_t ldc, int64_t sc) const {
    return gemm_effective_mode(plan_matmul_mode, batch, M, N, K, tri, smx, ldc, sc);
  }
  // The 3xTF32 / 1xTF32 / exact mode of GEMMs the split-fp16 form does not cover.
  int tf32_mode() const { return plan_matmul_mode == kGemmStrict16 ? kGemmStrict : plan_matmul_mode; }

  void gemm_step(StepList& out, int batch, int64_t M, int64_t N, int64_t K, Slot* a,
                 bool ta, int64_t lda, int64_t sa, Slot* b, bool tb, int64_t ldb, int64_t sb,
                 Slot* c, int64_t ldc, int64_t sc, Slot* bias, float alpha, bool acc, bool relu,
                 int tri = 0, Slot* smx_p = nullptr, Slot* residual = nullptr, LeakFix fix = LeakFix()) {
    Prepared pa, pb;
    pa.hi = a, pa.trans = ta, pa.ld = lda, pa.bs = sa;
    pb.hi = b, pb.trans = tb, pb.ld = ldb, pb.bs = sb;
    const int mode_now = gemm_mode_for(batch, M, N, K, tri, smx_p != nullptr, ldc, sc);
    if (mode_now == kGemmStrict16) {
      // Both operands packed K-major (op(A) is [M, K], op(B) is [K, N]).
      pa.lo = pack16(out, a, !ta, M, K, lda);
      pb.lo = pack16(out, b, tb, N, K, ldb);
    } else {
      const bool tc = mode_now != kGemmExact && K > 0 && tma_aligned(lda, sa, batch) && tma_aligned(ldb, sb, batch);
      if (tc) {
        const bool conv_a = gemm_converts_a(batch, M, N, K, mode_now, ldc, sc);
        pa = prepare(out, a, true, ta, lda, sa, batch, M, N, K, mode_now, !conv_a);
        pb = prepare(out, b, false, tb, ldb, sb, batch, M, N, K, mode_now);
      }
    }
    const bool tc = mode_now == kGemmStrict16 ||
                    (mode_now != kGemmExact && K > 0 && tma_aligned(lda, sa, batch) && tma_aligned(ldb, sb, batch));
    Context* cx = ctx;
    const int chunk_now = plan_accum_chunk;
    // A residual is added in the GEMM's epilogue where the kernel form has
    // it (operand layouts as prepared); otherwise by a kernel after it.
    const bool res_in_gemm = residual && !acc && tc &&
                             gemm_fuses_box_epilogue(batch, M, N, K, pa.trans, pb.trans, mode_now, ldc, sc);
    // Split-K workspace (the shared scratch slot) for GEMMs whose output
    // tiles cannot fill the GPU.
    const int64_t ws_elems =
        tc && tri == 0 && !res_in_gemm ? gemm_splitk_ws_elems(batch, M, N, K, mode_now, ldc, sc) : 0;
    if (ws_elems > 0) need_scratch((size_t)ws_elems);
    Slot** scr = &scratch;
    out.push_back([=](cudaStream_t st) {
      GemmOperand A{pa.hi->p, pa.trans, pa.ld, pa.bs};
      GemmOperand B{pb.hi->p, pb.trans, pb.ld, pb.bs};
      GemmOutput O{c->p, ldc, sc};
      GemmEpilogue ep{bias ? bias->p : nullptr, alpha, acc ? 1 : 0, relu ? 1 : 0, tri};
      ep.chunk_kb = chunk_now;
      ep.smx_p = smx_p ? smx_p->p : nullptr;
      if (res_in_gemm) ep.residual = residual->p;
      GemmScratch s{nullptr, nullptr, 0, 0, 1};
      if (pa.lo) {
        s.a_lo = pa.lo->p;
        s.a_elems = (int64_t)pa.lo->n;
      }
      if (pb.lo) {
        s.b_lo = pb.lo->p;
        s.b_elems = (int64_t)pb.lo->n;
      }
      if (ws_elems > 0) {
        s.ws = (*scr)->p;
        s.ws_elems = ws_elems;
      }
      gemm_launch(batch, M, N, K, A, B, O, ep, mode_now, s, cx->d_err, st);
      if (fix.leak) {
        const int tile_rows = gemm_causal_tile_rows(batch, M, N, K, A, B, O, mode_now);
        if (tile_rows > 0)
          launch_causal_leak_fix(fix.mode, fix.leak->p, fix.rows, B.ptr, B.trans, B.ld, B.batch_stride, c->p, ldc, sc,
                                 batch, M, K, N, tile_rows, st);
      }
      if (residual && !res_in_gemm) {
        if (acc || ldc != N || (batch > 1 && sc != M * N)) throw CudaError("residual GEMM needs a fresh contiguous output");
        launch_binary_tt(kAdd, residual->p, c->p, c->p, (int64_t)batch * M * N, st);
      }
    });
  }

  // C = alpha * lhs . rhs for rank 2, or batched over equal leading dims.
  // shape_only: check and return the result's shape without planning work
  // (the value is produced later, folded into its consumer).
  HVal plan_matmul(const HVal& l, const HVal& r, StepList& out, bool shape_only = false,
                   float alpha = 1.0f, int tri = 0, int lid = -1, int rid = -1) {
    if (l.shape.size() < 2 || r.shape.size() < 2) fail("matmul currently requires rank-2 tensors");
    if (l.shape.size() != r.shape.size()) fail("matmul currently requires rank-2 tensors");
    for (size_t i = 0; i + 2 < l.shape.size(); ++i)
      if (l.shape[i] != r.shape[i]) fail("matmul currently requires rank-2 tensors");
    const int64_t m = l.shape[l.shape.size() - 2], k = l.shape.back();
    const int64_t k2 = r.shape[r.shape.size() - 2], n = r.shape.back();
    if (k != k2)
      fail("matmul inner dimension mismatch: lhs=" + shape_str(l.shape) + " rhs=" + shape_str(r.shape));
    std::vector<int64_t> os(l.shape.begin(), l.shape.end() - 2);
    const int batch = (int)numel(os);
    os.push_back(m);
    os.push_back(n);
    if (shape_only) {
      HVal o;
      o.t = HVal::Tensor;
      o.shape = os;
      return o;
    }
    HVal o = new_tensor(os);
    // A folded transpose operand is read from its source with trans set:
    // lhs x^T with x stored [k, m], rhs y^T with y stored [n, k].
    Slot *as = l.slot, *bs = r.slot;
    bool ta = false, tb = false;
    int64_t lda = k, ldb = n;
    if (auto f = folded_transpose.find(lid); f != folded_transpose.end()) {
      as = val(f->second).slot;
      ta = true;
      lda = m;
    }
    if (auto f = folded_transpose.find(rid); f != folded_transpose.end()) {
      bs = val(f->second).slot;
      tb = true;
      ldb = k;
    }
    LeakFix fix;
    if (auto lk = causal_leak.find(lid); tri == 2 && lk != causal_leak.end()) fix = {lk->second, m, 2};
    gemm_step(out, batch, m, n, k, as, ta, lda, m * k, bs, tb, ldb, k * n, o.slot, n, m * n, nullptr, alpha, false,
              false, tri, nullptr, nullptr, fix);
    return o;
  }

  // True if `vid`'s only consumer is a causal_mask that the executor fuses
  // with the Softmax consuming it (train and run modes).
  bool feeds_fused_mask(int vid) const {
    if (mode == kModeBackward) return false;
    const GNode* c = sole_consumer(vid);
    if (!c || c->kind != kNCall || c->op != "causal_mask") return false;
    const GNode* p = sole_consumer(c->output);
    return p && is_softmax_apply_of(*p, c->output);
  }

  // True if some consumer of `vid` is a matmul taking it as the left operand.
  bool is_matmul_lhs(int vid) const {
    for (int ci : consumers[vid]) {
      const GNode& c = nodes[ci];
      if (c.kind == kNPrimitive && c.op == "matmul" && !c.inputs.empty() && c.inputs[0] == vid) return true;
    }
    return false;
  }

  // The scale node of a folded matmul: one GEMM with alpha = the constant.
  HVal plan_folded_scale(const GNode& node) {
    const int m = folded_scale.at(node.output);
    float f = 1.0f;
    scales_by_const(node, m, &f);
    const auto& ops = deferred_matmul.at(m);
    // Attention scores read only through a fused causal mask: tiles wholly
    // above the diagonal are never read, so they are not computed.
    int tri = 0;
    if (feeds_fused_mask(node.output) && val(ops.first).shape.size() >= 2) {
      causal_scores.insert(m);
      tri = 1;
    }
    return plan_matmul(val(ops.first), val(ops.second), forward, false, f, tri, ops.first, ops.second);
  }

  // ---- forward planning --------------------------------------------------------
  void plan_forward() {
    hv.assign(values.size(), HVal());
    for (const GValue& v : values) {
      if (!v.is_param) continue;
      if (v.kind != kVTensor) fail("Graph executor currently supports tensor parameters only");
      auto it = shapes.find(v.name);
      std::vector<int64_t> shape;
      auto in_it = inputs.find(v.name);
      if (it != shapes.end()) {
        shape = it->second;
      } else if (in_it != inputs.end()) {
        shape = {(int64_t)in_it->second.size()};
      } else {
        fail("Missing --shape for tensor parameter '" + v.name + "'");
      }
      HVal h = new_tensor(shape);
      Slot* s = h.slot;
      const int64_t n = numel(shape);
      if (in_it != inputs.end()) {
        if ((int64_t)in_it->second.size() != n)
          fail("input '" + v.name + "' has " + std::to_string(in_it->second.size()) +
               " values, shape " + shape_str(shape) + " needs " + std::to_string(n));
        const std::vector<float>* host = &in_it->second;
        upload.push_back({v.name, [s, host, n](cudaStream_t st) {
                            TYSOR_CUDA(cudaMemcpyAsync(s->p, host->data(), sizeof(float) * n,
                                                       cudaMemcpyHostToDevice, st));
                          }});
      } else {
        setup.push_back([s, n](cudaStream_t st) { fill_pattern(s->p, n, 5, st); });
      }
      hv[v.id] = h;
    }
    for (const GNode& node : nodes) {
      cur_label = "fwd " + node_label(node);
      hv[node.output] = plan_node(node);
    }
    cur_label.clear();
  }

  std::string node_label(const GNode& node) const {
    std::string what;
    switch (node.kind) {
      case kNBinary: what = std::string("binary ") + node.binop; break;
      case kNApply: {
        const GNode* c = node.inputs.empty() ? nullptr : producer_node(node.inputs[0]);
        what = "apply " + (c ? c->op : std::string("?"));
        break;
      }
      default: what = node.op; break;
    }
    return what + " #" + std::to_string(node.output);
  }

  HVal plan_node(const GNode& node) {
    switch (node.kind) {
      case kNConst: {
        HVal h;
        if (node.ckind == 0) {
          h.t = HVal::Int;
          h.i = node.ival;
        } else if (node.ckind == 1) {
          h.t = HVal::Float;
          h.f = node.fval;
        } else {
          h.t = HVal::Bool;
          h.b = node.ival != 0;
        }
        return h;
      }
      case kNBinary: return plan_binary(node);
      case kNPrimitive: return plan_primitive(node);
      case kNCall: return plan_call(node);
      case kNCtor: return plan_ctor(node);
      case kNApply: return plan_apply(node);
    }
    fail("unknown node kind");
  }

  static int binop_code(char c) {
    switch (c) {
      case '+': return kAdd;
      case '-': return kSub;
      case '*': return kMul;
      case '/': return kDiv;
    }
    fail("unsupported tensor binary op");
  }

  HVal plan_binary(const GNode& node) {
    if (folded_scale.count(node.output)) return plan_folded_scale(node);
    if (auto rs = residual_sum.find(node.output); rs != residual_sum.end()) return rs->second;
    for (int side = 0; side < 2; ++side) {
      auto fs = fused_silu.find(node.inputs[side]);
      if (fs == fused_silu.end()) continue;
      const HVal& sv = val(node.inputs[side]);
      const HVal& other = val(node.inputs[1 - side]);
      if (node.binop == '*' && other.t == HVal::Tensor) {
        if (sv.shape != other.shape) fail("tensor shape mismatch");
        HVal o = new_tensor(sv.shape);
        Slot *x = val(fs->second).slot, *u = other.slot, *c = o.slot;
        const int64_t n = numel(sv.shape);
        forward.push_back([=](cudaStream_t st) { launch_silu_mul(x->p, u->p, c->p, n, st); });
        return o;
      }
      materialize_silu(node.inputs[side]);
      break;
    }
    const HVal& l = val(node.inputs[0]);
    const HVal& r = val(node.inputs[1]);
    const int op = binop_code(node.binop);
    if (l.t == HVal::Tensor && r.t == HVal::Tensor) {
      if (l.shape != r.shape) fail("tensor shape mismatch");
      HVal o = new_tensor(l.shape);
      Slot *a = l.slot, *b = r.slot, *c = o.slot;
      const int64_t n = numel(l.shape);
      forward.push_back([=](cudaStream_t st) { launch_binary_tt(op, a->p, b->p, c->p, n, st); });
      return o;
    }
    if (l.t == HVal::Tensor) {
      const float s = (float)number(r);
      HVal o = new_tensor(l.shape);
      Slot *a = l.slot, *c = o.slot;
      const int64_t n = numel(l.shape);
      forward.push_back([=](cudaStream_t st) { launch_binary_ts(op, a->p, s, c->p, n, st); });
      return o;
    }
    if (r.t == HVal::Tensor) {
      const float s = (float)number(l);
      HVal o = new_tensor(r.shape);
      Slot *b = r.slot, *c = o.slot;
      const int64_t n = numel(r.shape);
      forward.push_back([=](cudaStream_t st) { launch_binary_st(op, s, b->p, c->p, n, st); });
      return o;
    }
    // scalar-scalar in f64 (graph_executor.rs:299-305)
    const double a = number(l), b = number(r);
    HVal h;
    h.t = HVal::Float;
    h.f = node.binop == '+' ? a + b : node.binop == '-' ? a - b : node.binop == '*' ? a * b : a / b;
    return h;
  }

  // ---- fusions --------------------------------------------------------------
  // Values consumed by exactly one node (and not returned or used as the
  // objective) can be folded into that consumer without changing any result
  // the reference defines:
  //  * matmul -> scale-by-constant: the constant becomes the GEMM's alpha
  //    (the product is rounded once, as the two ops in sequence round it);
  //  * causal_mask -> Softmax: one masked-softmax kernel (same arithmetic),
  //    and in training one kernel for both backward rules.
  std::vector<std::vector<int>> consumers;  // node indices reading each value
  std::vector<int> external_uses;           // returned / objective
  std::map<int, std::pair<int, int>> deferred_matmul;  // matmul out -> (lhs, rhs)
  std::map<int, int> folded_scale;          // scale node out -> matmul out
  std::map<int, int> masked_input;          // causal_mask out -> its input
  std::map<int, int> fused_silu;            // SiLU out -> its input, computed inside the '*' reading it
  std::map<int, HVal> residual_sum;         // '+' out -> its value, written by the linear it adds
  std::set<int> residual_lin;               // linear outputs added to a residual inside their GEMM
  std::map<int, int> seqmajor_transpose;    // transpose(1, 2) out -> its input, read in place by rope / repeat_kv
  // Fused causal attention: score matmuls (output ids) whose scaled output
  // feeds a fused mask+softmax, and the fused softmax outputs (probabilities).
  std::set<int> causal_scores;
  std::set<int> causal_probs;
  std::map<int, Slot*> causal_leak;  // probabilities -> per-row masked probability
  // transpose(x, -2, -1) outputs read only by one matmul: the GEMM reads x
  // with its trans flag flipped and the copy is never made (value -> x).
  std::map<int, int> folded_transpose;
  std::map<int, std::pair<Slot*, float>> grad_alias;   // value -> (grad slot, factor)

  void build_uses() {
    consumers.assign(values.size(), {});
    external_uses.assign(values.size(), 0);
    for (size_t i = 0; i < nodes.size(); ++i)
      for (int in : nodes[i].inputs) consumers[in].push_back((int)i);
    for (int o : outputs) external_uses[o]++;
    if (objective >= 0) external_uses[objective]++;
  }

  const GNode* sole_consumer(int id) const {
    if (external_uses[id] != 0 || consumers[id].size() != 1) return nullptr;
    return &nodes[consumers[id][0]];
  }

  // SiLU(x) whose output feeds only one tensor '*' (SwiGLU's product) and
  // whose input feeds only it: the product runs as one pass (silu_mul) and
  // its backward as another, and the activation is never stored.  --backward
  // reports every value's gradient, so the fusion is for --run and --train.
  bool silu_fuses_into_mul(const GNode& node) const {
    if (mode == kModeBackward) return false;
    const GNode* c = sole_consumer(node.output);
    if (!c || c->kind != kNBinary || c->binop != '*' || c->inputs.size() != 2 || c->inputs[0] == c->inputs[1])
      return false;
    const int other = c->inputs[0] == node.output ? c->inputs[1] : c->inputs[0];
    if (fused_silu.count(other)) return false;  // one fused operand per product
    const GNode* xp = sole_consumer(node.inputs.at(1));
    return xp && xp->output == node.output;
  }

  // The other operand of the '+' that is the sole consumer of linear node
  // `node`'s [m, n] output, if that operand is a planned [m, n] tensor
  // (train and run modes); -1 otherwise.
  int residual_operand(const GNode& node, int64_t m, int64_t n) const {
    if (mode == kModeBackward) return -1;
    const GNode* c = sole_consumer(node.output);
    if (!c || c->kind != kNBinary || c->binop != '+' || c->inputs.size() != 2 || c->inputs[0] == c->inputs[1])
      return -1;
    const int other = c->inputs[0] == node.output ? c->inputs[1] : c->inputs[0];
    if (other < 0 || other >= (int)hv.size()) return -1;
    const HVal& ov = hv[other];
    if (ov.t != HVal::Tensor || !ov.slot || ov.shape != std::vector<int64_t>{m, n}) return -1;
    return other;
  }

  // Gives a fused SiLU output its own buffer after all (its '*' turned out
  // not to be a tensor product).
  void materialize_silu(int vid) {
    const int xi = fused_silu.at(vid);
    fused_silu.erase(vid);
    HVal& h = hv.at(vid);
    h.slot = alloc((size_t)numel(h.shape));
    Slot *a = val(xi).slot, *c = h.slot;
    const int64_t n = numel(h.shape);
    forward.push_back([=](cudaStream_t st) { launch_unary(kUnarySilu, a->p, c->p, n, 0.0f, st); });
  }

  const GNode* producer_node(int id) const {
    for (const GNode& n : nodes)
      if (n.output == id) return &n;
    return nullptr;
  }

  // True if `s` scales tensor `m` by a constant, with the constant in *f.
  bool scales_by_const(const GNode& s, int m, float* f) const {
    int c = -1;
    if (s.kind == kNPrimitive && s.op == "scale" && s.inputs.size() == 2 && s.inputs[0] == m) c = s.inputs[1];
    if (s.kind == kNBinary && s.binop == '*' && s.inputs.size() == 2) {
      if (s.inputs[0] == m && s.inputs[1] != m) c = s.inputs[1];
      else if (s.inputs[1] == m && s.inputs[0] != m) c = s.inputs[0];
    }
    if (c < 0) return false;
    const GNode* p = producer_node(c);
    if (!p || p->kind != kNConst) return false;
    *f = (float)(p->ckind == 0 ? (double)p->ival : p->ckind == 1 ? p->fval : (p->ival ? 1.0 : 0.0));
    return true;
  }

  bool is_softmax_apply_of(const GNode& p, int x) const {
    if (p.kind != kNApply || p.inputs.size() != 2 || p.inputs[1] != x) return false;
    const GNode* c = producer_node(p.inputs[0]);
    return c && c->kind == kNCtor && c->op == "Softmax";
  }

  HVal plan_primitive(const GNode& node) {
    if (node.op == "matmul") {
      const HVal& l = val(node.inputs.at(0));
      const HVal& r = val(node.inputs.at(1));
      if (l.t != HVal::Tensor || r.t != HVal::Tensor) fail("Graph executor expected tensor value");
      const GNode* s = sole_consumer(node.output);
      float f;
      if (s && scales_by_const(*s, node.output, &f)) {
        // Planned by the scale node; here only the shape (errors unchanged).
        HVal o = plan_matmul(l, r, forward, true);
        deferred_matmul[node.output] = {node.inputs[0], node.inputs[1]};
        folded_scale[s->output] = node.output;
        return o;
      }
      // Probabilities of a fused causal softmax are exact zeros above the
      // diagonal: contract each row tile only over the keys it can see.
      return plan_matmul(l, r, forward, false, 1.0f, causal_probs.count(node.inputs[0]) ? 2 : 0, node.inputs[0],
                         node.inputs[1]);
    }
    if (node.op == "relu") {
      const HVal& x = tensor(node.inputs.at(0), "relu");
      HVal o = new_tensor(x.shape);
      Slot *a = x.slot, *c = o.slot;
      const int64_t n = numel(x.shape);
      forward.push_back([=](cudaStream_t st) { launch_unary(kUnaryRelu, a->p, c->p, n, 0.0f, st); });
      return o;
    }
    if (node.op == "scale") {
      if (folded_scale.count(node.output)) return plan_folded_scale(node);
      const HVal& x = tensor(node.inputs.at(0), "scale");
      const float s = (float)number(val(node.inputs.at(1)));
      HVal o = new_tensor(x.shape);
      Slot *a = x.slot, *c = o.slot;
      const int64_t n = numel(x.shape);
      forward.push_back([=](cudaStream_t st) { launch_binary_ts(kMul, a->p, s, c->p, n, st); });
      return o;
    }
    fail("Unsupported primitive graph op '" + node.op + "'");
  }

  static void rope_dims(const std::vector<int64_t>& s, int64_t hd, int64_t* outer, int64_t* seq) {
    if (s.empty() || s.back() != hd) fail("rope head_dim mismatch");
    if (hd % 2 != 0) fail("rope requires an even head_dim");
    *seq = s.size() >= 2 ? s[s.size() - 2] : s[0];
    *outer = numel(s) / (*seq * hd);
  }

  HVal plan_call(const GNode& node) {
    const std::string& op = node.op;
    if (op == "rms_norm") {
      const HVal& x = tensor(node.inputs.at(0), "rms_norm");
      const int64_t h = integer(val(node.inputs.at(1)));
      if (x.shape.empty() || x.shape.back() != h)
        fail("rms_norm hidden size mismatch: expected " + std::to_string(h) + ", got " + shape_str(x.shape));
      HVal o = new_tensor(x.shape);
      Slot *a = x.slot, *c = o.slot;
      const int64_t rows = numel(x.shape) / h;
      forward.push_back([=](cudaStream_t st) { launch_rms_norm(a->p, c->p, rows, h, st); });
      return o;
    }
    if (op == "cross_entropy") {
      const HVal& lg = tensor(node.inputs.at(0), "logits");
      const HVal& tg = tensor(node.inputs.at(1), "target");
      const int64_t w = lg.shape.empty() ? 1 : lg.shape.back();
      const int64_t rows = numel(lg.shape) / (w > 0 ? w : 1);
      HVal o = new_tensor({rows, 1});
      Slot *a = lg.slot, *t = tg.slot, *c = o.slot;
      if (lg.shape != tg.shape && numel(tg.shape) == rows) {
        Context* cx = ctx;
        forward.push_back([=](cudaStream_t st) {
          launch_cross_entropy_labels(a->p, t->p, c->p, rows, w, cx->d_err, st);
        });
        return o;
      }
      if (lg.shape != tg.shape) fail("cross_entropy requires logits and target to have identical shapes");
      forward.push_back([=](cudaStream_t st) { launch_cross_entropy(a->p, t->p, c->p, rows, w, st); });
      return o;
    }
    if (op == "tied_logits") {
      // Extension: h . E^T with E the [num, dim] table of an Embedding
      // constructor (tied output projection).  E is read K-major, as stored.
      const HVal& x = tensor(node.inputs.at(0), "tied_logits");
      const HVal& cl = val(node.inputs.at(1));
      if (cl.t != HVal::Embedding) fail("tied_logits expects an Embedding constructor as its second argument");
      if (x.shape.size() != 2 || x.shape[1] != cl.dim)
        fail("tied_logits expects [rows, " + std::to_string(cl.dim) + "] input, got " + shape_str(x.shape));
      Slot* w = tied_weight_slot(cl);
      const int64_t m = x.shape[0], n = cl.num, k = cl.dim;
      HVal o = new_tensor({m, n});
      gemm_step(forward, 1, m, n, k, x.slot, false, k, 0, w, true, k, 0, o.slot, n, 0, nullptr, 1.0f, false, false);
      return o;
    }
    if (op == "reshape") {
      const HVal& x = tensor(node.inputs.at(0), "reshape");
      std::vector<int64_t> s;
      for (size_t i = 1; i < node.inputs.size(); ++i) s.push_back(integer(val(node.inputs[i])));
      int64_t n = 1;
      for (auto d : s) n *= d;
      if (n != numel(x.shape) || s.empty()) fail("reshape requires matching element counts");
      HVal o;
      o.t = HVal::Tensor;
      o.shape = s;
      o.slot = view(x.slot, 0, (size_t)n);
      return o;
    }
    if (op == "flatten_heads") {
      const HVal& x = tensor(node.inputs.at(0), "flatten_heads");
      HVal o;
      o.t = HVal::Tensor;
      o.shape = x.shape;
      if (x.shape.size() >= 3) {
        o.shape.assign(x.shape.begin(), x.shape.end() - 2);
        o.shape.push_back(x.shape[x.shape.size() - 2] * x.shape.back());
      }
      o.slot = view(x.slot, 0, (size_t)numel(x.shape));
      return o;
    }
    if (op == "repeat_kv") {
      const HVal& x = tensor(node.inputs.at(0), "repeat_kv");
      const int64_t rep = integer(val(node.inputs.at(1)));
      if (rep <= 0) fail("repeat_kv repeats must be positive");
      if (x.shape.size() < 2) fail("repeat_kv expects rank >= 2");
      std::vector<int64_t> s = x.shape;
      s[1] *= rep;
      HVal o = new_tensor(s);
      int64_t inner = 1;
      for (size_t i = 2; i < x.shape.size(); ++i) inner *= x.shape[i];
      const int64_t outer = x.shape[0], heads = x.shape[1];
      // A folded transpose(1, 2): read its [B, S, heads, hd] input in place.
      auto sm = seqmajor_transpose.find(node.inputs.at(0));
      Slot *a = sm != seqmajor_transpose.end() ? val(sm->second).slot : x.slot, *c = o.slot;
      const int64_t seq = sm != seqmajor_transpose.end() ? x.shape[2] : 0;
      forward.push_back([=](cudaStream_t st) { launch_repeat_kv(a->p, c->p, outer, heads, inner, rep, st, seq); });
      return o;
    }
    if (op == "causal_mask") {
      const HVal& x = tensor(node.inputs.at(0), "causal_mask");
      if (x.shape.size() < 2) fail("causal_mask expects rank >= 2");
      const int64_t q = x.shape[x.shape.size() - 2], k = x.shape.back();
      const int64_t outer = numel(x.shape) / (q * k > 0 ? q * k : 1);
      const GNode* p = sole_consumer(node.output);
      // --backward rejects causal_mask (backward.rs:354-383), so the fusion
      // (which would also fuse its backward) is used in --run and --train only.
      if (p && mode != kModeBackward && is_softmax_apply_of(*p, node.output) && x.slot) {
        masked_input[node.output] = node.inputs[0];
        HVal o;
        o.t = HVal::Tensor;
        o.shape = x.shape;
        return o;
      }
      HVal o = new_tensor(x.shape);
      Slot *a = x.slot, *c = o.slot;
      forward.push_back([=](cudaStream_t st) { launch_causal_mask(a->p, c->p, outer, q, k, st); });
      return o;
    }
    if (op == "rope") {
      const HVal& x = tensor(node.inputs.at(0), "rope");
      const int64_t hd = integer(val(node.inputs.at(1)));
      const double theta = number(val(node.inputs.at(2)));
      int64_t outer, seq;
      rope_dims(x.shape, hd, &outer, &seq);
      HVal o = new_tensor(x.shape);
      const float2* tab = ctx->rope_table(seq, hd / 2, theta);
      // A folded transpose(1, 2): read its [B, S, H, hd] input in place.
      auto sm = seqmajor_transpose.find(node.inputs.at(0));
      Slot *a = sm != seqmajor_transpose.end() ? val(sm->second).slot : x.slot, *c = o.slot;
      const int64_t hs = sm != seqmajor_transpose.end() ? x.shape[1] : 0;
      forward.push_back([=](cudaStream_t st) { launch_rope(a->p, c->p, tab, outer, seq, hd / 2, st, hs); });
      return o;
    }
    if (op == "transpose") {
      const HVal& x = tensor(node.inputs.at(0), "transpose");
      int64_t a = integer(val(node.inputs.at(1))), b = integer(val(node.inputs.at(2)));
      const int64_t rank = (int64_t)x.shape.size();
      if (a < 0) a += rank;
      if (b < 0) b += rank;
      if (a < 0 || b < 0 || a >= rank || b >= rank || rank > 8) fail("transpose axis out of range");
      if (a > b) std::swap(a, b);
      std::vector<int64_t> s = x.shape;
      std::swap(s[a], s[b]);
      const GNode* c = sole_consumer(node.output);
      // transpose(1, 2) of [B, S, H, hd] read only by rope or repeat_kv:
      // those kernels read the untransposed layout in place (and write the
      // gradient back in it).  Train and run modes.
      if (mode != kModeBackward && rank == 4 && a == 1 && b == 2 && c && c->kind == kNCall &&
          (c->op == "rope" || c->op == "repeat_kv") && c->inputs.at(0) == node.output && x.slot) {
        seqmajor_transpose[node.output] = node.inputs[0];
        HVal o;
        o.t = HVal::Tensor;
        o.shape = s;
        return o;
      }
      // Folded into its only consumer, a matmul, when it swaps the last two
      // axes (train and run modes; --backward reports every value's grad).
      if (mode != kModeBackward && rank >= 2 && a == rank - 2 && b == rank - 1 && c && c->kind == kNPrimitive &&
          c->op == "matmul" && x.slot) {
        folded_transpose[node.output] = node.inputs[0];
        HVal o;
        o.t = HVal::Tensor;
        o.shape = s;
        return o;
      }
      HVal o = new_tensor(s);
      std::vector<int64_t> dims = x.shape;
      Slot *src = x.slot, *dst = o.slot;
      const int ia = (int)a, ib = (int)b;
      forward.push_back([=](cudaStream_t st) {
        launch_transpose(src->p, dst->p, dims.data(), (int)dims.size(), ia, ib, 0, st);
      });
      return o;
    }
    fail("Unsupported library graph call '" + op + "'");
  }

  HVal plan_ctor(const GNode& node) {
    HVal h;
    h.ctor_id = node.output;
    const auto& in = node.inputs;
    if (node.op == "linear") {
      h.t = HVal::Linear;
      if (in.size() == 1) {
        h.out_features = integer(val(in[0]));
      } else if (in.size() == 2 && val(in[1]).t == HVal::Bool) {
        h.out_features = integer(val(in[0]));
        h.with_bias = boolean(val(in[1]));
      } else {
        h.in_features = integer(val(in.at(0)));
        h.out_features = integer(val(in.at(1)));
        if (in.size() == 3) h.with_bias = boolean(val(in[2]));
      }
      return h;
    }
    if (node.op == "SiLU" || node.op == "Softmax") {
      h.t = HVal::Act;
      h.act = node.op;
      return h;
    }
    if (node.op == "Embedding") {
      h.t = HVal::Embedding;
      h.num = integer(val(in.at(0)));
      h.dim = integer(val(in.at(1)));
      return h;
    }
    if (node.op == "Dropout") {
      h.t = HVal::Act;
      h.act = "Dropout";
      h.prob = number(val(in.at(0)));
      return h;
    }
    if (node.op == "RMSNorm") {
      h.t = HVal::RmsNorm;
      h.hidden = integer(val(in.at(0)));
      h.eps = in.size() > 1 ? number(val(in[1])) : 1e-5;
      return h;
    }
    fail("Unsupported library constructor '" + node.op + "'");
  }

  std::string linear_weight_name(int id) { return "linear_" + std::to_string(id) + "_weight"; }
  std::string linear_bias_name(int id) { return "linear_" + std::to_string(id) + "_bias"; }
  std::string embedding_weight_name(int id) { return "embedding_" + std::to_string(id) + "_weight"; }
  std::string gain_name(int id) { return "rmsnorm_" + std::to_string(id) + "_gain"; }

  // Table of an Embedding constructor: named parameter (train, created on
  // first use) or the constant pattern.
  Slot* tied_weight_slot(const HVal& cl) {
    if (mode == kModeTrain) return ensure_param(embedding_weight_name(cl.ctor_id), {cl.num, cl.dim}, 2).value;
    return const_pattern({cl.num, cl.dim}, 2);
  }

  // Weight of a linear apply: named parameter (train) or constant pattern.
  Slot* linear_weight_slot(const HVal& cl, int64_t in_f) {
    if (mode == kModeTrain)
      return ensure_param(linear_weight_name(cl.ctor_id), {in_f, cl.out_features}, 0).value;
    return const_pattern({in_f, cl.out_features}, 0);
  }

  HVal plan_apply(const GNode& node) {
    const HVal& cl = val(node.inputs.at(0));
    const HVal& x = val(node.inputs.at(1));
    if (x.t != HVal::Tensor) fail("Graph executor expected tensor value");
    switch (cl.t) {
      case HVal::Linear: {
        if (x.shape.size() != 2) {
          if (mode != kModeTrain) fail("linear currently requires rank-2 input tensors");
          fail("matmul currently requires rank-2 tensors");
        }
        const int64_t in_f = cl.in_features >= 0 ? cl.in_features : x.shape[1];
        if (mode != kModeTrain && x.shape[1] != in_f)
          fail("linear expected input feature size " + std::to_string(in_f) + ", got " + std::to_string(x.shape[1]));
        if (x.shape[1] != in_f)
          fail("matmul inner dimension mismatch: lhs=" + shape_str(x.shape) + " rhs=" +
               shape_str({in_f, cl.out_features}));
        Slot* w = linear_weight_slot(cl, in_f);
        Slot* b = nullptr;
        if (cl.with_bias) {
          if (mode == kModeTrain) b = ensure_param(linear_bias_name(cl.ctor_id), {cl.out_features}, 1).value;
          else b = const_pattern({cl.out_features}, 1);
        }
        const int64_t m = x.shape[0], n = cl.out_features;
        // A residual connection x + linear(.) (or linear(.) + x) whose other
        // operand already exists: the GEMM writes the sum (its epilogue adds
        // the residual) and the linear's own output is never stored.
        const int res = residual_operand(node, m, n);
        if (res >= 0) {
          HVal sum = new_tensor({m, n});
          gemm_step(forward, 1, m, n, in_f, x.slot, false, in_f, 0, w, false, n, 0, sum.slot, n, 0, b, 1.0f,
                    false, false, 0, nullptr, val(res).slot);
          residual_sum[sole_consumer(node.output)->output] = sum;
          residual_lin.insert(node.output);
          HVal o;
          o.t = HVal::Tensor;
          o.shape = {m, n};
          return o;
        }
        HVal o = new_tensor({m, n});
        gemm_step(forward, 1, m, n, in_f, x.slot, false, in_f, 0, w, false, n, 0, o.slot, n, 0, b, 1.0f,
                  false, false);
        return o;
      }
      case HVal::Embedding: {
        Slot* w;
        if (mode == kModeTrain) w = ensure_param(embedding_weight_name(cl.ctor_id), {cl.num, cl.dim}, 2).value;
        else w = const_pattern({cl.num, cl.dim}, 2);
        std::vector<int64_t> s = x.shape;
        s.push_back(cl.dim);
        HVal o = new_tensor(s);
        Slot *ix = x.slot, *c = o.slot;
        const int64_t count = numel(x.shape), num = cl.num, dim = cl.dim;
        Context* cx = ctx;
        forward.push_back([=](cudaStream_t st) { launch_embedding(ix->p, w->p, c->p, count, num, dim, cx->d_err, st); });
        return o;
      }
      case HVal::RmsNorm: {
        if (x.shape.empty() || x.shape.back() != cl.hidden)
          fail("rms_norm hidden size mismatch: expected " + std::to_string(cl.hidden) + ", got " + shape_str(x.shape));
        Slot* g;
        if (mode == kModeTrain) g = ensure_param(gain_name(cl.ctor_id), {cl.hidden}, 3).value;
        else g = const_pattern({cl.hidden}, 3);
        HVal o = new_tensor(x.shape);
        Slot *a = x.slot, *c = o.slot;
        const int64_t h = cl.hidden, rows = numel(x.shape) / h;
        const float eps = (float)cl.eps;
        forward.push_back([=](cudaStream_t st) { launch_rms_norm_gain(a->p, g->p, c->p, rows, h, eps, st); });
        return o;
      }
      case HVal::Act: {
        if (cl.act == "SiLU" && x.slot && silu_fuses_into_mul(node)) {
          fused_silu[node.output] = node.inputs.at(1);
          HVal o;
          o.t = HVal::Tensor;
          o.shape = x.shape;
          return o;
        }
        HVal o = new_tensor(x.shape);
        Slot *a = x.slot, *c = o.slot;
        const int64_t n = numel(x.shape);
        if (cl.act == "SiLU") {
          forward.push_back([=](cudaStream_t st) { launch_unary(kUnarySilu, a->p, c->p, n, 0.0f, st); });
        } else if (cl.act == "Softmax") {
          if (x.shape.empty()) fail("softmax requires a tensor with at least one dimension");
          const int64_t w = x.shape.back();
          if (w == 0 || n % w != 0) fail("softmax requires the last dimension to divide the data length");
          auto mi = masked_input.find(node.inputs.at(1));
          if (mi != masked_input.end()) {
            Slot* src = val(mi->second).slot;
            const int64_t q = x.shape[x.shape.size() - 2];
            const int64_t outer = n / (q * w);
            causal_probs.insert(node.output);
            // When a matmul will skip the masked entries, the kernel records
            // each row's masked probability for the GEMMs' fix-ups.
            const bool lhs = is_matmul_lhs(node.output);
            Slot* leak = lhs ? alloc((size_t)(outer * q)) : nullptr;
            if (leak) causal_leak[node.output] = leak;
            // A strict GEMM reading the probabilities as its left operand and
            // needing their low part gets it from this kernel (offered where
            // the GEMM's operand preparation looks it up) instead of a split
            // pass.  The probabilities are a fresh, zero-filled buffer written
            // only here, so the wholly masked (exact zero) groups are not
            // stored.
            std::shared_ptr<LazyLo> lo;
            if (lhs && tf32_mode() == kGemmStrict && w % 4 == 0)
              lo = offer_lo(std::make_tuple(c, false, q, w, w, q * w, outer), (size_t)n);
            forward.push_back([=](cudaStream_t st) {
              launch_masked_softmax(src->p, c->p, outer, q, w, leak ? leak->p : nullptr, lo && lo->slot ? lo->slot->p : nullptr,
                                    1, st);
            });
          } else {
            forward.push_back([=](cudaStream_t st) { launch_softmax(a->p, c->p, n / w, w, st); });
          }
        } else {
          if (!(cl.prob >= 0.0 && cl.prob < 1.0)) fail("dropout probability must be in [0, 1)");
          const float keep = (float)(1.0 - cl.prob);
          forward.push_back([=](cudaStream_t st) { launch_binary_ts(kMul, a->p, keep, c->p, n, st); });
        }
        return o;
      }
      default: fail("Unsupported graph apply operation");
    }
  }

  // ---- backward planning ---------------------------------------------------------
  // Returns the gradient slot of `vid` and whether this contribution must be
  // accumulated into an existing value (accumulate_value, executor.rs:545-552).
  std::pair<Slot*, bool> contrib(int vid) {
    auto it = vgrad.find(vid);
    if (it != vgrad.end()) return {it->second, true};
    const HVal& h = val(vid);
    Slot* s = alloc((size_t)numel(h.shape));
    vgrad[vid] = s;
    return {s, false};
  }

  std::pair<Slot*, bool> param_contrib(const std::string& name) {
    Param& p = params.at(name);
    if (!p.grad) p.grad = alloc((size_t)numel(p.shape));
    bool acc = p.grad_written;
    p.grad_written = true;
    grads_touched.push_back(name);
    return {p.grad, acc};
  }
  // Parameters whose gradient the node being planned writes; its items are
  // all pushed before the next node is planned.
  std::vector<std::string> grads_touched;
  void mark_grads_ready() {
    for (const std::string& name : grads_touched) params.at(name).grad_ready = backward.size();
    grads_touched.clear();
  }

  // In training a node's output gradient is dead once the node is done, so
  // one input whose gradient it would merely copy (a view's input, one
  // operand of '+' or '-') can take the buffer itself: later contributions
  // add into it as they would into the copy.  One input per node at most
  // (two sharing it would see each other's additions); the other copies
  // run first, being emitted first.
  Slot* given_g = nullptr;  // the node's gradient buffer, once handed to an input
  bool give_gradient(Slot* g, int vid) {
    if (mode != kModeTrain || vgrad.count(vid) || given_g == g) return false;
    vgrad[vid] = g;
    given_g = g;
    return true;
  }

  void emit_copy(Slot* g, int vid, int64_t n) {
    if (give_gradient(g, vid)) return;
    auto [d, acc] = contrib(vid);
    backward.push_back([=](cudaStream_t st) {
      if (acc) launch_add_inplace(d->p, g->p, n, st);
      else launch_unary(kUnaryCopy, g->p, d->p, n, 0.0f, st);
    });
  }
  void emit_neg(Slot* g, int vid, int64_t n) {
    auto [d, acc] = contrib(vid);
    backward.push_back([=](cudaStream_t st) {
      if (acc) launch_binary_tt(kSub, d->p, g->p, d->p, n, st);
      else launch_unary(kUnaryNeg, g->p, d->p, n, 0.0f, st);
    });
  }
  void emit_tt(int op, Slot* g, Slot* other, int vid, int64_t n) {
    auto [d, acc] = contrib(vid);
    backward.push_back([=](cudaStream_t st) {
      if (acc) launch_binary_tt_acc(op, g->p, other->p, d->p, n, st);
      else launch_binary_tt(op, g->p, other->p, d->p, n, st);
    });
  }
  void emit_ts(int op, Slot* g, float s, int vid, int64_t n) {
    auto [d, acc] = contrib(vid);
    backward.push_back([=](cudaStream_t st) {
      if (acc) launch_binary_ts_acc(op, g->p, s, d->p, n, 0, st);
      else launch_binary_ts(op, g->p, s, d->p, n, st);
    });
  }
  // d(lhs) of lhs.rhs: g . rhs^T ; d(rhs): lhs^T . g  (layers.rs:521-527)
  // `alpha` scales the incoming gradient (a folded scale-by-constant).
  // P . V where P = Softmax(causal_mask(s)) is read by nothing else: the
  // GEMM for dP = g . V^T writes the diagonal softmax backward's result dS
  // straight into s's gradient (its epilogue reads P), so dP is never
  // stored and the Softmax node has no gradient left to propagate.  False
  // when the shapes or layouts do not allow it.
  bool fuse_softmax_backward(const GNode& mm, Slot* g, const HVal& l, const HVal& r, float alpha) {
    const int pid = mm.inputs[0], vid = mm.inputs[1];
    const GNode* only = sole_consumer(pid);
    if (!only || only->output != mm.output || folded_transpose.count(vid) || folded_transpose.count(pid)) return false;
    const GNode* sm = producer_node(pid);
    if (!sm || sm->kind != kNApply || sm->inputs.size() < 2) return false;
    auto mi = masked_input.find(sm->inputs[1]);
    if (mi == masked_input.end() || vgrad.count(mi->second) || !l.slot || !r.slot) return false;
    const int64_t m = l.shape[l.shape.size() - 2], k = l.shape.back(), n = r.shape.back();
    std::vector<int64_t> lead(l.shape.begin(), l.shape.end() - 2);
    const int batch = (int)numel(lead);
    if (!tma_aligned(n, m * n, batch) || !tma_aligned(n, k * n, batch)) return false;
    if (!gemm_fuses_box_epilogue(batch, m, k, n, false, true, tf32_mode(), k, m * k)) return false;
    auto [d, acc] = contrib(mi->second);
    gemm_step(backward, batch, m, k, n, g, false, n, m * n, r.slot, true, n, k * n, d, k, m * k, nullptr, alpha, acc,
              false, 1, l.slot);
    return true;
  }

  void emit_matmul_grads(Slot* g, const HVal& l, const HVal& r, int lid, int rid, bool want_l,
                         bool want_r, float alpha = 1.0f, int tri_l = 0, int tri_r = 0) {
    const int64_t m = l.shape[l.shape.size() - 2], k = l.shape.back(), n = r.shape.back();
    std::vector<int64_t> lead(l.shape.begin(), l.shape.end() - 2);
    const int batch = (int)numel(lead);
    // Folded transpose operands: l = x^T (x stored [k, m]) or r = y^T (y
    // stored [n, k]); their gradient goes straight to x or y, transposed by
    // swapping the GEMM's operands (the transpose node has none to pass on).
    const auto fl = folded_transpose.find(lid), fr = folded_transpose.find(rid);
    const bool fold_l = fl != folded_transpose.end(), fold_r = fr != folded_transpose.end();
    Slot* lp = fold_l ? val(fl->second).slot : l.slot;  // physical lhs
    Slot* rp = fold_r ? val(fr->second).slot : r.slot;  // physical rhs
    if (want_l) {
      if (!fold_l) {
        // d(l) [m, k] = g . r^T
        auto [d, acc] = contrib(lid);
        if (fold_r) gemm_step(backward, batch, m, k, n, g, false, n, m * n, rp, false, k, n * k, d, k, m * k, nullptr,
                              alpha, acc, false, tri_l);
        else gemm_step(backward, batch, m, k, n, g, false, n, m * n, rp, true, n, k * n, d, k, m * k, nullptr, alpha,
                       acc, false, tri_l);
      } else {
        // d(x) [k, m] = (g . r^T)^T = r . g^T
        auto [d, acc] = contrib(fl->second);
        if (fold_r) gemm_step(backward, batch, k, m, n, rp, true, k, n * k, g, true, n, m * n, d, m, k * m, nullptr,
                              alpha, acc, false, 0);
        else gemm_step(backward, batch, k, m, n, rp, false, n, k * n, g, true, n, m * n, d, m, k * m, nullptr, alpha,
                       acc, false, 0);
      }
    }
    if (want_r) {
      if (!fold_r) {
        // d(r) [k, n] = l^T . g
        auto [d, acc] = contrib(rid);
        LeakFix fix;
        if (auto lk = causal_leak.find(lid); tri_r == 3 && lk != causal_leak.end()) fix = {lk->second, m, 3};
        if (fold_l) gemm_step(backward, batch, k, n, m, lp, false, m, k * m, g, false, n, m * n, d, n, k * n, nullptr,
                              alpha, acc, false, tri_r, nullptr, nullptr, fix);
        else gemm_step(backward, batch, k, n, m, lp, true, k, m * k, g, false, n, m * n, d, n, k * n, nullptr, alpha,
                       acc, false, tri_r, nullptr, nullptr, fix);
      } else {
        // d(y) [n, k] = (l^T . g)^T = g^T . l.  A causal contraction that
        // started at the output's first column (keys) now starts at its first
        // row.
        auto [d, acc] = contrib(fr->second);
        const int tri = tri_r == 4 ? 3 : 0;
        if (fold_l) gemm_step(backward, batch, n, k, m, g, true, n, m * n, lp, true, m, k * m, d, k, n * k, nullptr,
                              alpha, acc, false, tri);
        else gemm_step(backward, batch, n, k, m, g, true, n, m * n, lp, false, k, m * k, d, k, n * k, nullptr, alpha,
                       acc, false, tri);
      }
    }
  }

  void plan_backward() {
    cur_label = "bwd objective seed";
    const int oid = objective;
    if (oid < 0) fail("Graph does not have a return value");
    const HVal& obj = val(oid);
    if (obj.t != HVal::Tensor) fail("Train executor expected tensor value");
    {
      Slot* s = alloc((size_t)numel(obj.shape));
      vgrad[oid] = s;
      const int64_t n = numel(obj.shape);
      backward.push_back([=](cudaStream_t st) { launch_fill(s->p, n, 1.0f, st); });
    }
    const bool train = mode == kModeTrain;
    grads_touched.clear();
    for (auto it = nodes.rbegin(); it != nodes.rend(); ++it) {
      mark_grads_ready();
      const GNode& node = *it;
      cur_label = "bwd " + node_label(node);
      given_g = nullptr;
      Slot* g = nullptr;
      float galpha = 1.0f;
      auto gi = vgrad.find(node.output);
      if (gi != vgrad.end()) {
        g = gi->second;
      } else {
        auto ai = grad_alias.find(node.output);
        if (ai == grad_alias.end()) continue;
        g = ai->second.first;
        galpha = ai->second.second;
      }
      const HVal& out = val(node.output);
      const int64_t n = out.t == HVal::Tensor ? numel(out.shape) : 0;
      auto fs = folded_scale.find(node.output);
      if (fs != folded_scale.end()) {
        // The matmul's only gradient is this node's, times the constant:
        // handed to the matmul's backward GEMMs as their alpha.
        float f = 1.0f;
        scales_by_const(node, fs->second, &f);
        grad_alias[fs->second] = {g, f};
        continue;
      }
      switch (node.kind) {
        case kNConst:
        case kNCtor: break;
        case kNBinary: {
          const HVal& l = val(node.inputs[0]);
          const HVal& r = val(node.inputs[1]);
          const int li = node.inputs[0], ri = node.inputs[1];
          if (l.t == HVal::Tensor && r.t == HVal::Tensor) {
            switch (node.binop) {
              case '+': emit_copy(g, li, n); emit_copy(g, ri, n); break;
              case '-': emit_copy(g, li, n); emit_neg(g, ri, n); break;
              case '*': {
                const bool fl = fused_silu.count(li) != 0, fr = fused_silu.count(ri) != 0;
                if (fl || fr) {
                  // h = silu(x) * u: both gradients in one pass; the SiLU
                  // node adds nothing later (its input feeds only it).
                  const int xi = fused_silu.at(fl ? li : ri), ui = fl ? ri : li;
                  Slot *xs = val(xi).slot, *us = val(ui).slot;
                  auto [dx, accx] = contrib(xi);
                  auto [du, accu] = contrib(ui);
                  backward.push_back([=](cudaStream_t st) {
                    launch_silu_mul_backward(xs->p, us->p, g->p, dx->p, du->p, n, accx, accu, st);
                  });
                  break;
                }
                if (li == ri && !vgrad.count(li)) {
                  // x * x into a fresh gradient: both contributions in one pass.
                  auto [d, acc] = contrib(li);
                  (void)acc;
                  Slot* xs = l.slot;
                  backward.push_back([=](cudaStream_t st) { launch_square_backward(g->p, xs->p, d->p, n, st); });
                  break;
                }
                emit_tt(kMul, g, r.slot, li, n);
                emit_tt(kMul, g, l.slot, ri, n);
                break;
              }
              case '/': {
                emit_tt(kDiv, g, r.slot, li, n);
                if (!train) {
                  auto [d, acc] = contrib(ri);
                  Slot *ls = l.slot, *rs = r.slot;
                  backward.push_back([=](cudaStream_t st) { launch_div_rhs_grad(g->p, ls->p, rs->p, d->p, n, acc, st); });
                }
                break;
              }
              default: fail("Unsupported binary op in train backward");
            }
          } else if (l.t == HVal::Tensor) {
            if (node.binop == '+' || node.binop == '-') emit_copy(g, li, n);
            else emit_ts(binop_code(node.binop), g, (float)number(r), li, n);
          } else if (r.t == HVal::Tensor) {
            switch (node.binop) {
              case '+': emit_copy(g, ri, n); break;
              case '-': emit_neg(g, ri, n); break;
              case '*': emit_ts(kMul, g, (float)number(l), ri, n); break;
              default:
                if (!train) fail("Backward for scalar/tensor division is not implemented yet");
            }
          }
          break;
        }
        case kNPrimitive: {
          if (node.op == "matmul") {
            const HVal& l = val(node.inputs[0]);
            const HVal& r = val(node.inputs[1]);
            // Causal attention: the score gradient is an exact zero above the
            // diagonal (dQ contracts keys <= query, d(K^T) queries >= key); the
            // probability gradient is read only below it, and dV contracts
            // queries >= key.
            int tri_l = 0, tri_r = 0;
            if (causal_scores.count(node.output)) {
              tri_l = 2;
              tri_r = 4;
            } else if (causal_probs.count(node.inputs[0])) {
              tri_l = 1;
              tri_r = 3;
            }
            bool want_l = true;
            if (tri_l == 1 && fuse_softmax_backward(node, g, l, r, galpha)) want_l = false;
            emit_matmul_grads(g, l, r, node.inputs[0], node.inputs[1], want_l, true, galpha, tri_l, tri_r);
          } else if (node.op == "relu") {
            auto [d, acc] = contrib(node.inputs[0]);
            Slot* y = out.slot;
            backward.push_back([=](cudaStream_t st) { launch_relu_backward(y->p, g->p, d->p, n, acc, st); });
          } else if (node.op == "scale") {
            emit_ts(kMul, g, (float)number(val(node.inputs[1])), node.inputs[0], n);
          } else {
            fail(train ? "Unsupported primitive op in train backward"
                       : "Unsupported primitive op '" + node.op + "' in graph backward");
          }
          break;
        }
        case kNCall: plan_call_backward(node, g, out, n, train); break;
        case kNApply: plan_apply_backward(node, g, out, n, train); break;
      }
    }
    mark_grads_ready();
  }

  void plan_call_backward(const GNode& node, Slot* g, const HVal& out, int64_t n, bool train) {
    const std::string& op = node.op;
    const int xi = node.inputs.at(0);
    const HVal& x = val(xi);
    if (op == "rms_norm") {
      if (x.shape != out.shape) fail("backward_rms_norm_input shape mismatch");
      emit_copy(g, xi, n);
      return;
    }
    if (op == "cross_entropy") {
      const HVal& t = val(node.inputs.at(1));
      const int64_t w = x.shape.back(), rows = numel(x.shape) / w;
      const bool labels = x.shape != t.shape;
      {
        auto [d, acc] = contrib(xi);
        Slot *lg = x.slot, *tg = t.slot;
        Context* cx = ctx;
        backward.push_back([=](cudaStream_t st) {
          if (labels) launch_cross_entropy_labels_backward(lg->p, tg->p, d->p, rows, w, acc, cx->d_err, st);
          else launch_cross_entropy_backward(lg->p, tg->p, d->p, rows, w, acc, st);
        });
      }
      if (!train) {
        auto [d, acc] = contrib(node.inputs.at(1));
        const int64_t tn = numel(t.shape);
        if (!acc) backward.push_back([=](cudaStream_t st) { launch_fill(d->p, tn, 0.0f, st); });
      }
      return;
    }
    if (op == "transpose") {
      int64_t a = integer(val(node.inputs[1])), b = integer(val(node.inputs[2]));
      const int64_t rank = (int64_t)x.shape.size();
      if (a < 0) a += rank;
      if (b < 0) b += rank;
      if (a > b) std::swap(a, b);
      auto [d, acc] = contrib(xi);
      std::vector<int64_t> dims = out.shape;
      const int ia = (int)a, ib = (int)b;
      backward.push_back([=](cudaStream_t st) {
        launch_transpose(g->p, d->p, dims.data(), (int)dims.size(), ia, ib, acc, st);
      });
      return;
    }
    if (!train) fail("Unsupported library op '" + op + "' in graph backward");
    if (op == "tied_logits") {
      // dh (+)= g . E  and  dE (+)= g^T . h  (g: [m, num], E: [num, dim])
      const HVal& cl = val(node.inputs.at(1));
      Slot* w = tied_weight_slot(cl);
      const int64_t m = x.shape[0], nv = cl.num, k = cl.dim;
      {
        auto [d, acc] = contrib(xi);
        gemm_step(backward, 1, m, k, nv, g, false, nv, 0, w, false, k, 0, d, k, 0, nullptr, 1.0f, acc, false);
      }
      auto [dw, accw] = param_contrib(embedding_weight_name(cl.ctor_id));
      gemm_step(backward, 1, nv, k, m, g, true, nv, 0, x.slot, false, k, 0, dw, k, 0, nullptr, 1.0f, accw, false);
      return;
    }
    if (op == "reshape" || op == "flatten_heads") {
      if (numel(x.shape) != n) fail("reshape backward requires matching element counts");
      emit_copy(g, xi, n);
    } else if (op == "repeat_kv") {
      const int64_t rep = integer(val(node.inputs.at(1)));
      int64_t inner = 1;
      for (size_t i = 2; i < x.shape.size(); ++i) inner *= x.shape[i];
      const int64_t outer = x.shape[0], heads = x.shape[1];
      // Through a folded transpose(1, 2): the gradient goes to its input.
      auto sm = seqmajor_transpose.find(xi);
      const int64_t seq = sm != seqmajor_transpose.end() ? x.shape[2] : 0;
      auto [d, acc] = contrib(sm != seqmajor_transpose.end() ? sm->second : xi);
      backward.push_back([=](cudaStream_t st) {
        launch_repeat_kv_backward(g->p, d->p, outer, heads, inner, rep, acc, st, seq);
      });
    } else if (op == "causal_mask") {
      const int64_t q = out.shape[out.shape.size() - 2], k = out.shape.back();
      const int64_t outer = n / (q * k > 0 ? q * k : 1);
      auto [d, acc] = contrib(xi);
      backward.push_back([=](cudaStream_t st) { launch_causal_mask_backward(g->p, d->p, outer, q, k, acc, st); });
    } else if (op == "rope") {
      const int64_t hd = integer(val(node.inputs.at(1)));
      const double theta = number(val(node.inputs.at(2)));
      int64_t outer, seq;
      rope_dims(out.shape, hd, &outer, &seq);
      const float2* tab = ctx->rope_table(seq, hd / 2, theta);
      // Through a folded transpose(1, 2): the gradient goes to its input.
      auto sm = seqmajor_transpose.find(xi);
      const int64_t hs = sm != seqmajor_transpose.end() ? out.shape[1] : 0;
      auto [d, acc] = contrib(sm != seqmajor_transpose.end() ? sm->second : xi);
      backward.push_back([=](cudaStream_t st) {
        launch_rope_backward(g->p, d->p, tab, outer, seq, hd / 2, acc, st, hs);
      });
    }
    // Other library calls contribute nothing in train mode (executor.rs:661-687).
  }

  void plan_apply_backward(const GNode& node, Slot* g, const HVal& out, int64_t n, bool train) {
    const HVal& cl = val(node.inputs.at(0));
    const int xi = node.inputs.at(1);
    const HVal& x = val(xi);
    switch (cl.t) {
      case HVal::Linear: {
        const int64_t in_f = cl.in_features >= 0 ? cl.in_features : (x.shape.size() > 1 ? x.shape[1] : 0);
        const int64_t m = x.shape[0], nf = cl.out_features;
        Slot* w;
        if (train) {
          auto pit = params.find(linear_weight_name(cl.ctor_id));
          w = pit != params.end() ? pit->second.value : const_pattern({in_f, nf}, 0);
        } else {
          w = const_pattern({in_f, nf}, 4);  // backward.rs:225-235 fake weight
        }
        {
          auto [d, acc] = contrib(xi);
          gemm_step(backward, 1, m, in_f, nf, g, false, nf, 0, w, true, nf, 0, d, in_f, 0, nullptr, 1.0f, acc, false);
        }
        if (train) {
          auto [dw, accw] = param_contrib(linear_weight_name(cl.ctor_id));
          gemm_step(backward, 1, in_f, nf, m, x.slot, true, in_f, 0, g, false, nf, 0, dw, nf, 0, nullptr, 1.0f,
                    accw, false);
          if (cl.with_bias) {
            auto [db, accb] = param_contrib(linear_bias_name(cl.ctor_id));
            need_scratch((size_t)colsum_partial_elems(m, nf));
            Slot** scr = &scratch;
            backward.push_back([=](cudaStream_t st) { launch_colsum(g->p, db->p, (*scr)->p, m, nf, accb, st); });
          }
        }
        return;
      }
      case HVal::Embedding: {
        if (!train) fail("Graph backward does not support this library apply yet");
        auto [dw, accw] = param_contrib(embedding_weight_name(cl.ctor_id));
        const int64_t count = numel(x.shape), num = cl.num, dim = cl.dim;
        need_scratch(embedding_backward_work_bytes(count, num) / sizeof(float) + 1);
        Slot** scr = &scratch;
        Slot* ix = x.slot;
        backward.push_back([=](cudaStream_t st) {
          launch_embedding_backward(g->p, ix->p, dw->p, count, num, dim, (*scr)->p, accw, st);
        });
        return;
      }
      case HVal::RmsNorm: {
        const int64_t h = cl.hidden, rows = numel(x.shape) / h;
        const float eps = (float)cl.eps;
        Slot* gain;
        Slot* dg = nullptr;
        bool accg = false;
        if (train) {
          gain = params.at(gain_name(cl.ctor_id)).value;
          auto pc = param_contrib(gain_name(cl.ctor_id));
          dg = pc.first;
          accg = pc.second;
        } else {
          gain = const_pattern({h}, 3);
          dg = alloc((size_t)h);  // discarded in --backward
        }
        auto [d, acc] = contrib(xi);
        need_scratch((size_t)rms_gain_partial_elems(rows, h));
        Slot** scr = &scratch;
        Slot* xs = x.slot;
        backward.push_back([=](cudaStream_t st) {
          launch_rms_norm_gain_backward(xs->p, gain->p, g->p, d->p, dg->p, (*scr)->p, rows, h, eps, acc, accg, st);
        });
        return;
      }
      case HVal::Act: {
        if (fused_silu.count(node.output)) return;  // done by its '*' (silu_mul_backward)
        auto mi = masked_input.find(xi);
        if (cl.act == "Softmax" && mi != masked_input.end()) {
          // Softmax(causal_mask(x)): both backward rules in one pass, straight
          // into x's gradient (the mask's output never holds a gradient).
          auto [d, acc] = contrib(mi->second);
          Slot* ys = out.slot;
          const int64_t q = out.shape[out.shape.size() - 2], k = out.shape.back();
          const int64_t outer = n / (q * k);
          // As in the forward: when the scores come from a (folded-scale)
          // matmul, its strict backward GEMMs read this gradient's low part
          // from here; a fresh zero-filled gradient skips its masked zeros.
          std::shared_ptr<LazyLo> lo;
          if (!acc && folded_scale.count(mi->second) && tf32_mode() == kGemmStrict && k % 4 == 0)
            lo = offer_lo(std::make_tuple(d, false, q, k, k, q * k, outer), (size_t)n);
          const int skip = acc ? 0 : 1;
          backward.push_back([=](cudaStream_t st) {
            launch_masked_softmax_backward(ys->p, g->p, d->p, outer, q, k, acc, lo && lo->slot ? lo->slot->p : nullptr,
                                           skip, st);
          });
          return;
        }
        auto [d, acc] = contrib(xi);
        Slot* xs = x.slot;
        Slot* ys = out.slot;
        if (cl.act == "SiLU") {
          backward.push_back([=](cudaStream_t st) { launch_silu_backward(xs->p, g->p, d->p, n, acc, st); });
        } else if (cl.act == "Softmax") {
          backward.push_back([=](cudaStream_t st) { launch_softmax_backward(ys->p, g->p, d->p, n, acc, st); });
        } else {
          const float keep = (float)(1.0 - cl.prob);
          backward.push_back([=](cudaStream_t st) {
            if (acc) launch_binary_ts_acc(kMul, g->p, keep, d->p, n, 0, st);
            else launch_binary_ts(kMul, g->p, keep, d->p, n, st);
          });
        }
        return;
      }
      default: fail(train ? "Unsupported apply in train backward" : "Graph backward does not support this library apply yet");
    }
  }

  // ---- update planning (train) ------------------------------------------------------
  void plan_update() {
    cur_label = "update (loss, all-reduce, sgd)";
    // The loss (sum of the objective) comes from this step's forward values
    // (executor.rs:803-811); it is reduced before the backward starts, so
    // that it can travel with the first gradient bucket of a data-parallel
    // step.
    const HVal& obj = val(objective);
    const int64_t n = numel(obj.shape);
    Slot* o = obj.slot;
    Slot** ls = &loss;
    need_scratch(1024);
    Slot** scr = &scratch;
    const int* order = &loss_order;
    backward.fns.insert(backward.fns.begin(), [=](cudaStream_t st) {
      if (*order == 1) launch_sequential_sum(o->p, (*ls)->p, n, st);
      else launch_reduce_sum(o->p, (*ls)->p, (*scr)->p, n, st);
    });
    backward.labels.insert(backward.labels.begin(), "bwd loss (sum of the objective)");
    for (auto& [name, p] : params) (void)name, p.grad_ready += 1;
    // Data parallel: the gradient buckets are all-reduced on the comm stream
    // as the backward finishes them (see place_buckets); the update waits
    // for the last one.
    update.push_back([this](cudaStream_t st) {
      if (allreduce && !buckets.empty()) {
        TYSOR_CUDA(cudaEventRecord(comm_done, comm_stream));
        TYSOR_CUDA(cudaStreamWaitEvent(st, comm_done, 0));
      }
    });
    // One SGD pass over all parameters when they sit in one block laid out
    // like the gradient block (each element's update is the same p - lr * g;
    // the order the reference visits them in does not change any value).
    if (params_in_block()) {
      Slot **pb = &param_block, **gbl = &grad_block;
      size_t* pn = &param_block_n;
      float* lr_ptr = &lr_f;
      // The gradient block starts with the loss and its padding (64
      // floats); the parameters' gradients follow in the parameter block's
      // order.
      update.push_back([=](cudaStream_t st) {
        if (*pn > 0) launch_sgd((*pb)->p, (*gbl)->p + kLossFloats, *lr_ptr, (int64_t)*pn, st);
      });
      return;
    }
    std::vector<std::string> names(param_order);
    std::sort(names.begin(), names.end());  // BTreeMap order (executor.rs:750)
    for (const std::string& name : names) {
      Param& p = params.at(name);
      if (!p.grad) continue;
      Slot *pv = p.value, *pg = p.grad;
      const int64_t pn = numel(p.shape);
      float* lr_ptr = &lr_f;
      update.push_back([=](cudaStream_t st) { launch_sgd(pv->p, pg->p, *lr_ptr, pn, st); });
    }
  }
  float lr_f = 0.01f;
  // The loss's slot at the head of the gradient block, padded like every
  // slot to 64 floats.
  static constexpr size_t kLossFloats = 64;
  // Data-parallel gradient buckets: contiguous ranges of the gradient block
  // (laid out in the order the backward finishes the gradients), each
  // all-reduced on comm_stream once the backward item that completes it has
  // run.
  struct Bucket {
    size_t begin = 0, count = 0;  // floats of the gradient block
    size_t ready = 0;             // backward items that must run first
    cudaEvent_t ready_ev = nullptr;
  };
  std::vector<Bucket> buckets;
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t comm_done = nullptr;
  // 0: tree sum of the objective (default); 1: the reference's sequential f32
  // sum in index order (tysor_cuda_graph_set_loss_order).
  int loss_order = 0;

  // Whether every trained parameter owns its value buffer (not a view) of
  // its gradient's size, so the values can form one block.
  bool params_in_block() const {
    std::set<const Slot*> seen;
    for (const std::string& name : param_order) {
      const Param& p = params.at(name);
      if (!p.grad) continue;
      if (!p.value || p.value->base || p.value->n != p.grad->n || !seen.insert(p.value).second) return false;
    }
    return true;
  }

  // ---- arena layout --------------------------------------------------------------------
  // Trained parameters in the order the backward finishes their gradients
  // (ties in parameter order): the gradient and parameter blocks follow it,
  // so each all-reduce bucket is one contiguous range.
  std::vector<std::string> grad_order() const {
    std::vector<std::string> names;
    for (const std::string& name : param_order)
      if (params.at(name).grad) names.push_back(name);
    std::stable_sort(names.begin(), names.end(), [this](const std::string& a, const std::string& b) {
      return params.at(a).grad_ready < params.at(b).grad_ready;
    });
    return names;
  }

  void layout() {
    // The loss and the parameter gradients share one contiguous block so
    // that a data-parallel step all-reduces them in a few bucketed
    // collectives (the loss first: it is reduced before the backward).
    size_t gtotal = 0;
    std::vector<Slot*> gslots;
    if (mode == kModeTrain) {
      loss = alloc(1);
      gslots.push_back(loss);
      gtotal += kLossFloats;
    }
    const std::vector<std::string> gorder = grad_order();
    for (const std::string& name : gorder) {
      Param& p = params.at(name);
      gslots.push_back(p.grad);
      gtotal += (p.grad->n + 63) & ~(size_t)63;
    }
    scratch = alloc(scratch_floats + 64);
    size_t total = 0;
    std::map<Slot*, size_t> off;
    // grad block first
    size_t gb_start = 0;
    for (Slot* s : gslots) {
      off[s] = total;
      total += (s->n + 63) & ~(size_t)63;
    }
    const size_t gb_end = total;
    // then the trained parameters, in the same order and padding
    const bool pblock = mode == kModeTrain && params_in_block();
    if (pblock) {
      for (const std::string& name : gorder) {
        Param& p = params.at(name);
        off[p.value] = total;
        total += (p.value->n + 63) & ~(size_t)63;
      }
    }
    const size_t pb_end = total;
    for (Slot& s : slots) {
      if (s.base || off.count(&s)) continue;
      off[&s] = total;
      total += (s.n + 63) & ~(size_t)63;
    }
    if (arena) cudaFree(arena);
    TYSOR_CUDA(cudaMalloc(&arena, sizeof(float) * (total + 64)));
    // Zeroed once so the padding inside the gradient block is defined.
    TYSOR_CUDA(cudaMemsetAsync(arena, 0, sizeof(float) * (total + 64), ctx->stream));
    float* basep = (float*)arena;
    for (Slot& s : slots)
      if (!s.base) s.p = basep + off[&s];
    for (Slot& s : slots)
      if (s.base) s.p = s.base->p + s.offset;
    if (mode == kModeTrain) {
      slots.push_back(Slot{gb_end - gb_start, nullptr, 0, basep + gb_start});
      grad_block = &slots.back();
      if (pblock) {
        slots.push_back(Slot{pb_end - gb_end, nullptr, 0, basep + gb_end});
        param_block = &slots.back();
        param_block_n = pb_end - gb_end;
      }
      place_buckets(gorder, off);
    }
  }

  // Cuts the gradient block into buckets of at least bucket_floats() (the
  // last may be smaller) and inserts, after the backward item that completes
  // each bucket, an item that (when data parallel) hands it to comm_stream:
  // an event on the compute stream, a wait on the comm stream, the NCCL
  // all-reduce there.  The collectives thus overlap the rest of the
  // backward; every rank issues the same buckets in the same order.
  void place_buckets(const std::vector<std::string>& gorder, const std::map<Slot*, size_t>& off) {
    for (Bucket& b : buckets)
      if (b.ready_ev) cudaEventDestroy(b.ready_ev);
    buckets.clear();
    const size_t target = bucket_floats();
    Bucket cur;
    cur.begin = 0;
    cur.ready = 1;  // the loss item
    size_t end = kLossFloats;  // the loss and its padding
    for (const std::string& name : gorder) {
      const Param& p = params.at(name);
      end = off.at(p.grad) + ((p.grad->n + 63) & ~(size_t)63);
      cur.ready = std::max(cur.ready, p.grad_ready);
      if (end - cur.begin >= target) {
        cur.count = end - cur.begin;
        buckets.push_back(cur);
        cur = Bucket();
        cur.begin = end;
      }
    }
    if (end > cur.begin) {
      cur.count = end - cur.begin;
      buckets.push_back(cur);
    }
    for (Bucket& b : buckets) TYSOR_CUDA(cudaEventCreateWithFlags(&b.ready_ev, cudaEventDisableTiming));
    if (!comm_done) TYSOR_CUDA(cudaEventCreateWithFlags(&comm_done, cudaEventDisableTiming));
    if (!comm_stream) {
      int lo = 0, hi = 0;
      TYSOR_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
      TYSOR_CUDA(cudaStreamCreateWithPriority(&comm_stream, cudaStreamNonBlocking, hi));
    }
    // Rebuild the backward list with the bucket hand-offs in place.
    StepList out{{}, {}, backward.cur};
    size_t next = 0;
    for (size_t i = 0; i <= backward.fns.size(); ++i) {
      while (next < buckets.size() && buckets[next].ready == i) {
        const size_t k = next++;
        out.fns.push_back([this, k](cudaStream_t st) {
          if (!allreduce) return;
          Bucket& b = buckets[k];
          TYSOR_CUDA(cudaEventRecord(b.ready_ev, st));
          TYSOR_CUDA(cudaStreamWaitEvent(comm_stream, b.ready_ev, 0));
          comm_allreduce_on(ctx, grad_block->p + b.begin, b.count, comm_stream);
        });
        out.labels.push_back("bwd all-reduce bucket " + std::to_string(k) + " (" +
                             std::to_string(buckets[k].count * 4 / (1 << 20)) + " MB)");
      }
      if (i < backward.fns.size()) {
        out.fns.push_back(std::move(backward.fns[i]));
        out.labels.push_back(std::move(backward.labels[i]));
      }
    }
    backward.fns = std::move(out.fns);
    backward.labels = std::move(out.labels);
  }

  // Bucket size: TYSOR_CUDA_BUCKET_MB (default 64 MB), read when planning.
  static size_t bucket_floats() {
    const char* v = getenv("TYSOR_CUDA_BUCKET_MB");
    long mb = v ? atol(v) : 64;
    if (mb < 1) mb = 1;
    return (size_t)mb * (1 << 20) / sizeof(float);
  }

  void plan(int m) {
    if (!dirty && mode == m && plan_matmul_mode == ctx->matmul_mode && plan_accum_chunk == ctx->accum_chunk_kb)
      return;
    release();
    mode = m;
    plan_matmul_mode = ctx->matmul_mode;
    plan_accum_chunk = ctx->accum_chunk_kb;
    build_uses();
    plan_forward();
    if (mode != kModeRun) plan_backward();
    if (mode == kModeTrain) plan_update();
    cur_label.clear();
    layout();
    dirty = false;
  }

  void run_list(const StepList& list) {
    for (const StepFn& f : list) f(ctx->stream);
  }

  void ensure_setup() {
    if (setup_done) return;
    for (const StepFn& f : setup) f(ctx->stream);
    setup_done = true;
  }
};

Executor* E(void* g) {
  if (!g) throw CudaError("null graph");
  Executor* e = static_cast<Executor*>(g);
  TYSOR_CUDA(cudaSetDevice(e->ctx->device));
  return e;
}

template <typename F>
bool guarded_g(F&& f) {
  try {
    f();
    return true;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return false;
  }
}

Slot* value_slot(Executor* e, int id, std::vector<int64_t>* shape) {
  if (id < 0 || id >= (int)e->hv.size()) throw CudaError("value id out of range");
  const HVal& h = e->hv[id];
  if (h.t == HVal::Tensor && !h.slot &&
      (e->folded_transpose.count(id) || e->masked_input.count(id) || e->fused_silu.count(id) ||
       e->seqmajor_transpose.count(id) || e->residual_lin.count(id)))
    throw CudaError("value " + std::to_string(id) + " is not materialised: it was fused into its consumer");
  if (h.t != HVal::Tensor || !h.slot) throw CudaError("value " + std::to_string(id) + " is not a tensor");
  if (shape) *shape = h.shape;
  return h.slot;
}

}  // namespace
}  // namespace tysor

using namespace tysor;

extern "C" {

void* tysor_cuda_graph_new(void* context, const char* graph_text) {
  Executor* out = nullptr;
  guarded_g([&] {
    if (!context) throw CudaError("null context");
    if (!graph_text) throw CudaError("null graph text");
    auto e = std::make_unique<Executor>();
    e->ctx = static_cast<Context*>(context);
    e->parse(graph_text);
    out = e.release();
  });
  return out;
}

void tysor_cuda_graph_free(void* graph) {
  if (!graph) return;
  Executor* e = static_cast<Executor*>(graph);
  cudaSetDevice(e->ctx->device);
  cudaStreamSynchronize(e->ctx->stream);
  delete e;
}

bool tysor_cuda_graph_set_shape(void* graph, const char* name, const int64_t* dims, int rank) {
  return guarded_g([&] {
    Executor* e = E(graph);
    if (rank < 1) throw CudaError("shape must contain at least one dimension");
    std::vector<int64_t> s(dims, dims + rank);
    for (auto d : s)
      if (d <= 0) throw CudaError("invalid dimension in shape");
    e->shapes[name] = s;
    e->dirty = true;
  });
}

bool tysor_cuda_graph_set_input(void* graph, const char* name, const float* data, size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    auto it = e->inputs.find(name);
    const bool same_size = it != e->inputs.end() && it->second.size() == count;
    e->inputs[name].assign(data, data + count);
    e->device_inputs.erase(name);
    if (!same_size) e->dirty = true;  // the plan reads the stored vector at each call
  });
}

bool tysor_cuda_graph_upload_input(void* graph, const char* name, const float* data,
                                   size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    if (e->mode < 0 || e->dirty) throw CudaError("graph buffers are not planned yet: run it once first");
    for (const GValue& v : e->values) {
      if (!v.is_param || v.name != name) continue;
      Slot* s = e->hv.at(v.id).slot;
      if (!s || count != s->n)
        throw CudaError("input '" + std::string(name) + "' holds " + std::to_string(s ? s->n : 0) +
                        " values, " + std::to_string(count) + " given");
      TYSOR_CUDA(cudaMemcpyAsync(s->p, data, sizeof(float) * count, cudaMemcpyHostToDevice, e->ctx->stream));
      // Later calls must not overwrite it with a stored input.
      e->device_inputs.insert(v.name);
      return;
    }
    throw CudaError(std::string("no graph input named '") + name + "'");
  });
}

bool tysor_cuda_graph_prefetch_input(void* graph, const char* name, const float* data,
                                     size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    if (e->mode < 0 || e->dirty) throw CudaError("graph buffers are not planned yet: run it once first");
    Slot* s = e->input_slot(name);
    if (!s) throw CudaError(std::string("no graph input named '") + name + "'");
    if (count != s->n)
      throw CudaError("input '" + std::string(name) + "' holds " + std::to_string(s->n) + " values, " +
                      std::to_string(count) + " given");
    e->prefetch_input(name, s, data, count);
    // Later calls must not overwrite it with a stored input.
    e->device_inputs.insert(name);
  });
}

bool tysor_cuda_graph_set_parameter(void* graph, const char* name, const float* data,
                                    size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    e->param_init[name].assign(data, data + count);
    e->dirty = true;
  });
}

bool tysor_cuda_graph_run(void* graph) {
  return guarded_g([&] {
    Executor* e = E(graph);
    const int64_t l0 = g_launches.load();
    e->plan(kModeRun);
    e->ensure_setup();
    e->run_uploads();
    e->run_list(e->forward);
    e->last_launches = g_launches.load() - l0;
    e->ctx->sync_and_check();
  });
}

bool tysor_cuda_graph_backward(void* graph) {
  return guarded_g([&] {
    Executor* e = E(graph);
    const int64_t l0 = g_launches.load();
    e->plan(kModeBackward);
    e->ensure_setup();
    e->run_uploads();
    e->run_list(e->forward);
    e->run_list(e->backward);
    e->last_launches = g_launches.load() - l0;
    e->ctx->sync_and_check();
  });
}

// Enqueues `iterations` train steps on the context stream (the first step
// of a plan eagerly, later ones as the captured graph) and each step's loss
// into the device history; with `host_losses`, each loss is also copied to
// host_losses[it] on the stream.  Waits for nothing.
void enqueue_train_steps(Executor* e, int iterations, double lr, float* host_losses) {
  if (iterations < 0) throw CudaError("iterations must be >= 0");
  e->plan(kModeTrain);
  e->lr_f = (float)lr;
  e->ensure_setup();
  e->run_uploads();
  cudaStream_t st = e->ctx->stream;
  if (iterations > e->loss_hist_cap) {
    // Grown outside any capture; the step loop itself allocates nothing.
    TYSOR_CUDA(cudaStreamSynchronize(st));
    if (e->loss_hist) TYSOR_CUDA(cudaFree(e->loss_hist));
    e->loss_hist = nullptr;
    e->loss_hist_cap = 0;
    const int cap = iterations < 1024 ? 1024 : iterations;
    TYSOR_CUDA(cudaMalloc(&e->loss_hist, sizeof(float) * cap));
    e->loss_hist_cap = cap;
  }
  float* d_losses = e->loss_hist;
  auto step = [&]() {
    e->run_list(e->forward);
    e->run_list(e->backward);
    e->run_list(e->update);
  };
  for (int it = 0; it < iterations; ++it) {
    const int64_t l0 = g_launches.load();
    // The first step of a plan runs eagerly (it configures kernels); every
    // later step, in this call or a later one, replays the captured graph.
    if (e->capture && e->stepped) {
      if (!e->exec) {
        cudaGraph_t g = nullptr;
        TYSOR_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        try {
          step();
        } catch (...) {
          cudaStreamEndCapture(st, &g);
          if (g) cudaGraphDestroy(g);
          throw;
        }
        TYSOR_CUDA(cudaStreamEndCapture(st, &g));
        TYSOR_CUDA(cudaGraphInstantiate(&e->exec, g, 0));
        cudaGraphDestroy(g);
        e->step_launches = g_launches.load() - l0;
      }
      TYSOR_CUDA(cudaGraphLaunch(e->exec, st));
    } else {
      step();
      e->step_launches = g_launches.load() - l0;
      e->stepped = true;
    }
    // The step's loss is kept by a one-element copy kernel (no copy-engine
    // work between the steps' kernels).
    launch_unary(kUnaryCopy, e->loss->p, d_losses + it, 1, 0.0f, st);
    if (host_losses)
      TYSOR_CUDA(cudaMemcpyAsync(host_losses + it, d_losses + it, sizeof(float), cudaMemcpyDeviceToHost, st));
    e->last_launches = e->step_launches + 1;  // kernels per step, the loss copy included
  }
}

bool tysor_cuda_graph_train(void* graph, int iterations, double lr, float* losses) {
  return guarded_g([&] {
    Executor* e = E(graph);
    enqueue_train_steps(e, iterations, lr, nullptr);
    std::vector<float> host(iterations > 0 ? iterations : 1);
    if (iterations > 0)
      TYSOR_CUDA(cudaMemcpyAsync(host.data(), e->loss_hist, sizeof(float) * iterations, cudaMemcpyDeviceToHost,
                                 e->ctx->stream));
    e->ctx->sync_and_check();
    if (losses)
      for (int i = 0; i < iterations; ++i) losses[i] = host[i];
  });
}

bool tysor_cuda_graph_train_enqueue(void* graph, int iterations, double lr, float* host_losses) {
  return guarded_g([&] { enqueue_train_steps(E(graph), iterations, lr, host_losses); });
}

bool tysor_cuda_graph_train_traced(void* graph, double lr, float* item_ms, int capacity,
                                   int* n_items) {
  return guarded_g([&] {
    Executor* e = E(graph);
    if (!n_items) throw CudaError("n_items must not be null");
    e->plan(kModeTrain);
    e->lr_f = (float)lr;
    e->ensure_setup();
    e->run_uploads();
    cudaStream_t st = e->ctx->stream;
    std::vector<const StepFn*> items;
    e->trace_labels.clear();
    for (const auto* list : {&e->forward, &e->backward, &e->update})
      for (size_t i = 0; i < list->size(); ++i) {
        items.push_back(&list->fns[i]);
        e->trace_labels.push_back(list->labels[i]);
      }
    std::vector<cudaEvent_t> ev(items.size() + 1, nullptr);
    try {
      for (auto& x : ev) TYSOR_CUDA(cudaEventCreate(&x));
      TYSOR_CUDA(cudaEventRecord(ev[0], st));
      for (size_t i = 0; i < items.size(); ++i) {
        (*items[i])(st);
        TYSOR_CUDA(cudaEventRecord(ev[i + 1], st));
      }
      e->ctx->sync_and_check();
      e->stepped = true;
      *n_items = (int)items.size();
      for (size_t i = 0; i < items.size() && (int)i < capacity; ++i) {
        float ms = 0.0f;
        TYSOR_CUDA(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        if (item_ms) item_ms[i] = ms;
      }
    } catch (...) {
      for (auto& x : ev)
        if (x) cudaEventDestroy(x);
      throw;
    }
    for (auto& x : ev) cudaEventDestroy(x);
  });
}

const char* tysor_cuda_graph_trace_label(void* graph, int item) {
  const char* out = nullptr;
  guarded_g([&] {
    Executor* e = E(graph);
    if (item < 0 || item >= (int)e->trace_labels.size()) throw CudaError("no such traced item");
    out = e->trace_labels[(size_t)item].c_str();
  });
  return out;
}

int tysor_cuda_graph_value_rank(void* graph, int value_id) {
  int rank = -1;
  guarded_g([&] {
    std::vector<int64_t> s;
    value_slot(E(graph), value_id, &s);
    rank = (int)s.size();
  });
  return rank;
}

bool tysor_cuda_graph_value_shape(void* graph, int value_id, int64_t* dims) {
  return guarded_g([&] {
    std::vector<int64_t> s;
    value_slot(E(graph), value_id, &s);
    for (size_t i = 0; i < s.size(); ++i) dims[i] = s[i];
  });
}

bool tysor_cuda_graph_read_value(void* graph, int value_id, float* out, size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    std::vector<int64_t> s;
    Slot* sl = value_slot(e, value_id, &s);
    if (count > sl->n) throw CudaError("read past the end of the value");
    e->ctx->sync_and_check();
    TYSOR_CUDA(cudaMemcpy(out, sl->p, sizeof(float) * count, cudaMemcpyDeviceToHost));
  });
}

bool tysor_cuda_graph_read_value_grad(void* graph, int value_id, float* out, size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    auto it = e->vgrad.find(value_id);
    if (it == e->vgrad.end()) throw CudaError("value has no gradient");
    if (count > it->second->n) throw CudaError("read past the end of the gradient");
    e->ctx->sync_and_check();
    TYSOR_CUDA(cudaMemcpy(out, it->second->p, sizeof(float) * count, cudaMemcpyDeviceToHost));
  });
}

int tysor_cuda_graph_num_parameters(void* graph) {
  int n = -1;
  guarded_g([&] { n = (int)E(graph)->param_order.size(); });
  return n;
}

const char* tysor_cuda_graph_parameter_name(void* graph, int index) {
  const char* out = nullptr;
  guarded_g([&] {
    Executor* e = E(graph);
    if (index < 0 || index >= (int)e->param_order.size()) throw CudaError("parameter index out of range");
    out = e->param_order[index].c_str();
  });
  return out;
}

size_t tysor_cuda_graph_parameter_count(void* graph, const char* name) {
  size_t n = 0;
  guarded_g([&] {
    Executor* e = E(graph);
    n = (size_t)numel(e->params.at(name).shape);
  });
  return n;
}

bool tysor_cuda_graph_read_parameter(void* graph, const char* name, float* out, size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    auto it = e->params.find(name);
    if (it == e->params.end()) throw CudaError(std::string("no parameter '") + name + "'");
    if (count > it->second.value->n) throw CudaError("read past the end of the parameter");
    e->ensure_setup();
    e->ctx->sync_and_check();
    TYSOR_CUDA(cudaMemcpy(out, it->second.value->p, sizeof(float) * count, cudaMemcpyDeviceToHost));
  });
}

bool tysor_cuda_graph_read_parameter_grad(void* graph, const char* name, float* out, size_t count) {
  return guarded_g([&] {
    Executor* e = E(graph);
    auto it = e->params.find(name);
    if (it == e->params.end() || !it->second.grad) throw CudaError(std::string("no gradient for '") + name + "'");
    if (count > it->second.grad->n) throw CudaError("read past the end of the gradient");
    e->ctx->sync_and_check();
    TYSOR_CUDA(cudaMemcpy(out, it->second.grad->p, sizeof(float) * count, cudaMemcpyDeviceToHost));
  });
}

int64_t tysor_cuda_graph_launch_count(void* graph) {
  int64_t n = -1;
  guarded_g([&] { n = E(graph)->last_launches; });
  return n;
}

bool tysor_cuda_graph_set_capture(void* graph, bool enable) {
  return guarded_g([&] {
    Executor* e = E(graph);
    e->capture = enable;
    if (!enable && e->exec) {
      cudaGraphExecDestroy(e->exec);
      e->exec = nullptr;
    }
  });
}

bool tysor_cuda_graph_set_loss_order(void* graph, int order) {
  return guarded_g([&] {
    Executor* e = E(graph);
    if (order != 0 && order != 1) throw CudaError("loss order must be 0 (tree) or 1 (sequential, the reference's)");
    if (order != e->loss_order && e->exec) {
      // The captured step holds the other reduction: capture again.
      TYSOR_CUDA(cudaStreamSynchronize(e->ctx->stream));
      cudaGraphExecDestroy(e->exec);
      e->exec = nullptr;
    }
    e->loss_order = order;
  });
}

bool tysor_cuda_graph_enable_allreduce(void* graph, bool enable) {
  return guarded_g([&] {
    Executor* e = E(graph);
    if (enable && !e->ctx->comm) throw CudaError("no communicator: call tysor_cuda_comm_init first");
    if (e->allreduce != enable) {
      e->allreduce = enable;
      if (e->exec) {
        cudaGraphExecDestroy(e->exec);
        e->exec = nullptr;
      }
    }
  });
}

}  // extern "C"
