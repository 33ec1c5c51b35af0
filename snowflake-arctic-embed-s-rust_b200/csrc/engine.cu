// Host engine behind the C ABI (include/arctic_cuda.h): one context per GPU owns the uploaded
// model, a device workspace sized for a token budget, pinned staging buffers, a stream and a device
// error word, and enqueues the forward pass of a packed batch:
//
//   row metadata -> embedding+LN+quant -> 11 x [QKV GEMM -> attention -> ctx quant ->
//   attn-out GEMM (+res, LN1, quant) -> FFN-up GEMM (GELU, quant) -> FFN-down GEMM (+res, LN2, quant)]
//   -> layer 11: KV GEMM over all rows, gather [CLS] rows, Q GEMM, [CLS] attention, ctx quant,
//      attn-out (+LN1), FFN-up, FFN-down (+LN2, L2 norm) -> [n, 384]
//
// which is PackedModel::forward_ragged_cls (src/model.rs:521-914) without its 64-sequence and
// 512-row limits; a single sequence (forward_cls, src/model.rs:185-513) is the n = 1 case and is
// replayed from a CUDA graph per length.
#include <cuda.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "../../include/arctic_cuda.h"
#include "gemm_i8.h"
#include "kernels.h"
#include "latency.h"
#include "ptx.cuh"
#include "rowmath.cuh"

using namespace ae;

namespace {

struct DevLinear {
  int n = 0, k = 0;
  int8_t* w = nullptr;
  float* ws = nullptr;
  float* bias = nullptr;
  float* inv_s = nullptr;
  CUtensorMap tmap;    // 64-row boxes (the GEMM kernels)
  CUtensorMap tmap32;  // 32-row boxes (the single-sequence cluster forward)
};

struct DevLayer {
  DevLinear qkv, q_only, kv_only, ao, fi, fo;
  float *ln1w = nullptr, *ln1b = nullptr, *ln2w = nullptr, *ln2b = nullptr;
};

struct DevModel {
  void* arena = nullptr;
  size_t arena_bytes = 0;
  int8_t* word_q = nullptr;
  float* word_s = nullptr;
  int8_t* pos_q = nullptr;
  float* pos_s = nullptr;
  float* type0 = nullptr;
  float *emb_lnw = nullptr, *emb_lnb = nullptr;
  DevLayer layers[kLayers];
  LatModel* lat = nullptr;  // what the single-sequence cluster forward reads (in the arena)
};

struct Workspace {
  uint32_t cap_tokens = 0, cap_seqs = 0;
  void* arena = nullptr;
  uint16_t* ids = nullptr;
  uint32_t* cu = nullptr;
  uint16_t* pos = nullptr;
  int32_t* cls_row = nullptr;
  float* hidden = nullptr;
  int8_t* act_q = nullptr;
  float* act_s = nullptr;
  float* qkv = nullptr;
  float* ctx = nullptr;
  int8_t* inter_q = nullptr;
  float* inter_s = nullptr;
  int8_t* cq = nullptr;
  float* cs = nullptr;
  float* ch = nullptr;
  float* q_cls = nullptr;
  float* cctx = nullptr;
  int8_t* cinter_q = nullptr;
  float* cinter_s = nullptr;
  float* out = nullptr;
  CUtensorMap tm_act_q, tm_inter_q, tm_cq, tm_cinter_q;
  // pinned host staging
  uint16_t* h_ids = nullptr;
  uint32_t* h_cu = nullptr;
  float* h_out = nullptr;
};

struct Graph {
  cudaGraph_t g = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint64_t kernels = 0;
};

}  // namespace

struct ae_ctx {
  int device = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  // ae_forward_cls's graphs: the embedding (384 floats) followed by the graph's own error word, so
  // that one device-to-host copy inside the graph brings both (no separate read of d_err per call)
  float* d_lat = nullptr;
  float* h_lat = nullptr;  // pinned
  int* h_err = nullptr;    // pinned copy of d_err, taken on the stream before a synchronisation
  uint32_t* d_cu_single = nullptr;  // [513][2]: {0, L} at 2L, the cu_seqlens of one sequence of L ids
  float* d_gemm_scratch = nullptr;  // ae_gemm_i8's split LayerNorm path: h of up to gemm_scratch_rows rows
  uint32_t gemm_scratch_rows = 0;
  bool has_model = false;
  DevModel model;
  void* h_model = nullptr;  // pinned host image of the model arena (reused across loads)
  size_t h_model_bytes = 0;
  Workspace ws;
  std::map<uint32_t, Graph> graphs;  // forward_cls graph per sequence length
  std::string err;
  int gelu_erf = 0;       // ARCTIC_GELU=erf selects the exact-erf GELU (outside the parity tolerance)
  int fused_qkv = 0;      // ARCTIC_FUSED_QKV=1: QKV projection fused into the attention (sequences <= 128 keys)
  int attn_mode = AE_ATTENTION_EXACT;  // ae_set_attention_mode, ARCTIC_ATTN=int8
  int few_mode = 0;         // ARCTIC_ATTN_FEW=tmem|narrow|lanes8|dm: the attention kernel of few long sequences
  bool lat_cluster = false;  // single sequences of <= 32 tokens as one cluster kernel (ARCTIC_LAT_CLUSTER=0: off)
  bool prof = false;      // record CUDA events around every launch (ae_profile)
  int prof_kind = 0;      // kind of the launches being enqueued
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> prof_events;
  std::vector<cudaEvent_t> prof_pool;
  uint64_t launches = 0;  // kernels enqueued (or replayed from a graph) on this context
  uint64_t graph_kernels = 0;
  // host packing of the last ragged batch: sequences grouped by attention length class
  std::vector<uint32_t> order;       // packed position -> caller's sequence index
  std::vector<ae::AttnSegment> segs;  // consecutive packed sequences of one class
  // ae_embed_batch_multi's two staging slots (kept across calls, grown as needed)
  struct PipeSlot {
    uint32_t cap_tok = 0, cap_seqs = 0;
    uint16_t* h_ids = nullptr;
    uint32_t* h_cu = nullptr;
    float* h_out = nullptr;
    uint16_t* d_ids = nullptr;
    uint32_t* d_cu = nullptr;
    float* d_out = nullptr;
    cudaEvent_t done = nullptr;
    std::vector<uint32_t> order, idx;
    std::vector<ae::AttnSegment> segs;
    uint32_t n = 0;
    bool busy = false;
  } pipe[2];
};

namespace {

thread_local std::string g_create_err;

int fail(ae_ctx* c, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  else g_create_err = buf;
  return code;
}

#define CUDA_TRY(c, expr)                                                                         \
  do {                                                                                            \
    cudaError_t e_ = (expr);                                                                      \
    if (e_ != cudaSuccess) return fail((c), AE_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

#define AE_TRY(expr)        \
  do {                      \
    int r_ = (expr);        \
    if (r_ != 0) return r_; \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ------------------------------------------------------------------------------------------ model
struct Carve {
  uint8_t* base;
  size_t off = 0;
  template <class T>
  T* take(size_t n) {
    off = align_up(off, 256);
    T* p = reinterpret_cast<T*>(base + off);
    off += n * sizeof(T);
    return p;
  }
};

size_t linear_bytes(const ae_linear_desc& d) {
  return align_up(d.n_out * d.k_in, 256) + 3 * align_up(d.n_out * 4, 256) + align_up(d.k_in * 4, 256) + 1024;
}

bool check_linear(const ae_linear_desc& d, uint64_t n, uint64_t k, bool allow_pruned) {
  if (allow_pruned && d.n_out == 0) return d.k_in == k && d.inv_smooth;
  return d.n_out == n && d.k_in == k && d.w_q && d.w_scale && d.bias && d.inv_smooth;
}

// Model upload: every tensor is copied (memcpy on host threads) to its offset in a host image of
// the device arena, held in pinned memory that the context keeps across loads, and one DMA moves
// the image to the arena. A reload of the same model shape reuses the arena (no cudaFree /
// cudaMalloc); when every tensor lands at its old address, the captured single-sequence graphs stay
// valid, since they hold device addresses, not data.
struct Uploader {
  const uint8_t* dev_base = nullptr;  // the model arena
  uint8_t* host = nullptr;            // pinned host image of the arena
  struct Copy {
    size_t off;
    const void* src;
    size_t n;
  };
  std::vector<Copy> copies;
  size_t bytes = 0;
  template <class T>
  void put(T* dst, const void* src, size_t n) {
    const size_t b = n * sizeof(T);
    copies.push_back(Copy{size_t(reinterpret_cast<const uint8_t*>(dst) - dev_base), src, b});
    bytes += b;
  }
  // Runs the copies, split into byte ranges of about equal size over a few host threads.
  void run() {
    const int nt = bytes >= (size_t(8) << 20) ? 4 : 1;
    auto part = [&](int t) {
      const size_t lo = bytes * size_t(t) / size_t(nt), hi = bytes * size_t(t + 1) / size_t(nt);
      size_t at = 0;
      for (const Copy& cp : copies) {
        const size_t a = std::max(lo, at), b = std::min(hi, at + cp.n);
        if (a < b) std::memcpy(host + cp.off + (a - at), static_cast<const uint8_t*>(cp.src) + (a - at), b - a);
        at += cp.n;
        if (at >= hi) break;
      }
    };
    std::vector<std::thread> th;
    for (int t = 1; t < nt; ++t) th.emplace_back(part, t);
    part(0);
    for (auto& x : th) x.join();
  }
};

int upload_linear(ae_ctx* c, Carve& cv, Uploader& img, const ae_linear_desc& d, DevLinear& o) {
  o.n = int(d.n_out);
  o.k = int(d.k_in);
  o.inv_s = cv.take<float>(d.k_in);
  img.put(o.inv_s, d.inv_smooth, d.k_in);
  if (d.n_out == 0) return 0;
  o.w = cv.take<int8_t>(d.n_out * d.k_in);
  o.ws = cv.take<float>(d.n_out);
  o.bias = cv.take<float>(d.n_out);
  img.put(o.w, d.w_q, d.n_out * d.k_in);
  img.put(o.ws, d.w_scale, d.n_out);
  img.put(o.bias, d.bias, d.n_out);
  if (make_tmap_i8(&o.tmap, o.w, o.n, o.k, kBoxB) != 0 || make_tmap_i8(&o.tmap32, o.w, o.n, o.k, 32) != 0)
    return fail(c, AE_ERR_CUDA, "cuTensorMapEncodeTiled failed for weights");
  return 0;
}

// True when every tensor of a and b sits at the same device address with the same shape (a tensor
// map is a function of its address and shape, so those agree too).
bool same_placement(const DevModel& a, const DevModel& b) {
  auto lin = [](const DevLinear& x, const DevLinear& y) {
    return x.n == y.n && x.k == y.k && x.w == y.w && x.ws == y.ws && x.bias == y.bias && x.inv_s == y.inv_s;
  };
  if (a.arena != b.arena || a.word_q != b.word_q || a.word_s != b.word_s || a.pos_q != b.pos_q || a.pos_s != b.pos_s ||
      a.type0 != b.type0 || a.emb_lnw != b.emb_lnw || a.emb_lnb != b.emb_lnb || a.lat != b.lat)
    return false;
  for (int l = 0; l < kLayers; ++l) {
    const DevLayer &x = a.layers[l], &y = b.layers[l];
    if (!lin(x.qkv, y.qkv) || !lin(x.q_only, y.q_only) || !lin(x.kv_only, y.kv_only) || !lin(x.ao, y.ao) ||
        !lin(x.fi, y.fi) || !lin(x.fo, y.fo) || x.ln1w != y.ln1w || x.ln1b != y.ln1b || x.ln2w != y.ln2w ||
        x.ln2b != y.ln2b)
      return false;
  }
  return true;
}

void free_model(ae_ctx* c) {
  if (c->model.arena) cudaFree(c->model.arena);
  c->model = DevModel();
  c->has_model = false;
}

// ------------------------------------------------------------------------------------------ workspace
void free_ws(ae_ctx* c) {
  Workspace& w = c->ws;
  if (w.arena) cudaFree(w.arena);
  if (w.h_ids) cudaFreeHost(w.h_ids);
  if (w.h_cu) cudaFreeHost(w.h_cu);
  if (w.h_out) cudaFreeHost(w.h_out);
  w = Workspace();
}

void drop_graphs(ae_ctx* c) {
  for (auto& kv : c->graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.g) cudaGraphDestroy(kv.second.g);
  }
  c->graphs.clear();
}

int reserve(ae_ctx* c, uint32_t tokens, uint32_t seqs) {
  Workspace& w = c->ws;
  if (tokens <= w.cap_tokens && seqs <= w.cap_seqs && w.arena) return 0;
  // grow geometrically, so that a stream of slowly growing batches reallocates a few times only
  if (w.arena) {
    if (tokens > w.cap_tokens) tokens = std::max<uint32_t>(tokens, w.cap_tokens + w.cap_tokens / 2);
    if (seqs > w.cap_seqs) seqs = std::max<uint32_t>(seqs, w.cap_seqs + w.cap_seqs / 2);
  }
  tokens = std::max(tokens, w.cap_tokens);
  seqs = std::max(seqs, w.cap_seqs);
  tokens = std::max<uint32_t>(align_up(tokens, 128), 128);
  seqs = std::max<uint32_t>(align_up(seqs, 128), 128);
  drop_graphs(c);
  free_ws(c);
  const size_t T = tokens, B = seqs;
  size_t bytes = 0;
  auto add = [&](size_t n) { bytes = align_up(bytes, 256) + n; };
  add(T * 2);                 // ids
  add((B + 1) * 4);           // cu
  add(T * 2);                 // pos
  add(B * 4);                 // cls_row
  add(T * kHidden * 4);       // hidden
  add(T * kHidden);           // act_q
  add(T * 4);                 // act_s
  add(T * 3 * kHidden * 4);   // qkv
  add(T * kHidden * 4);       // ctx
  add(T * kInter);            // inter_q
  add(T * 4);                 // inter_s
  add(B * kHidden);           // cq
  add(B * 4);                 // cs
  add(B * kHidden * 4);       // ch
  add(B * kHidden * 4);       // q_cls
  add(B * kHidden * 4);       // cctx
  add(B * kInter);            // cinter_q
  add(B * 4);                 // cinter_s
  add(B * kHidden * 4);       // out
  bytes += 4096;
  void* arena = nullptr;
  CUDA_TRY(c, cudaMalloc(&arena, bytes));
  CUDA_TRY(c, cudaMemset(arena, 0, bytes));
  w.arena = arena;
  Carve cv{static_cast<uint8_t*>(arena)};
  w.ids = cv.take<uint16_t>(T);
  w.cu = cv.take<uint32_t>(B + 1);
  w.pos = cv.take<uint16_t>(T);
  w.cls_row = cv.take<int32_t>(B);
  w.hidden = cv.take<float>(T * kHidden);
  w.act_q = cv.take<int8_t>(T * kHidden);
  w.act_s = cv.take<float>(T);
  w.qkv = cv.take<float>(T * 3 * kHidden);
  w.ctx = cv.take<float>(T * kHidden);
  w.inter_q = cv.take<int8_t>(T * kInter);
  w.inter_s = cv.take<float>(T);
  w.cq = cv.take<int8_t>(B * kHidden);
  w.cs = cv.take<float>(B);
  w.ch = cv.take<float>(B * kHidden);
  w.q_cls = cv.take<float>(B * kHidden);
  w.cctx = cv.take<float>(B * kHidden);
  w.cinter_q = cv.take<int8_t>(B * kInter);
  w.cinter_s = cv.take<float>(B);
  w.out = cv.take<float>(B * kHidden);
  w.cap_tokens = tokens;
  w.cap_seqs = seqs;
  if (make_tmap_i8(&w.tm_act_q, w.act_q, int(T), kHidden, kBoxA) || make_tmap_i8(&w.tm_inter_q, w.inter_q, int(T), kInter, kBoxA) ||
      make_tmap_i8(&w.tm_cq, w.cq, int(B), kHidden, kBoxA) || make_tmap_i8(&w.tm_cinter_q, w.cinter_q, int(B), kInter, kBoxA))
    return fail(c, AE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the workspace");
  CUDA_TRY(c, cudaMallocHost(&w.h_ids, T * 2));
  CUDA_TRY(c, cudaMallocHost(&w.h_cu, (B + 1) * 4));
  CUDA_TRY(c, cudaMallocHost(&w.h_out, B * kHidden * 4));
  return 0;
}

// ------------------------------------------------------------------------------------------ forward
// Profiling: a pair of events around the next launch(es) of the current kind.
cudaEvent_t prof_event(ae_ctx* c) {
  if (!c->prof_pool.empty()) {
    cudaEvent_t e = c->prof_pool.back();
    c->prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}
struct ProfScope {
  ae_ctx* c;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfScope(ae_ctx* cc, int kind) : c(cc) {
    if (!c->prof) return;
    c->prof_kind = kind;
    a = prof_event(c);
    b = prof_event(c);
    cudaEventRecord(a, c->stream);
  }
  ~ProfScope() {
    if (!c->prof || !a) return;
    cudaEventRecord(b, c->stream);
    c->prof_events.push_back({c->prof_kind, {a, b}});
  }
};

// `tt` selects the tile-transposed layout for the fp32 residual and output (the hidden state and
// the QKV / KV outputs of the packed rows; the [CLS]-row buffers stay row-major).
int gemm(ae_ctx* c, int epi, const CUtensorMap& ta, const DevLinear& L, int M, const float* a_scale, const float* res,
         int ldr, const float* gamma, const float* beta, const float* inv_next, float* out, int ldo, int8_t* out_q,
         float* out_s, int tt = 0) {
  GemmArgs g{};
  g.out_tt = tt;
  g.res_tt = tt;
  g.M = M;
  g.N = L.n;
  g.K = L.k;
  g.a_scale = a_scale;
  g.w_scale = L.ws;
  g.bias = L.bias;
  g.res = res;
  g.ldr = ldr;
  g.gamma = gamma;
  g.beta = beta;
  g.inv_smooth = inv_next;
  g.out_f32 = out;
  g.ldo = ldo;
  g.out_q = out_q;
  g.out_scale = out_s;
  g.acc_dbg = nullptr;
  g.err = c->d_err;
  g.gelu_erf = c->gelu_erf;
  int r = gemm_i8_launch(epi, ta, L.tmap, g, c->stream);
  ++c->launches;
  if (r) return fail(c, AE_ERR_CUDA, "GEMM launch failed (epilogue %d, M=%d N=%d K=%d): code %d", epi, M, L.n, L.k, r);
  return 0;
}

// quant (optional): {inverse smoothing factors, int8 rows, row scales} of the context rows; when
// the launch quantized them itself *quantized is set to 1 and the caller skips k_smooth_quant.
struct CtxQuant {
  const float* inv_s;
  int8_t* q;
  float* scale;
};
int attention(ae_ctx* c, const float* q, int q_C, int q_col, int q_tt, const float* kv, int kv_C, int k_col,
              int v_col, int kv_tt, float* out, const uint32_t* cu, int n, int max_len, int cls,
              const std::vector<AttnSegment>* segs = nullptr, const CtxQuant* quant = nullptr,
              int* quantized = nullptr) {
  if (quantized) *quantized = 0;
  AttnArgs a{};
  a.q = q;
  a.q_C = q_C;
  a.q_col = q_col;
  a.q_tt = q_tt;
  a.kv = kv;
  a.kv_C = kv_C;
  a.k_col = k_col;
  a.v_col = v_col;
  a.kv_tt = kv_tt;
  a.out = out;
  a.cu = cu;
  a.max_len = max_len;
  a.cls_mode = cls;
  a.err = c->d_err;
  a.few_mode = c->few_mode;
  if (quant) {
    a.quant_inv_s = quant->inv_s;
    a.quant_q = quant->q;
    a.quant_scale = quant->scale;
  }
  if (segs && segs->size() > 1) {  // one launch per length class, sized for that class
    for (const AttnSegment& g : *segs) {
      AttnArgs b = a;
      b.cu = cu + g.first;
      b.max_len = g.max_len;
      ++c->launches;
      if (launch_attention_exact(b, g.count, c->stream)) return fail(c, AE_ERR_CUDA, "attention launch failed");
    }
    return 0;
  }
  ++c->launches;
  if (launch_attention_exact(a, n, c->stream, quant ? quantized : nullptr))
    return fail(c, AE_ERR_CUDA, "attention launch failed");
  return 0;
}

// Sequences of fewer keys than this keep the fp32 attention in the int8 mode (the reference's
// crossover for one sequence, src/model.rs:245).
constexpr int kI8MinLen = 16;

// Attention of layers 0-10 in the int8 mode: per length run (or over the whole batch), the fp32
// kernels for the sequences below kI8MinLen, when the run may hold some, then the int8 kernel for
// the others. min_len: the shortest sequence of the batch when known, else 1.
int attention_i8(ae_ctx* c, const float* qkv, float* out, const uint32_t* cu, int n, int max_len, int min_len,
                 const std::vector<AttnSegment>* segs) {
  AttnArgs a{};
  a.q = qkv;
  a.q_C = 3 * kHidden;
  a.q_col = 0;
  a.q_tt = 1;
  a.kv = qkv;
  a.kv_C = 3 * kHidden;
  a.k_col = kHidden;
  a.v_col = 2 * kHidden;
  a.kv_tt = 1;
  a.out = out;
  a.err = c->d_err;
  std::vector<AttnSegment> whole;
  if (!segs || segs->empty()) {
    whole.push_back(AttnSegment{0, n, max_len, min_len});
    segs = &whole;
  }
  for (const AttnSegment& g : *segs) {
    AttnArgs b = a;
    b.cu = cu + g.first;
    b.max_len = g.max_len;
    if (g.min_len < kI8MinLen) {  // the sequences below the crossover, sized for them
      AttnArgs x = b;
      if (g.max_len >= kI8MinLen) {
        x.max_len = kI8MinLen - 1;
        x.skip_from = kI8MinLen;
      }
      ++c->launches;
      if (launch_attention_exact(x, g.count, c->stream)) return fail(c, AE_ERR_CUDA, "attention launch failed");
    }
    if (g.max_len >= kI8MinLen) {
      ++c->launches;
      if (launch_attention_i8(b, g.count, kI8MinLen, c->stream))
        return fail(c, AE_ERR_CUDA, "int8 attention launch failed");
    }
  }
  return 0;
}

// Residual GEMM followed by LayerNorm + SmoothQuant quantization (attention-out, FFN-down):
// fused into the GEMM epilogue when the batch has enough 128-row tiles to fill the GPU; otherwise
// a plain-epilogue GEMM split over narrow column slices writes h = fma(acc, as*ws, bias + res)
// into `scratch` (row-major) and a row kernel applies the same LayerNorm + quantization.
int gemm_ln(ae_ctx* c, const CUtensorMap& ta, const DevLinear& L, int M, const float* a_scale, float* hidden,
            int hidden_tt, const float* gamma, const float* beta, const float* inv_next, int8_t* out_q, float* out_s,
            float* scratch) {
  const int m_tiles = (M + 127) / 128;
  if (m_tiles >= 74) {
    return gemm(c, EPI_LN_QUANT, ta, L, M, a_scale, hidden, kHidden, gamma, beta, inv_next, hidden, kHidden, out_q,
                out_s, hidden_tt);
  }
  GemmArgs g{};
  g.M = M;
  g.N = L.n;
  g.K = L.k;
  g.a_scale = a_scale;
  g.w_scale = L.ws;
  g.bias = L.bias;
  g.res = hidden;
  g.ldr = kHidden;
  g.res_tt = hidden_tt;
  g.out_f32 = scratch;
  g.ldo = kHidden;
  g.err = c->d_err;
  ++c->launches;
  int r = gemm_i8_launch(EPI_F32, ta, L.tmap, g, c->stream);
  if (r) return fail(c, AE_ERR_CUDA, "GEMM launch failed (split residual path): code %d", r);
  ++c->launches;
  if (launch_ln_quant_rows(scratch, M, gamma, beta, inv_next, hidden, hidden_tt, out_q, out_s, c->stream))
    return fail(c, AE_ERR_CUDA, "LayerNorm row kernel launch failed");
  return 0;
}

// Enqueues the whole forward pass of a packed batch on the context's stream.
//
// segs (optional): the packed sequences as runs of one attention length class each (host packing
// knows the lengths); the attention of layers 0-10 then launches once per run.
// min_len: a lower bound of the sequence lengths (the int8 attention mode uses it when segs is
// not given).
// stop (ae_trace_forward): AE_TRACE_EMBED returns after the embedding kernel, AE_TRACE_ATTN0 after
// layer 0's attention and context quantization; -1 runs the whole pass.
int enqueue_forward(ae_ctx* c, const uint16_t* d_ids, const uint32_t* d_cu, int T, int n, int max_len, float* d_out,
                    const std::vector<AttnSegment>* segs = nullptr, int min_len = 1, int stop = -1) {
  Workspace& W = c->ws;
  const DevModel& M = c->model;
  cudaStream_t st = c->stream;
  const uint64_t launches0 = c->launches;
  c->launches += 2;  // row metadata + embedding
  {
    ProfScope ps(c, AE_KERNEL_ROW_META);
    if (launch_row_meta(d_cu, n, W.pos, W.cls_row, c->d_err, st))
      return fail(c, AE_ERR_CUDA, "row metadata launch failed");
  }
  EmbedArgs e{};
  e.T = T;
  e.ids = d_ids;
  e.pos = W.pos;
  e.word_q = M.word_q;
  e.word_s = M.word_s;
  e.pos_q = M.pos_q;
  e.pos_s = M.pos_s;
  e.type0 = M.type0;
  e.gamma = M.emb_lnw;
  e.beta = M.emb_lnb;
  e.inv_smooth = M.layers[0].qkv.inv_s;
  e.hidden = W.hidden;
  e.act_q = W.act_q;
  e.act_s = W.act_s;
  e.err = c->d_err;
  {
    ProfScope ps(c, AE_KERNEL_EMBED);
    if (launch_embed(e, st)) return fail(c, AE_ERR_CUDA, "embedding launch failed");
  }
  if (stop == AE_TRACE_EMBED) return 0;

  // QKV projection fused with the attention (sequences of at most 128 keys) only on request
  // (ARCTIC_FUSED_QKV=1): measured on config 3 it is 2 % slower than the QKV GEMM + attention
  // kernels (its load / MMA / dequantization prologue runs while the SM's FP32 pipes idle) and
  // 8 % slower for single sequences; by default a QKV GEMM writes the projections to global memory
  // for the attention kernels of every length class.
  const bool fused = max_len <= 128 && c->fused_qkv == 1 && c->attn_mode == AE_ATTENTION_EXACT;
  for (int l = 0; l + 1 < kLayers; ++l) {
    const DevLayer& Ly = M.layers[l];
    int ctx_quantized = 0;  // the attention kernel also wrote act_q / act_s
    if (fused) {
      ProfScope ps(c, AE_KERNEL_ATTENTION);
      QkvAttnArgs qa{};
      qa.a.out = W.ctx;
      qa.a.cu = d_cu;
      qa.a.max_len = max_len;
      qa.a.err = c->d_err;
      qa.a_scale = W.act_s;
      qa.w_scale = Ly.qkv.ws;
      qa.bias = Ly.qkv.bias;
      ++c->launches;
      if (launch_qkv_attention(W.tm_act_q, Ly.qkv.tmap, qa, n, st))
        return fail(c, AE_ERR_CUDA, "fused QKV + attention launch failed");
    } else {
      {
        ProfScope ps(c, AE_KERNEL_QKV);
        AE_TRY(gemm(c, EPI_F32, W.tm_act_q, Ly.qkv, T, W.act_s, nullptr, 0, nullptr, nullptr, nullptr, W.qkv,
                    3 * kHidden, nullptr, nullptr, 1));
      }
      {
        ProfScope ps(c, AE_KERNEL_ATTENTION);
        const CtxQuant cq{Ly.ao.inv_s, W.act_q, W.act_s};
        if (c->attn_mode == AE_ATTENTION_INT8)
          AE_TRY(attention_i8(c, W.qkv, W.ctx, d_cu, n, max_len, min_len, segs));
        else
          AE_TRY(attention(c, W.qkv, 3 * kHidden, 0, 1, W.qkv, 3 * kHidden, kHidden, 2 * kHidden, 1, W.ctx, d_cu, n,
                           max_len, 0, segs, &cq, &ctx_quantized));
      }
    }
    if (!ctx_quantized) {
      ++c->launches;
      ProfScope ps(c, AE_KERNEL_CTX_QUANT);
      if (launch_smooth_quant(W.ctx, Ly.ao.inv_s, W.act_q, W.act_s, T, st))
        return fail(c, AE_ERR_CUDA, "context quantization launch failed");
    }
    if (stop == AE_TRACE_ATTN0) return 0;
    {
      ProfScope ps(c, AE_KERNEL_ATTN_OUT);
      AE_TRY(gemm_ln(c, W.tm_act_q, Ly.ao, T, W.act_s, W.hidden, 1, Ly.ln1w, Ly.ln1b, Ly.fi.inv_s, W.act_q, W.act_s,
                     W.ctx));
    }
    {
      ProfScope ps(c, AE_KERNEL_FFN_UP);
      AE_TRY(gemm(c, EPI_GELU_QUANT, W.tm_act_q, Ly.fi, T, W.act_s, nullptr, 0, nullptr, nullptr, Ly.fo.inv_s, nullptr,
                  0, W.inter_q, W.inter_s));
    }
    {
      ProfScope ps(c, AE_KERNEL_FFN_DOWN);
      AE_TRY(gemm_ln(c, W.tm_inter_q, Ly.fo, T, W.inter_s, W.hidden, 1, Ly.ln2w, Ly.ln2b, M.layers[l + 1].qkv.inv_s,
                     W.act_q, W.act_s, W.ctx));
    }
  }
  const DevLayer& Z = M.layers[kLayers - 1];
  {
    ProfScope ps(c, AE_KERNEL_QKV);
    AE_TRY(gemm(c, EPI_F32, W.tm_act_q, Z.kv_only, T, W.act_s, nullptr, 0, nullptr, nullptr, nullptr, W.qkv,
                2 * kHidden, nullptr, nullptr, 1));
  }
  ProfScope ps_cls(c, AE_KERNEL_CLS);
  c->launches += 2;  // gather + [CLS] context quantization
  if (launch_gather_cls(W.cls_row, n, W.act_q, W.act_s, W.hidden, W.cq, W.cs, W.ch, st))
    return fail(c, AE_ERR_CUDA, "gather launch failed");
  AE_TRY(gemm(c, EPI_F32, W.tm_cq, Z.q_only, n, W.cs, nullptr, 0, nullptr, nullptr, nullptr, W.q_cls, kHidden, nullptr,
              nullptr));
  AE_TRY(attention(c, W.q_cls, kHidden, 0, 0, W.qkv, 2 * kHidden, 0, kHidden, 1, W.cctx, d_cu, n, max_len, 1));
  if (launch_smooth_quant(W.cctx, Z.ao.inv_s, W.cq, W.cs, n, st))
    return fail(c, AE_ERR_CUDA, "context quantization launch failed");
  AE_TRY(gemm_ln(c, W.tm_cq, Z.ao, n, W.cs, W.ch, 0, Z.ln1w, Z.ln1b, Z.fi.inv_s, W.cq, W.cs, W.cctx));
  AE_TRY(gemm(c, EPI_GELU_QUANT, W.tm_cq, Z.fi, n, W.cs, nullptr, 0, nullptr, nullptr, Z.fo.inv_s, nullptr, 0, W.cinter_q,
              W.cinter_s));
  if ((n + 127) / 128 >= 74) {
    AE_TRY(gemm(c, EPI_LN_FINAL, W.tm_cinter_q, Z.fo, n, W.cinter_s, W.ch, kHidden, Z.ln2w, Z.ln2b, nullptr, d_out,
                kHidden, nullptr, nullptr));
  } else {
    AE_TRY(gemm(c, EPI_F32, W.tm_cinter_q, Z.fo, n, W.cinter_s, W.ch, kHidden, nullptr, nullptr, nullptr, W.cctx,
                kHidden, nullptr, nullptr));
    ++c->launches;
    if (launch_ln_final_rows(W.cctx, n, Z.ln2w, Z.ln2b, d_out, st))
      return fail(c, AE_ERR_CUDA, "final LayerNorm row kernel launch failed");
  }
  c->graph_kernels = c->launches - launches0;
  return 0;
}

int dev_err_fail(ae_ctx* c, int h) {
  static const char* names[] = {"ok", "producer wait timed out", "MMA wait timed out", "epilogue wait timed out",
                                "sequence length outside 1..512", "token id out of range"};
  return fail(c, AE_ERR_DEVICE, "device error %d (%s)", h, (h >= 0 && h <= 5) ? names[h] : "?");
}

// The error word read back on the stream (enqueue before the synchronisation, check after it):
// saves the synchronous copy of check_dev_err on the hot host paths.
int enqueue_err_copy(ae_ctx* c) {
  CUDA_TRY(c, cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  return 0;
}
int check_err_copied(ae_ctx* c) {
  const int h = *c->h_err;
  if (h != 0) {
    int z = 0;
    cudaMemcpy(c->d_err, &z, sizeof(int), cudaMemcpyHostToDevice);
    return dev_err_fail(c, h);
  }
  return 0;
}

int check_dev_err(ae_ctx* c) {
  int h = 0;
  CUDA_TRY(c, cudaMemcpy(&h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h != 0) {
    int z = 0;
    cudaMemcpy(c->d_err, &z, sizeof(int), cudaMemcpyHostToDevice);
    return dev_err_fail(c, h);
  }
  return 0;
}

// Packs host sequences (truncating each to 512) into h_ids / h_cu, grouped by attention length
// class (stable inside a class), so that each class's attention launch is sized for its own longest
// sequence; rows are independent, so the order changes no result. order[k] = the caller's index of
// packed sequence k; segs = the runs of one class. Validates lengths and token ids.
int pack_into(ae_ctx* c, const uint16_t* ids, const uint32_t* cu, uint32_t n, uint16_t* h_ids, uint32_t* h_cu,
              std::vector<uint32_t>& order, std::vector<AttnSegment>& segs, int* T_out, int* maxlen_out) {
  auto len_of = [&](uint32_t i) { return std::min<uint32_t>(cu[i + 1] - cu[i], kMaxPos); };
  order.resize(n);
  segs.clear();
  uint32_t filled = 0;
  // the int8 attention mode keeps the sequences below its crossover in a class of their own
  const bool i8 = c->attn_mode == AE_ATTENTION_INT8;
  auto class_of = [&](int len) { return i8 ? (len < kI8MinLen ? 0 : 1 + attn_class(len)) : attn_class(len); };
  int max_len = 0;
  // a stable counting sort of the sequences by class: counts, extremes, then placement
  constexpr int kMaxClasses = kAttnClasses + 1;
  const int n_classes = kAttnClasses + (i8 ? 1 : 0);
  uint32_t count[kMaxClasses] = {}, next[kMaxClasses] = {};
  int cmax[kMaxClasses] = {}, cmin[kMaxClasses];
  for (int k = 0; k < kMaxClasses; ++k) cmin[k] = kMaxPos;
  for (uint32_t i = 0; i < n; ++i) {
    const int len = int(len_of(i));
    const int k = class_of(len);
    ++count[k];
    cmax[k] = std::max(cmax[k], len);
    cmin[k] = std::min(cmin[k], len);
  }
  for (int k = 0; k < n_classes; ++k) {
    next[k] = filled;
    if (count[k]) segs.push_back(AttnSegment{int(filled), int(count[k]), cmax[k], cmin[k]});
    filled += count[k];
    max_len = std::max(max_len, cmax[k]);
  }
  for (uint32_t i = 0; i < n; ++i) order[next[class_of(int(len_of(i)))]++] = i;
  uint32_t off = 0;
  h_cu[0] = 0;
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t i = order[k];
    const uint32_t len = len_of(i);
    const uint16_t* src = ids + cu[i];
    uint16_t mx = 0;  // the range check as a (vectorisable) maximum; the offending id only on failure
    for (uint32_t j = 0; j < len; ++j) mx = src[j] > mx ? src[j] : mx;
    if (mx >= kVocab) {
      for (uint32_t j = 0; j < len; ++j)
        if (src[j] >= kVocab) return fail(c, AE_ERR_TOKEN_RANGE, "token id %u at sequence %u is >= 30522", src[j], i);
    }
    std::memcpy(h_ids + off, src, len * 2);
    off += len;
    h_cu[k + 1] = off;
  }
  *T_out = int(off);
  *maxlen_out = max_len;
  return 0;
}

// Checks a host batch (non-decreasing cu_seqlens, no empty sequence), reserves the workspace for it
// and packs it into the context's pinned staging buffers.
int pack_host(ae_ctx* c, const uint16_t* ids, const uint32_t* cu, uint32_t n, int* T_out, int* maxlen_out) {
  uint64_t T = 0;
  for (uint32_t i = 0; i < n; ++i) {
    if (cu[i + 1] < cu[i]) return fail(c, AE_ERR_INVALID_ARG, "cu_seqlens must be non-decreasing");
    const uint32_t len = std::min<uint32_t>(cu[i + 1] - cu[i], kMaxPos);
    if (len == 0) return fail(c, AE_ERR_INVALID_ARG, "sequence %u is empty (input_ids must not be empty)", i);
    T += len;
  }
  if (T > 0x7fffffffu) return fail(c, AE_ERR_CAPACITY, "batch too large");
  AE_TRY(reserve(c, uint32_t(T), n));
  Workspace& W = c->ws;
  return pack_into(c, ids, cu, n, W.h_ids, W.h_cu, c->order, c->segs, T_out, maxlen_out);
}

int forward_ragged_host(ae_ctx* c, const uint16_t* ids, const uint32_t* cu, uint32_t n, float* out) {
  if (!c->has_model) return fail(c, AE_ERR_NO_MODEL, "no model loaded");
  if (n == 0) return 0;
  if (!ids || !cu || !out) return fail(c, AE_ERR_INVALID_ARG, "null pointer");
  int T = 0, max_len = 0;
  AE_TRY(pack_host(c, ids, cu, n, &T, &max_len));
  Workspace& W = c->ws;
  CUDA_TRY(c, cudaMemcpyAsync(W.ids, W.h_ids, size_t(T) * 2, cudaMemcpyHostToDevice, c->stream));
  CUDA_TRY(c, cudaMemcpyAsync(W.cu, W.h_cu, size_t(n + 1) * 4, cudaMemcpyHostToDevice, c->stream));
  AE_TRY(enqueue_forward(c, W.ids, W.cu, T, int(n), max_len, W.out, &c->segs));
  CUDA_TRY(c, cudaMemcpyAsync(W.h_out, W.out, size_t(n) * kHidden * 4, cudaMemcpyDeviceToHost, c->stream));
  AE_TRY(enqueue_err_copy(c));
  CUDA_TRY(c, cudaStreamSynchronize(c->stream));
  AE_TRY(check_err_copied(c));
  bool identity = true;  // a batch of one length class keeps the caller's order: one copy
  for (uint32_t k = 0; k < n && identity; ++k) identity = c->order[k] == k;
  if (identity) {
    std::memcpy(out, W.h_out, size_t(n) * kHidden * 4);
  } else {
    for (uint32_t k = 0; k < n; ++k)
      std::memcpy(out + size_t(c->order[k]) * kHidden, W.h_out + size_t(k) * kHidden, kHidden * 4);
  }
  return 0;
}

// ------------------------------------------------------------------------------------------ .ae8 parsing
// A read-only mapping of a whole file (pages taken from the page cache up front), or its bytes read
// into memory where mapping fails.
struct MappedFile {
  const uint8_t* data = nullptr;
  size_t size = 0;
  void* map = nullptr;
  std::vector<uint8_t> copy;
  bool open(const char* path) {
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return false;
    struct stat st;
    bool ok = fstat(fd, &st) == 0 && st.st_size >= 0;
    if (ok && st.st_size > 0) {
      size = size_t(st.st_size);
      map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE | MAP_POPULATE, fd, 0);
      if (map == MAP_FAILED) {
        map = nullptr;
        copy.resize(size);
        size_t got = 0;
        while (ok && got < size) {
          const ssize_t n = ::read(fd, copy.data() + got, size - got);
          if (n <= 0) ok = false;
          else got += size_t(n);
        }
        data = copy.data();
      } else {
        data = static_cast<const uint8_t*>(map);
      }
    }
    ::close(fd);
    return ok;
  }
  ~MappedFile() {
    if (map) munmap(map, size);
  }
};

// QuantizedModelRaw::load_ae8 (src/quantize.rs:76-137) over the bytes of a pack: every tensor is a
// u64 element count followed by its data. The descriptor's pointers point into the bytes
// themselves; float arrays may sit at any byte offset, so the loader only memcpy's from them.
struct Ae8 {
  const uint8_t* data = nullptr;
  size_t size = 0;
  size_t pos = 8;
  bool ok = true;
  uint64_t u64() {
    uint64_t v = 0;
    if (!ok || size - pos < 8) {
      ok = false;
      return 0;
    }
    std::memcpy(&v, data + pos, 8);
    pos += 8;
    return v;
  }
  const int8_t* i8vec(uint64_t* n_out = nullptr) {
    const uint64_t n = u64();
    if (!ok || n > size - pos) {
      ok = false;
      return nullptr;
    }
    const int8_t* p = reinterpret_cast<const int8_t*>(data + pos);
    pos += n;
    if (n_out) *n_out = n;
    return p;
  }
  const float* f32vec(uint64_t* n_out = nullptr) {
    const uint64_t n = u64();
    if (!ok || n > (size - pos) / 4) {
      ok = false;
      return nullptr;
    }
    const float* p = reinterpret_cast<const float*>(data + pos);
    pos += n * 4;
    if (n_out) *n_out = n;
    return p;
  }
  bool linear(ae_linear_desc& d) {
    d.n_out = u64();
    d.k_in = u64();
    uint64_t nw = 0, ns = 0, nb = 0, ni = 0;
    d.w_q = i8vec(&nw);
    d.w_scale = f32vec(&ns);
    d.bias = f32vec(&nb);
    d.inv_smooth = f32vec(&ni);
    if (ok && (nw != d.n_out * d.k_in || ns != d.n_out || nb != d.n_out || ni != d.k_in)) ok = false;
    if (d.n_out == 0) d.w_q = nullptr;
    return ok;
  }
};

// Token-weighted greedy (longest first) assignment of sequences to shards. Cost of a sequence of L
// tokens: 19,759,104 L int8 MACs + 8,448 L^2 attention MACs. Each shard lists its sequences longest
// first, so the batches cut from it hold sequences of similar length.
std::vector<std::vector<uint32_t>> plan_shards(const uint32_t* cu, uint32_t n, int n_shards) {
  auto len_of = [&](uint32_t i) { return std::min<uint32_t>(cu[i + 1] - cu[i], kMaxPos); };
  std::vector<uint32_t> order(n);
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return len_of(a) > len_of(b); });
  std::vector<double> load(n_shards, 0.0);
  std::vector<std::vector<uint32_t>> shard(n_shards);
  for (uint32_t i : order) {
    const double L = len_of(i);
    const int d = int(std::min_element(load.begin(), load.end()) - load.begin());
    load[d] += 19759104.0 * L + 8448.0 * L * L;
    shard[d].push_back(i);
  }
  return shard;
}

// The device batches of one context's shard (sequence indices s, batch b = s[ends[b - 1] ..
// ends[b])), pipelined over two staging slots: while batch b runs on the GPU, the host packs batch
// b + 1 into the other slot, then waits for batch b - 1 and copies its embeddings out by index.
int run_batches(ae_ctx* c, const std::vector<uint32_t>& s, const std::vector<size_t>& ends, const uint16_t* ids,
                const uint32_t* cu, uint32_t max_tok, uint32_t max_seqs, float* out) {
  auto len_of = [&](uint32_t i) { return std::min<uint32_t>(cu[i + 1] - cu[i], kMaxPos); };
  for (auto& sl : c->pipe) {
    sl.busy = false;
    if (sl.cap_tok >= max_tok && sl.cap_seqs >= max_seqs) continue;
    const uint32_t t = std::max(max_tok, sl.cap_tok), q = std::max(max_seqs, sl.cap_seqs);
    if (sl.h_ids) cudaFreeHost(sl.h_ids);
    if (sl.h_cu) cudaFreeHost(sl.h_cu);
    if (sl.h_out) cudaFreeHost(sl.h_out);
    if (sl.d_ids) cudaFree(sl.d_ids);
    if (sl.d_cu) cudaFree(sl.d_cu);
    if (sl.d_out) cudaFree(sl.d_out);
    sl.h_ids = nullptr;
    sl.h_cu = nullptr;
    sl.h_out = nullptr;
    sl.d_ids = nullptr;
    sl.d_cu = nullptr;
    sl.d_out = nullptr;
    sl.cap_tok = sl.cap_seqs = 0;
    CUDA_TRY(c, cudaMallocHost(&sl.h_ids, size_t(t) * 2));
    CUDA_TRY(c, cudaMallocHost(&sl.h_cu, size_t(q + 1) * 4));
    CUDA_TRY(c, cudaMallocHost(&sl.h_out, size_t(q) * kHidden * 4));
    CUDA_TRY(c, cudaMalloc(&sl.d_ids, size_t(t) * 2));
    CUDA_TRY(c, cudaMalloc(&sl.d_cu, size_t(q + 1) * 4));
    CUDA_TRY(c, cudaMalloc(&sl.d_out, size_t(q) * kHidden * 4));
    if (!sl.done) CUDA_TRY(c, cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
    sl.cap_tok = t;
    sl.cap_seqs = q;
  }
  auto drain = [&](ae_ctx::PipeSlot& sl) -> int {
    if (!sl.busy) return 0;
    sl.busy = false;
    CUDA_TRY(c, cudaEventSynchronize(sl.done));
    for (uint32_t k = 0; k < sl.n; ++k)
      std::memcpy(out + size_t(sl.idx[sl.order[k]]) * kHidden, sl.h_out + size_t(k) * kHidden, kHidden * 4);
    return 0;
  };
  std::vector<uint16_t> bids;
  std::vector<uint32_t> bcu;
  int r = 0;
  size_t i = 0;
  for (size_t bi = 0; bi < ends.size() && !r; ++bi) {
    ae_ctx::PipeSlot& sl = c->pipe[bi & 1];
    if ((r = drain(sl))) break;  // batch bi - 2
    const size_t j = ends[bi];
    bids.clear();
    bcu.assign(1, 0);
    sl.idx.clear();
    uint32_t tok = 0;
    for (size_t k = i; k < j; ++k) {
      const uint32_t L = len_of(s[k]);
      bids.insert(bids.end(), ids + cu[s[k]], ids + cu[s[k]] + L);
      tok += L;
      bcu.push_back(tok);
      sl.idx.push_back(s[k]);
    }
    const uint32_t nb = uint32_t(j - i);
    int T = 0, max_len = 0;
    if ((r = pack_into(c, bids.data(), bcu.data(), nb, sl.h_ids, sl.h_cu, sl.order, sl.segs, &T, &max_len))) break;
    if (cudaMemcpyAsync(sl.d_ids, sl.h_ids, size_t(T) * 2, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(sl.d_cu, sl.h_cu, size_t(nb + 1) * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
      r = fail(c, AE_ERR_CUDA, "batch input copy failed");
      break;
    }
    if ((r = enqueue_forward(c, sl.d_ids, sl.d_cu, T, int(nb), max_len, sl.d_out, &sl.segs))) break;
    if (cudaMemcpyAsync(sl.h_out, sl.d_out, size_t(nb) * kHidden * 4, cudaMemcpyDeviceToHost, c->stream) !=
            cudaSuccess ||
        cudaEventRecord(sl.done, c->stream) != cudaSuccess) {
      r = fail(c, AE_ERR_CUDA, "batch output copy failed");
      break;
    }
    sl.n = nb;
    sl.busy = true;
    i = j;
  }
  const size_t nbat = ends.size();
  for (size_t k = 0; k < 2; ++k) {  // the last two batches, oldest first
    ae_ctx::PipeSlot& sl = c->pipe[(nbat + k) & 1];
    const int rd = drain(sl);
    if (!r) r = rd;
  }
  if (cudaStreamSynchronize(c->stream) != cudaSuccess && !r) r = fail(c, AE_ERR_CUDA, "stream synchronisation failed");
  if (!r) r = check_dev_err(c);
  return r;
}

}  // namespace

// ============================================================================================ C ABI
extern "C" {

int ae_ctx_create(int device, ae_ctx** out) {
  if (!out) return fail(nullptr, AE_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return fail(nullptr, AE_ERR_CUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
  if (device < 0 || device >= n || device >= kMaxDevices)
    return fail(nullptr, AE_ERR_INVALID_ARG, "device %d out of range (%d visible)", device, n);
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return fail(nullptr, AE_ERR_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
  if (prop.major != 10 || prop.minor != 0)
    return fail(nullptr, AE_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
                prop.minor);
  DeviceGuard g(device);
  auto* c = new ae_ctx();
  c->device = device;
  // a blocking stream: work that callers put on the legacy default stream (e.g. torch's default
  // stream preparing the inputs of ae_forward_ragged_device) is ordered with the context's work
  e = cudaStreamCreate(&c->own_stream);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&c->d_lat, (kHidden + 1) * sizeof(float));
  if (e == cudaSuccess) e = cudaMallocHost(&c->h_lat, (kHidden + 1) * sizeof(float));
  if (e == cudaSuccess) e = cudaMallocHost(&c->h_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->d_lat, 0, (kHidden + 1) * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&c->d_cu_single, sizeof(uint32_t) * 2 * (kMaxPos + 1));
  if (e == cudaSuccess) {
    std::vector<uint32_t> t(2 * (kMaxPos + 1));
    for (int L = 0; L <= kMaxPos; ++L) {
      t[2 * L] = 0;
      t[2 * L + 1] = uint32_t(L);
    }
    e = cudaMemcpy(c->d_cu_single, t.data(), t.size() * sizeof(uint32_t), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, sizeof(int));
  if (e != cudaSuccess) {
    if (c->d_err) cudaFree(c->d_err);
    if (c->d_lat) cudaFree(c->d_lat);
    if (c->h_lat) cudaFreeHost(c->h_lat);
    if (c->h_err) cudaFreeHost(c->h_err);
    if (c->d_cu_single) cudaFree(c->d_cu_single);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
    return fail(nullptr, AE_ERR_CUDA, "context setup: %s", cudaGetErrorString(e));
  }
  c->stream = c->own_stream;
  const char* gm = std::getenv("ARCTIC_GELU");
  c->gelu_erf = (gm && std::strcmp(gm, "erf") == 0) ? 1 : 0;
  const char* fq = std::getenv("ARCTIC_FUSED_QKV");
  c->fused_qkv = (fq && std::strcmp(fq, "1") == 0) ? 1 : 0;
  const char* am = std::getenv("ARCTIC_ATTN");
  c->attn_mode = (am && std::strcmp(am, "int8") == 0) ? AE_ATTENTION_INT8 : AE_ATTENTION_EXACT;
  const char* fw = std::getenv("ARCTIC_ATTN_FEW");
  c->few_mode = !fw ? 0 : std::strcmp(fw, "tmem") == 0 ? 1 : std::strcmp(fw, "narrow") == 0 ? 2 : std::strcmp(fw, "lanes8") == 0 ? 3 : std::strcmp(fw, "dm") == 0 ? 4 : 0;
  const char* lc = std::getenv("ARCTIC_LAT_CLUSTER");
  c->lat_cluster = !(lc && std::strcmp(lc, "0") == 0) && lat_prime();
  if (gemm_i8_prime() || attention_prime()) {
    ae_ctx_destroy(c);
    return fail(nullptr, AE_ERR_CUDA, "kernel attribute setup failed on device %d", device);
  }
  *out = c;
  return 0;
}

int ae_ctx_destroy(ae_ctx* c) {
  if (!c) return 0;
  DeviceGuard g(c->device);
  cudaStreamSynchronize(c->stream);
  drop_graphs(c);
  free_ws(c);
  free_model(c);
  if (c->h_model) cudaFreeHost(c->h_model);
  for (auto& sl : c->pipe) {
    if (sl.h_ids) cudaFreeHost(sl.h_ids);
    if (sl.h_cu) cudaFreeHost(sl.h_cu);
    if (sl.h_out) cudaFreeHost(sl.h_out);
    if (sl.d_ids) cudaFree(sl.d_ids);
    if (sl.d_cu) cudaFree(sl.d_cu);
    if (sl.d_out) cudaFree(sl.d_out);
    if (sl.done) cudaEventDestroy(sl.done);
  }
  for (auto& e : c->prof_events) {
    cudaEventDestroy(e.second.first);
    cudaEventDestroy(e.second.second);
  }
  for (auto e : c->prof_pool) cudaEventDestroy(e);
  if (c->d_err) cudaFree(c->d_err);
  if (c->d_lat) cudaFree(c->d_lat);
  if (c->h_lat) cudaFreeHost(c->h_lat);
  if (c->h_err) cudaFreeHost(c->h_err);
  if (c->d_cu_single) cudaFree(c->d_cu_single);
  if (c->d_gemm_scratch) cudaFree(c->d_gemm_scratch);
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete c;
  return 0;
}

const char* ae_last_error(const ae_ctx* c) { return c ? c->err.c_str() : g_create_err.c_str(); }

int ae_ctx_set_stream(ae_ctx* c, void* s) {
  if (!c) return AE_ERR_INVALID_ARG;
  drop_graphs(c);
  c->stream = s ? static_cast<cudaStream_t>(s) : c->own_stream;
  return 0;
}

int ae_ctx_device(const ae_ctx* c) { return c ? c->device : AE_ERR_INVALID_ARG; }

namespace {

// ae_model_load: validates the descriptor, builds the arena image in the context's pinned staging
// buffer and moves it with one DMA (see Uploader).
int load_model(ae_ctx* c, const ae_model_desc* d) {
  // validation (the sizes src/quantize.rs:9-18 fix; the reference asserts them while packing)
  if (!d->word_emb_q || !d->word_emb_scale || !d->pos_emb_q || !d->pos_emb_scale || !d->type_emb_q ||
      !d->type_emb_scale || !d->emb_ln_weight || !d->emb_ln_bias)
    return fail(c, AE_ERR_BAD_PACK, "embedding tables missing");
  for (int l = 0; l < kLayers; ++l) {
    const ae_layer_desc& L = d->layers[l];
    const bool last = l == kLayers - 1;
    if (!L.ln1_weight || !L.ln1_bias || !L.ln2_weight || !L.ln2_bias)
      return fail(c, AE_ERR_BAD_PACK, "layer %d: LayerNorm parameters missing", l);
    if (!check_linear(L.attn_out, kHidden, kHidden, false) || !check_linear(L.ffn_inter, kInter, kHidden, false) ||
        !check_linear(L.ffn_out, kHidden, kInter, false))
      return fail(c, AE_ERR_BAD_PACK, "layer %d: attn_out / ffn shapes must be 384x384, 1536x384, 384x1536", l);
    if (!last) {
      if (!check_linear(L.qkv, 3 * kHidden, kHidden, false))
        return fail(c, AE_ERR_BAD_PACK, "layer %d: qkv must be 1152x384", l);
    } else {
      if (L.has_split != 1 || !check_linear(L.q_only, kHidden, kHidden, false) ||
          !check_linear(L.kv_only, 2 * kHidden, kHidden, false) || L.qkv.k_in != kHidden || !L.qkv.inv_smooth ||
          (L.qkv.n_out != 0 && !check_linear(L.qkv, 3 * kHidden, kHidden, false)))
        return fail(c, AE_ERR_BAD_PACK, "layer 11 must carry the [CLS]-pruned split (q_only 384x384, kv_only 768x384)");
    }
  }
  cudaStreamSynchronize(c->stream);
  size_t bytes = size_t(kVocab) * kHidden + kVocab * 4 + kMaxPos * kHidden + kMaxPos * 4 + 3 * kHidden * 4 + 64 * 1024 +
                 align_up(sizeof(LatModel), 256);
  for (int l = 0; l < kLayers; ++l) {
    const ae_layer_desc& L = d->layers[l];
    bytes += linear_bytes(L.qkv) + linear_bytes(L.attn_out) + linear_bytes(L.ffn_inter) + linear_bytes(L.ffn_out) +
             4 * kHidden * 4 + 4096;
    if (L.has_split) bytes += linear_bytes(L.q_only) + linear_bytes(L.kv_only);
  }
  // the arena of the previous model is reused when it is large enough
  if (!c->model.arena || c->model.arena_bytes < bytes) {
    drop_graphs(c);
    free_model(c);
    void* arena = nullptr;
    CUDA_TRY(c, cudaMalloc(&arena, bytes));
    c->model.arena = arena;
    c->model.arena_bytes = bytes;
  }
  if (c->h_model_bytes < bytes) {
    if (c->h_model) cudaFreeHost(c->h_model);
    c->h_model = nullptr;
    c->h_model_bytes = 0;
    CUDA_TRY(c, cudaMallocHost(&c->h_model, bytes));
    c->h_model_bytes = bytes;
  }
  DevModel M = DevModel();
  M.arena = c->model.arena;
  M.arena_bytes = c->model.arena_bytes;
  Carve cv{static_cast<uint8_t*>(M.arena)};
  Uploader img;
  img.dev_base = static_cast<const uint8_t*>(M.arena);
  img.host = static_cast<uint8_t*>(c->h_model);
  M.word_q = cv.take<int8_t>(size_t(kVocab) * kHidden);
  M.word_s = cv.take<float>(kVocab);
  M.pos_q = cv.take<int8_t>(size_t(kMaxPos) * kHidden);
  M.pos_s = cv.take<float>(kMaxPos);
  M.type0 = cv.take<float>(kHidden);
  M.emb_lnw = cv.take<float>(kHidden);
  M.emb_lnb = cv.take<float>(kHidden);
  int r = 0;
  std::vector<float> type0(kHidden);
  float type_scale;  // the pack's float arrays need not be 4-byte aligned in a mapped file
  std::memcpy(&type_scale, d->type_emb_scale, 4);
  for (int j = 0; j < kHidden; ++j) type0[j] = float(d->type_emb_q[j]) * type_scale;  // src/model.rs:50-54
  img.put(M.word_q, d->word_emb_q, size_t(kVocab) * kHidden);
  img.put(M.word_s, d->word_emb_scale, kVocab);
  img.put(M.pos_q, d->pos_emb_q, size_t(kMaxPos) * kHidden);
  img.put(M.pos_s, d->pos_emb_scale, kMaxPos);
  img.put(M.type0, type0.data(), kHidden);
  img.put(M.emb_lnw, d->emb_ln_weight, kHidden);
  img.put(M.emb_lnb, d->emb_ln_bias, kHidden);
  for (int l = 0; l < kLayers && !r; ++l) {
    const ae_layer_desc& L = d->layers[l];
    DevLayer& D = M.layers[l];
    r = upload_linear(c, cv, img, L.qkv, D.qkv);
    if (!r && L.has_split) r = upload_linear(c, cv, img, L.q_only, D.q_only);
    if (!r && L.has_split) r = upload_linear(c, cv, img, L.kv_only, D.kv_only);
    if (!r) r = upload_linear(c, cv, img, L.attn_out, D.ao);
    if (!r) r = upload_linear(c, cv, img, L.ffn_inter, D.fi);
    if (!r) r = upload_linear(c, cv, img, L.ffn_out, D.fo);
    if (!r) {
      D.ln1w = cv.take<float>(kHidden);
      D.ln1b = cv.take<float>(kHidden);
      D.ln2w = cv.take<float>(kHidden);
      D.ln2b = cv.take<float>(kHidden);
      img.put(D.ln1w, L.ln1_weight, kHidden);
      img.put(D.ln1b, L.ln1_bias, kHidden);
      img.put(D.ln2w, L.ln2_weight, kHidden);
      img.put(D.ln2b, L.ln2_bias, kHidden);
    }
  }
  // the single-sequence cluster forward's view of the model: device pointers and 32-row tensor maps
  std::unique_ptr<LatModel> lat(new LatModel());
  if (!r) {
    std::memset(lat.get(), 0, sizeof(LatModel));
    auto lin = [](const DevLinear& x) { return LatLinear{x.ws, x.bias, x.inv_s}; };
    for (int l = 0; l < kLayers; ++l) {
      const DevLayer& D = M.layers[l];
      LatLayer& T = lat->layer[l];
      T.qkv = lin(D.qkv);
      T.q_only = lin(D.q_only);
      T.kv_only = lin(D.kv_only);
      T.ao = lin(D.ao);
      T.fi = lin(D.fi);
      T.fo = lin(D.fo);
      T.ln1w = D.ln1w;
      T.ln1b = D.ln1b;
      T.ln2w = D.ln2w;
      T.ln2b = D.ln2b;
      const DevLinear* src[LAT_MAPS] = {&D.qkv, &D.q_only, &D.kv_only, &D.ao, &D.fi, &D.fo};
      for (int k = 0; k < LAT_MAPS; ++k)
        if (src[k]->w) lat->tm[l][k] = src[k]->tmap32;
    }
    lat->word_q = M.word_q;
    lat->word_s = M.word_s;
    lat->pos_q = M.pos_q;
    lat->pos_s = M.pos_s;
    lat->type0 = M.type0;
    lat->emb_lnw = M.emb_lnw;
    lat->emb_lnb = M.emb_lnb;
    M.lat = cv.take<LatModel>(1);
    img.put(M.lat, lat.get(), 1);
  }
  if (!r && cv.off > bytes) r = fail(c, AE_ERR_BAD_PACK, "internal: model arena overflow");
  if (!r) {
    // from here on the arena's contents change: a failure leaves no model
    c->has_model = false;
    img.run();
    if (cudaMemcpyAsync(M.arena, c->h_model, cv.off, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
      r = fail(c, AE_ERR_CUDA, "model upload failed");
  }
  if (r) {
    drop_graphs(c);
    free_model(c);
    return r;
  }
  // graphs captured against the previous model stay valid only if every tensor (and so every
  // tensor map) is where it was
  if (!same_placement(M, c->model)) drop_graphs(c);
  c->model = M;
  c->has_model = true;
  return 0;
}

}  // namespace

int ae_model_load(ae_ctx* c, const ae_model_desc* d) {
  if (!c || !d) return fail(c, AE_ERR_INVALID_ARG, "null argument");
  DeviceGuard g(c->device);
  return load_model(c, d);
}

int ae_model_load_file(ae_ctx* c, const char* path) {
  if (!c || !path) return fail(c, AE_ERR_INVALID_ARG, "null argument");
  DeviceGuard g(c->device);
  MappedFile mf;
  if (!mf.open(path)) return fail(c, AE_ERR_BAD_PACK, "cannot open %s", path);
  Ae8 p;
  p.data = mf.data;
  p.size = mf.size;
  if (p.size < 8 || std::memcmp(p.data, "ARCTIC8\x01", 8) != 0)
    return fail(c, AE_ERR_BAD_PACK, "invalid .ae8 magic header");
  ae_model_desc d{};
  uint64_t n0, n1, n2, n3, n4, n5, n6, n7;
  d.word_emb_q = p.i8vec(&n0);
  d.word_emb_scale = p.f32vec(&n1);
  d.pos_emb_q = p.i8vec(&n2);
  d.pos_emb_scale = p.f32vec(&n3);
  d.type_emb_q = p.i8vec(&n4);
  d.type_emb_scale = p.f32vec(&n5);
  d.emb_ln_weight = p.f32vec(&n6);
  d.emb_ln_bias = p.f32vec(&n7);
  if (p.ok && (n0 != uint64_t(kVocab) * kHidden || n1 != uint64_t(kVocab) || n2 != uint64_t(kMaxPos) * kHidden ||
               n3 != uint64_t(kMaxPos) || n4 < uint64_t(kHidden) || n5 < 1 || n6 != uint64_t(kHidden) ||
               n7 != uint64_t(kHidden)))
    return fail(c, AE_ERR_BAD_PACK, "embedding tables have unexpected sizes");
  for (int l = 0; l < kLayers && p.ok; ++l) {
    ae_layer_desc& L = d.layers[l];
    p.linear(L.qkv);
    uint8_t split = 0;
    if (p.pos < p.size) split = p.data[p.pos++];
    else p.ok = false;
    L.has_split = split == 1;
    if (L.has_split) {
      p.linear(L.q_only);
      p.linear(L.kv_only);
    }
    p.linear(L.attn_out);
    uint64_t a, b, cc, dd;
    L.ln1_weight = p.f32vec(&a);
    L.ln1_bias = p.f32vec(&b);
    p.linear(L.ffn_inter);
    p.linear(L.ffn_out);
    L.ln2_weight = p.f32vec(&cc);
    L.ln2_bias = p.f32vec(&dd);
    if (p.ok && (a != kHidden || b != kHidden || cc != kHidden || dd != kHidden))
      return fail(c, AE_ERR_BAD_PACK, "layer %d: LayerNorm vectors must have 384 entries", l);
  }
  if (!p.ok) return fail(c, AE_ERR_BAD_PACK, "truncated or inconsistent .ae8 pack");
  return load_model(c, &d);
}

int ae_reserve(ae_ctx* c, uint32_t max_tokens, uint32_t max_seqs) {
  if (!c) return AE_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  return reserve(c, max_tokens, max_seqs);
}

int ae_forward_ragged(ae_ctx* c, const uint16_t* ids, const uint32_t* cu, uint32_t n, float* out) {
  if (!c) return AE_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  return forward_ragged_host(c, ids, cu, n, out);
}

int ae_forward_cls(ae_ctx* c, const uint16_t* ids, uint32_t len, float* out) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (!c->has_model) return fail(c, AE_ERR_NO_MODEL, "no model loaded");
  if (!ids || !out) return fail(c, AE_ERR_INVALID_ARG, "null pointer");
  if (len == 0) return fail(c, AE_ERR_INVALID_ARG, "input_ids must not be empty");
  DeviceGuard g(c->device);
  const uint32_t L = std::min<uint32_t>(len, kMaxPos);
  for (uint32_t j = 0; j < L; ++j)
    if (ids[j] >= kVocab) return fail(c, AE_ERR_TOKEN_RANGE, "token id %u at position %u is >= 30522", ids[j], j);
  AE_TRY(reserve(c, kMaxPos, 1));
  Workspace& W = c->ws;
  auto it = c->graphs.find(L);
  if (it == c->graphs.end()) {
    // capture: H2D ids, forward, D2H out, all at fixed addresses (cu_seqlens {0, L} from the
    // context's constant table)
    Graph gr;
    CUDA_TRY(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    int r = 0;
    if (cudaMemcpyAsync(W.ids, W.h_ids, L * 2, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
      r = fail(c, AE_ERR_CUDA, "capture of the input copy failed");
    const uint64_t before = c->launches;
    const bool prof = c->prof;
    c->prof = false;  // no event records inside the graph
    int* const d_err = c->d_err;
    c->d_err = reinterpret_cast<int*>(c->d_lat + kHidden);  // the graph's kernels report here
    // at most 32 tokens: the whole forward as one 12-CTA cluster kernel (the same arithmetic; the
    // int8 attention mode keeps the multi-kernel path for the sequences it covers)
    const bool one_kernel = c->lat_cluster && c->model.lat && L <= uint32_t(kLatMaxTokens) &&
                            (c->attn_mode == AE_ATTENTION_EXACT || L < uint32_t(kI8MinLen));
    if (!r && one_kernel) {
      ++c->launches;
      if (launch_forward_lat(c->model.lat, W.ids, int(L), c->d_lat, c->d_err, c->gelu_erf, c->stream))
        r = fail(c, AE_ERR_CUDA, "cluster forward launch failed");
    } else if (!r) {
      r = enqueue_forward(c, W.ids, c->d_cu_single + 2 * L, int(L), 1, int(L), c->d_lat, nullptr, int(L));
    }
    c->prof = prof;
    c->d_err = d_err;
    gr.kernels = c->launches - before;
    c->launches = before;  // captured, not launched
    if (!r && cudaMemcpyAsync(c->h_lat, c->d_lat, (kHidden + 1) * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
      r = fail(c, AE_ERR_CUDA, "capture of output copy failed");
    cudaError_t e = cudaStreamEndCapture(c->stream, &gr.g);
    if (r) {
      if (gr.g) cudaGraphDestroy(gr.g);
      return r;
    }
    if (e != cudaSuccess) return fail(c, AE_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&gr.exec, gr.g, 0);
    if (e != cudaSuccess) {
      cudaGraphDestroy(gr.g);
      return fail(c, AE_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
    }
    it = c->graphs.emplace(L, gr).first;
  }
  std::memcpy(W.h_ids, ids, L * 2);
  CUDA_TRY(c, cudaGraphLaunch(it->second.exec, c->stream));
  c->launches += it->second.kernels;
  CUDA_TRY(c, cudaStreamSynchronize(c->stream));
  int h_err = 0;
  std::memcpy(&h_err, c->h_lat + kHidden, sizeof(int));  // the graph's error word, copied with the output
  if (h_err != 0) {
    cudaMemsetAsync(c->d_lat + kHidden, 0, sizeof(int), c->stream);
    cudaStreamSynchronize(c->stream);
    return dev_err_fail(c, h_err);
  }
  std::memcpy(out, c->h_lat, kHidden * 4);
  return 0;
}

int ae_forward_ragged_device(ae_ctx* c, const uint16_t* d_ids, const uint32_t* d_cu, uint32_t n, uint32_t T,
                             uint32_t max_len, float* d_out) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (!c->has_model) return fail(c, AE_ERR_NO_MODEL, "no model loaded");
  if (n == 0) return 0;
  if (!d_ids || !d_cu || !d_out || T == 0) return fail(c, AE_ERR_INVALID_ARG, "null pointer or empty batch");
  if (max_len == 0 || max_len > uint32_t(kMaxPos)) return fail(c, AE_ERR_INVALID_ARG, "max_len must be 1..512");
  DeviceGuard g(c->device);
  AE_TRY(reserve(c, T, n));
  return enqueue_forward(c, d_ids, d_cu, int(T), int(n), int(max_len), d_out);
}

uint64_t ae_kernel_launches(const ae_ctx* c) { return c ? c->launches : 0; }

int ae_profile(ae_ctx* c, int enable) {
  if (!c) return AE_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  for (auto& e : c->prof_events) {
    c->prof_pool.push_back(e.second.first);
    c->prof_pool.push_back(e.second.second);
  }
  c->prof_events.clear();
  c->prof = enable != 0;
  return 0;
}

int ae_profile_read(ae_ctx* c, float* total_ms, uint32_t* launches) {
  if (!c || !total_ms || !launches) return AE_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  for (int k = 0; k < AE_KERNEL_KINDS; ++k) {
    total_ms[k] = 0.0f;
    launches[k] = 0;
  }
  for (auto& e : c->prof_events) {
    float ms = 0.0f;
    CUDA_TRY(c, cudaEventElapsedTime(&ms, e.second.first, e.second.second));
    total_ms[e.first] += ms;
    launches[e.first] += 1;
  }
  return 0;
}

int ae_plan_shards(const uint32_t* cu, uint32_t n, int n_shards, int32_t* shard_of) {
  if (!cu || !shard_of || n_shards <= 0) return AE_ERR_INVALID_ARG;
  for (uint32_t i = 0; i < n; ++i)
    if (cu[i + 1] < cu[i]) return AE_ERR_INVALID_ARG;
  const auto plan = plan_shards(cu, n, n_shards);
  for (int d = 0; d < n_shards; ++d)
    for (uint32_t i : plan[d]) shard_of[i] = d;
  return 0;
}

int ae_sync(ae_ctx* c) {
  if (!c) return AE_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  CUDA_TRY(c, cudaStreamSynchronize(c->stream));
  return check_dev_err(c);
}

int ae_gemm_i8(ae_ctx* c, int epi, uint32_t M, uint32_t N, uint32_t K, const int8_t* d_a, const float* d_a_scale,
               const int8_t* d_w, const float* d_w_scale, const float* d_bias, const float* d_res, const float* d_gamma,
               const float* d_beta, const float* d_inv_smooth, float* d_out, int8_t* d_out_q, float* d_out_scale,
               int32_t* d_acc) {
  if (!c) return AE_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  if (!d_a || !d_a_scale || !d_w || !d_w_scale || !d_bias || M == 0 || K % 128)
    return fail(c, AE_ERR_INVALID_ARG, "ae_gemm_i8: bad arguments");
  {  // the epilogues use 16-byte vector loads and stores
    const void* ptrs[] = {d_a_scale, d_w_scale, d_bias, d_res, d_gamma, d_beta, d_inv_smooth, d_out, d_out_q,
                          d_out_scale, d_acc};
    for (const void* q : ptrs)
      if (reinterpret_cast<uintptr_t>(q) & 15u)
        return fail(c, AE_ERR_INVALID_ARG, "ae_gemm_i8: every device pointer must be 16-byte aligned");
  }
  CUtensorMap ta, tb;
  if (make_tmap_i8(&ta, d_a, int(M), int(K), kBoxA) || make_tmap_i8(&tb, d_w, int(N), int(K), kBoxB))
    return fail(c, AE_ERR_INVALID_ARG, "ae_gemm_i8: operands must be 16-byte aligned");
  GemmArgs a{};
  a.M = int(M);
  a.N = int(N);
  a.K = int(K);
  a.a_scale = d_a_scale;
  a.w_scale = d_w_scale;
  a.bias = d_bias;
  a.res = d_res;
  a.ldr = int(N);
  a.gamma = d_gamma;
  a.beta = d_beta;
  a.inv_smooth = d_inv_smooth;
  a.out_f32 = d_out;
  a.ldo = int(N);
  a.out_q = d_out_q;
  a.out_scale = d_out_scale;
  a.acc_dbg = d_acc;
  a.err = c->d_err;
  a.gelu_erf = c->gelu_erf;
  switch (epi) {
    case EPI_F32:
      if (!d_out || N % 64) return fail(c, AE_ERR_INVALID_ARG, "epilogue 0 needs out and N a multiple of 128 or 192");
      break;
    case EPI_LN_QUANT:
      if (N != kHidden || !d_res || !d_gamma || !d_beta || !d_inv_smooth || !d_out || !d_out_q || !d_out_scale)
        return fail(c, AE_ERR_INVALID_ARG, "epilogue 1 needs N = 384 and res, gamma, beta, inv_smooth, outputs");
      break;
    case EPI_GELU_QUANT:
      if (N != kInter || !d_inv_smooth || !d_out_q || !d_out_scale)
        return fail(c, AE_ERR_INVALID_ARG, "epilogue 2 needs N = 1536 and inv_smooth, out_q, out_scale");
      break;
    case EPI_LN_FINAL:
      if (N != kHidden || !d_res || !d_gamma || !d_beta || !d_out)
        return fail(c, AE_ERR_INVALID_ARG, "epilogue 3 needs N = 384 and res, gamma, beta, out");
      break;
    default:
      return fail(c, AE_ERR_INVALID_ARG, "unknown epilogue %d", epi);
  }
  if ((epi == EPI_LN_QUANT || epi == EPI_LN_FINAL) && (M + 127) / 128 < 74) {
    // few row tiles (fewer than half the SMs): as the forward does, a plain-epilogue GEMM over
    // narrow column slices writes h = fma(acc, as*ws, bias + res) into scratch and a row kernel
    // applies the same LayerNorm (and quantization) -- the same bits as the fused epilogue
    if (c->gemm_scratch_rows < M) {
      if (c->d_gemm_scratch) {
        CUDA_TRY(c, cudaStreamSynchronize(c->stream));
        cudaFree(c->d_gemm_scratch);
        c->d_gemm_scratch = nullptr;
        c->gemm_scratch_rows = 0;
      }
      CUDA_TRY(c, cudaMalloc(&c->d_gemm_scratch, size_t(M) * kHidden * sizeof(float)));
      c->gemm_scratch_rows = M;
    }
    GemmArgs h = a;
    h.out_f32 = c->d_gemm_scratch;
    h.ldo = kHidden;
    h.out_q = nullptr;
    h.out_scale = nullptr;
    const int r = gemm_i8_launch(EPI_F32, ta, tb, h, c->stream);
    if (r) return fail(c, AE_ERR_CUDA, "GEMM launch failed (split LayerNorm path): code %d", r);
    const int q = epi == EPI_LN_QUANT
                      ? launch_ln_quant_rows(c->d_gemm_scratch, int(M), d_gamma, d_beta, d_inv_smooth, d_out, 0,
                                             d_out_q, d_out_scale, c->stream)
                      : launch_ln_final_rows(c->d_gemm_scratch, int(M), d_gamma, d_beta, d_out, c->stream);
    if (q) return fail(c, AE_ERR_CUDA, "LayerNorm row kernel launch failed");
    return 0;
  }
  const int r = gemm_i8_launch(epi, ta, tb, a, c->stream);
  if (r) return fail(c, AE_ERR_CUDA, "GEMM launch failed: code %d", r);
  return 0;
}

int ae_measure_int8_peak(ae_ctx* c, uint32_t iters, float* ms, double* tops) {
  if (!c || !ms || !tops || iters == 0 || iters > 1000000)
    return fail(c, AE_ERR_INVALID_ARG, "ae_measure_int8_peak: iters must be 1..1000000 and outputs non-null");
  DeviceGuard g(c->device);
  int ctas = 0;
  if (i8_peak_launch(int(std::min<uint32_t>(iters, 1000)), c->d_err, c->stream, &ctas))  // warm-up
    return fail(c, AE_ERR_CUDA, "peak probe launch failed");
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  CUDA_TRY(c, cudaEventCreate(&e0));
  CUDA_TRY(c, cudaEventCreate(&e1));
  cudaEventRecord(e0, c->stream);
  const int r = i8_peak_launch(int(iters), c->d_err, c->stream, &ctas);
  cudaEventRecord(e1, c->stream);
  const cudaError_t e = cudaEventSynchronize(e1);
  float t = 0.0f;
  if (e == cudaSuccess) cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  c->launches += 2;
  if (r) return fail(c, AE_ERR_CUDA, "peak probe launch failed");
  if (e != cudaSuccess) return fail(c, AE_ERR_CUDA, "peak probe: %s", cudaGetErrorString(e));
  AE_TRY(check_dev_err(c));
  *ms = t;
  *tops = t > 0.0f ? i8_peak_ops(int(iters), ctas) / (double(t) * 1e-3) / 1e12 : 0.0;
  return 0;
}

int ae_selftest_wait_timeout(ae_ctx* c, uint32_t limit_us) {
  if (!c || limit_us == 0 || limit_us > 1000000) return fail(c, AE_ERR_INVALID_ARG, "limit_us must be 1..1000000");
  DeviceGuard g(c->device);
  if (launch_wait_selftest(c->d_err, uint64_t(limit_us) * 1000, c->stream))
    return fail(c, AE_ERR_CUDA, "self-test launch failed");
  CUDA_TRY(c, cudaStreamSynchronize(c->stream));
  return check_dev_err(c);
}

int ae_attention_f32(ae_ctx* c, const float* d_qkv, const uint32_t* d_cu, uint32_t n, uint32_t max_len, float* d_ctx) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (!d_qkv || !d_cu || !d_ctx || max_len == 0 || max_len > uint32_t(kMaxPos))
    return fail(c, AE_ERR_INVALID_ARG, "ae_attention_f32: bad arguments");
  DeviceGuard g(c->device);
  return attention(c, d_qkv, 3 * kHidden, 0, 0, d_qkv, 3 * kHidden, kHidden, 2 * kHidden, 0, d_ctx, d_cu, int(n),
                   int(max_len), 0);
}

int ae_attention_i8(ae_ctx* c, const float* d_qkv, const uint32_t* d_cu, uint32_t n, uint32_t max_len, float* d_ctx) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (!d_qkv || !d_cu || !d_ctx || max_len == 0 || max_len > uint32_t(kMaxPos))
    return fail(c, AE_ERR_INVALID_ARG, "ae_attention_i8: bad arguments");
  if (n == 0) return 0;
  DeviceGuard g(c->device);
  AttnArgs a{};
  a.q = d_qkv;
  a.q_C = 3 * kHidden;
  a.kv = d_qkv;
  a.kv_C = 3 * kHidden;
  a.k_col = kHidden;
  a.v_col = 2 * kHidden;
  a.out = d_ctx;
  a.cu = d_cu;
  a.max_len = int(max_len);
  a.err = c->d_err;
  ++c->launches;
  if (launch_attention_i8(a, int(n), 1, c->stream)) return fail(c, AE_ERR_CUDA, "int8 attention launch failed");
  return 0;
}

int ae_set_attention_mode(ae_ctx* c, int mode) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (mode != AE_ATTENTION_EXACT && mode != AE_ATTENTION_INT8)
    return fail(c, AE_ERR_INVALID_ARG, "unknown attention mode %d", mode);
  if (mode != c->attn_mode) {
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    drop_graphs(c);
    c->attn_mode = mode;
  }
  return 0;
}

int ae_get_attention_mode(const ae_ctx* c) { return c ? c->attn_mode : AE_ERR_INVALID_ARG; }

int ae_trace_forward(ae_ctx* c, const uint16_t* ids, const uint32_t* cu, uint32_t n, int stage, float* f32, int8_t* q,
                     float* scale) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (!c->has_model) return fail(c, AE_ERR_NO_MODEL, "no model loaded");
  if (stage != AE_TRACE_EMBED && stage != AE_TRACE_ATTN0) return fail(c, AE_ERR_INVALID_ARG, "unknown stage %d", stage);
  if (!ids || !cu || !f32 || !q || !scale || n == 0) return fail(c, AE_ERR_INVALID_ARG, "null pointer or no sequence");
  DeviceGuard g(c->device);
  int T = 0, max_len = 0;
  AE_TRY(pack_host(c, ids, cu, n, &T, &max_len));
  Workspace& W = c->ws;
  CUDA_TRY(c, cudaMemcpyAsync(W.ids, W.h_ids, size_t(T) * 2, cudaMemcpyHostToDevice, c->stream));
  CUDA_TRY(c, cudaMemcpyAsync(W.cu, W.h_cu, size_t(n + 1) * 4, cudaMemcpyHostToDevice, c->stream));
  const bool prof = c->prof;
  c->prof = false;
  int r = enqueue_forward(c, W.ids, W.cu, T, int(n), max_len, W.out, &c->segs, 1, stage);
  // an attention kernel that quantized the context rows itself did not store them in fp32: run the
  // same attention once more without the quantization (the rows it computes are the same bits)
  if (!r && stage == AE_TRACE_ATTN0 && c->attn_mode == AE_ATTENTION_EXACT)
    r = attention(c, W.qkv, 3 * kHidden, 0, 1, W.qkv, 3 * kHidden, kHidden, 2 * kHidden, 1, W.ctx, W.cu, int(n), max_len,
                  0, &c->segs);
  c->prof = prof;
  AE_TRY(r);
  const size_t Tp = align_up(size_t(T), 128);
  std::vector<float> rows(Tp * kHidden);
  std::vector<int8_t> qr(size_t(T) * kHidden);
  std::vector<float> sr(T);
  CUDA_TRY(c, cudaMemcpyAsync(rows.data(), stage == AE_TRACE_EMBED ? W.hidden : W.ctx,
                              (stage == AE_TRACE_EMBED ? Tp : size_t(T)) * kHidden * 4, cudaMemcpyDeviceToHost,
                              c->stream));
  CUDA_TRY(c, cudaMemcpyAsync(qr.data(), W.act_q, qr.size(), cudaMemcpyDeviceToHost, c->stream));
  CUDA_TRY(c, cudaMemcpyAsync(sr.data(), W.act_s, sr.size() * 4, cudaMemcpyDeviceToHost, c->stream));
  CUDA_TRY(c, cudaStreamSynchronize(c->stream));
  AE_TRY(check_dev_err(c));
  // packed rows -> the caller's order; the hidden state is tile-transposed: (t, j) at
  // ((t >> 7) * 384 + j) * 128 + (t & 127)
  std::vector<uint32_t> dst0(n);
  uint32_t off = 0;
  for (uint32_t i = 0; i < n; ++i) {
    dst0[i] = off;
    off += std::min<uint32_t>(cu[i + 1] - cu[i], kMaxPos);
  }
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t i = c->order[k];
    for (uint32_t t = W.h_cu[k]; t < W.h_cu[k + 1]; ++t) {
      const size_t d = dst0[i] + (t - W.h_cu[k]);
      if (stage == AE_TRACE_EMBED) {
        for (int j = 0; j < kHidden; ++j) f32[d * kHidden + j] = rows[((size_t(t) >> 7) * kHidden + j) * 128 + (t & 127)];
      } else {
        std::memcpy(f32 + d * kHidden, &rows[size_t(t) * kHidden], kHidden * 4);
      }
      std::memcpy(q + d * kHidden, &qr[size_t(t) * kHidden], kHidden);
      scale[d] = sr[t];
    }
  }
  return 0;
}

// ArcticEmbedS::embed_batch (src/lib.rs:138-260) across GPUs: token-weighted greedy shards, one host
// thread per context; each context packs its shard (longest first) into batches of <= max_tokens.
int ae_embed_batch_multi(ae_ctx* const* ctxs, int n_ctx, const uint16_t* ids, const uint32_t* cu, uint32_t n,
                         uint32_t max_tokens, float* out) {
  if (!ctxs || n_ctx <= 0) return fail(nullptr, AE_ERR_INVALID_ARG, "no contexts");
  if (n == 0) return 0;
  if (!ids || !cu || !out) return fail(ctxs[0], AE_ERR_INVALID_ARG, "null pointer");
  if (max_tokens == 0) max_tokens = 65536;
  max_tokens = std::max<uint32_t>(max_tokens, kMaxPos);
  for (uint32_t i = 0; i < n; ++i) {
    if (cu[i + 1] < cu[i]) return fail(ctxs[0], AE_ERR_INVALID_ARG, "cu_seqlens must be non-decreasing");
    if (cu[i + 1] == cu[i]) return fail(ctxs[0], AE_ERR_INVALID_ARG, "sequence %u is empty (input_ids must not be empty)", i);
  }
  auto len_of = [&](uint32_t i) { return std::min<uint32_t>(cu[i + 1] - cu[i], kMaxPos); };
  std::vector<std::vector<uint32_t>> shard = plan_shards(cu, n, n_ctx);
  std::vector<int> rc(n_ctx, 0);
  auto worker = [&](int d) {
    ae_ctx* c = ctxs[d];
    DeviceGuard g(c->device);
    // longest first: each batch then holds sequences of similar length (tight attention launches)
    std::vector<uint32_t> s = shard[d];
    std::stable_sort(s.begin(), s.end(), [&](uint32_t x, uint32_t y) { return len_of(x) > len_of(y); });
    // batch boundaries first, so that the workspace is sized once for the largest batch
    std::vector<size_t> ends;
    uint32_t most_tok = 0, most_seqs = 0;
    for (size_t i = 0; i < s.size();) {
      size_t j = i;
      uint32_t tok = 0;
      while (j < s.size() && tok + len_of(s[j]) <= max_tokens) tok += len_of(s[j++]);
      ends.push_back(j);
      most_tok = std::max(most_tok, tok);
      most_seqs = std::max<uint32_t>(most_seqs, uint32_t(j - i));
      i = j;
    }
    if (s.empty()) return;
    rc[d] = reserve(c, most_tok, most_seqs);
    if (!rc[d]) rc[d] = run_batches(c, s, ends, ids, cu, most_tok, most_seqs, out);
  };
  std::vector<std::thread> th;
  for (int d = 1; d < n_ctx; ++d) th.emplace_back(worker, d);
  worker(0);
  for (auto& t : th) t.join();
  for (int d = 0; d < n_ctx; ++d)
    if (rc[d]) {
      if (d != 0) ctxs[0]->err = "context " + std::to_string(d) + ": " + ctxs[d]->err;
      return rc[d];
    }
  return 0;
}

}  // extern "C"

// ============================================================================================
// Allocation-free single-sequence forward.
//
// Some callers cannot call cudaMalloc at the time they embed: hosts whose device memory is handed
// out once at start-up by their own pool (a service with a fixed memory budget), and real-time
// paths that must not block on the allocator (cudaMalloc / cudaFree can synchronise the device).
// ae_forward_cls_noalloc serves them: its scratch (the activations of one <= 512-token sequence,
// about 6 MB) lives in the file-scope device array below instead of the context's cudaMalloc'd
// workspace, so the call itself allocates nothing.
namespace {

constexpr size_t kNoAllocBytes = size_t(8) << 20;  // 8 MiB: holds the workspace of one 512-token sequence
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

// Per-device view of g_noalloc_scratch: its device address (from cudaGetSymbolAddress, not the
// host-side name) carved into a Workspace, with tensor maps for the GEMM A operands. The address
// belongs to the CUDA context the module was loaded in: after a device reset (or any teardown of
// the primary context) the array can move, so the view records its context's id and is rebuilt
// when the current context differs.
struct NoAllocState {
  bool ready = false;
  unsigned long long ctx_id = 0;
  Workspace ws;
};
NoAllocState g_noalloc[kMaxDevices];
std::mutex g_noalloc_mu;

// Unique id of the calling thread's current CUDA context (cuCtxGetId: ids are never reused within
// a process), or 0 when the driver cannot report it.
unsigned long long current_ctx_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext cx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&cx) != CUDA_SUCCESS || !cx || get_id(cx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

__global__ void k_noalloc_cu(uint32_t* cu, uint32_t len) {
  cu[0] = 0;
  cu[1] = len;
}

int noalloc_setup(ae_ctx* c, NoAllocState& st, unsigned long long ctx_id) {
  st.ready = false;
  void* base = nullptr;
  CUDA_TRY(c, cudaGetSymbolAddress(&base, g_noalloc_scratch));
  st.ws = Workspace();
  Workspace& w = st.ws;
  const size_t T = kMaxPos, B = 128;  // one sequence; [CLS] buffers keep the 128-row tile height
  Carve cv{static_cast<uint8_t*>(base)};
  w.ids = cv.take<uint16_t>(T);
  w.cu = cv.take<uint32_t>(B + 1);
  w.pos = cv.take<uint16_t>(T);
  w.cls_row = cv.take<int32_t>(B);
  w.hidden = cv.take<float>(T * kHidden);
  w.act_q = cv.take<int8_t>(T * kHidden);
  w.act_s = cv.take<float>(T);
  w.qkv = cv.take<float>(T * 3 * kHidden);
  w.ctx = cv.take<float>(T * kHidden);
  w.inter_q = cv.take<int8_t>(T * kInter);
  w.inter_s = cv.take<float>(T);
  w.cq = cv.take<int8_t>(B * kHidden);
  w.cs = cv.take<float>(B);
  w.ch = cv.take<float>(B * kHidden);
  w.q_cls = cv.take<float>(B * kHidden);
  w.cctx = cv.take<float>(B * kHidden);
  w.cinter_q = cv.take<int8_t>(B * kInter);
  w.cinter_s = cv.take<float>(B);
  w.out = cv.take<float>(B * kHidden);
  if (cv.off > kNoAllocBytes) return fail(c, AE_ERR_CAPACITY, "internal: static scratch too small");
  w.cap_tokens = uint32_t(T);
  w.cap_seqs = uint32_t(B);
  if (make_tmap_i8(&w.tm_act_q, w.act_q, int(T), kHidden, kBoxA) || make_tmap_i8(&w.tm_inter_q, w.inter_q, int(T), kInter, kBoxA) ||
      make_tmap_i8(&w.tm_cq, w.cq, int(B), kHidden, kBoxA) || make_tmap_i8(&w.tm_cinter_q, w.cinter_q, int(B), kInter, kBoxA))
    return fail(c, AE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the static scratch");
  st.ctx_id = ctx_id;
  st.ready = true;
  return 0;
}

}  // namespace

extern "C" int ae_forward_cls_noalloc(ae_ctx* c, const uint16_t* d_ids, uint32_t len, float* d_out384) {
  if (!c) return AE_ERR_INVALID_ARG;
  if (!c->has_model) return fail(c, AE_ERR_NO_MODEL, "no model loaded");
  if (!d_ids || !d_out384) return fail(c, AE_ERR_INVALID_ARG, "null pointer");
  if (len == 0 || len > uint32_t(kMaxPos))
    return fail(c, AE_ERR_CAPACITY,
                "ae_forward_cls_noalloc takes 1..512 token ids (its static scratch holds one 512-token sequence); "
                "got %u",
                len);
  DeviceGuard g(c->device);
  NoAllocState& st = g_noalloc[c->device];
  Workspace W;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    const unsigned long long id = current_ctx_id();
    if (!st.ready || (id != 0 && id != st.ctx_id)) AE_TRY(noalloc_setup(c, st, id));
    W = st.ws;
  }
  k_noalloc_cu<<<1, 1, 0, c->stream>>>(W.cu, len);
  CUDA_TRY(c, cudaGetLastError());
  ++c->launches;
  // run the forward on the static scratch: the context's own workspace is set aside for the call,
  // and so is per-kernel profiling (its host-side events are not part of this call's contract)
  Workspace saved = c->ws;
  const bool prof = c->prof;
  c->ws = W;
  c->prof = false;
  const int r = enqueue_forward(c, d_ids, W.cu, int(len), 1, int(len), d_out384, nullptr, int(len));
  c->ws = saved;
  c->prof = prof;
  return r;
}
