// Host side of the C ABI declared in include/vxg_attn_cuda.h.
//
// Conventions follow the reference's native GPU ABI (native/abi.h, native/util.hpp,
// native/cuda.cu): opaque handles, int status + message buffer, a failed call synchronises its
// stream before returning, and a device error poisons the context (docs/GPU.md:5-8).
#include "vxg_attn_cuda.h"
#include "kernels.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <initializer_list>
#include <map>
#include <set>
#include <string>
#include <vector>

namespace {

constexpr const char* kVersion = "vxg-attn-cuda 0.1.0 (sm_100a)";

struct AbiError : std::runtime_error {
  int code;
  AbiError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_msg(char* dst, size_t cap, const std::string& m) {
  if (dst && cap) std::snprintf(dst, cap, "%s", m.c_str());
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw AbiError(VXG_ATTN_ERR_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
}

void require(bool ok, int code, const char* what) {
  if (!ok) throw AbiError(code, what);
}

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  void reserve(size_t bytes, const char* what) {
    if (bytes <= n) return;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    size_t want = bytes < 4096 ? 4096 : bytes + bytes / 4;
    check(cudaMalloc(&p, want), what);
    n = want;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
};

// Carves 256-byte aligned sub-buffers out of one device allocation.
struct Carver {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  }
};

struct Ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  uint32_t* d_status = nullptr;
  uint32_t* h_status = nullptr;
  bool poisoned = false;
  std::string poison;
  int force_generic = 0;
  bool timing = false;
  std::vector<cudaEvent_t> ev;  // pairs (begin, end) of timed split passes
  size_t ev_used = 0;           // events recorded since the last reset (pairs * 2)
  DevBuf part;                  // split-KV partials
  DevBuf io;                    // device staging for host-memory calls
  DevBuf aux;                   // prepared q / gate / rope table for the drop-in step
  DevBuf aux2;                  // DeltaNet scratch (conv output, normalised q/k, gates)
  DevBuf pre;                   // prefill: dequantised f16 cache
  std::set<struct Kv*> pools;   // KV pools created on this context (orphaned on destroy)
  // Overlapped host-memory decode steps (vxg_attn_cuda_q8_decode_host_async): two staging
  // slots; uploads and downloads run on their own streams, so the copies of step t+1 and t-1
  // overlap the kernels of step t on `stream`.
  struct Slot {
    DevBuf buf;                    // inputs, output and a status word of one step
    uint32_t* h_status = nullptr;  // pinned copy of the step's status word
    cudaEvent_t up = nullptr, done = nullptr, down = nullptr;
    uint64_t ticket = 0;           // step held by the slot (0: none)
    bool open = false;             // its outcome has not been collected yet
  };
  Slot slot[2];
  cudaStream_t up_stream = nullptr, down_stream = nullptr;
  uint64_t next_ticket = 1;
  struct Outcome { int code; std::string msg; };
  std::map<uint64_t, Outcome> outcomes;  // collected, not yet waited for
};

struct Kv {
  Ctx* ctx = nullptr;           // nullptr once the owning context has been destroyed
  int device = 0;
  uint32_t n_seq = 0, n_kv = 0, hd = 0, cap = 0;
  bool f32 = false;             // fp32 K/V (KvCacheMode::Fp32) instead of Q8_0 blocks
  uint8_t* k = nullptr;
  uint8_t* v = nullptr;
  size_t tok_bytes() const {
    return f32 ? (size_t)n_kv * hd * sizeof(float) : (size_t)n_kv * (hd / 32) * vxg::kBlk;
  }
  size_t seq_bytes() const { return (size_t)cap * tok_bytes(); }
};

Ctx& use_ctx(void* h) {
  require(h != nullptr, VXG_ATTN_ERR_NULL_PTR, "null context");
  Ctx& c = *static_cast<Ctx*>(h);
  if (c.poisoned)
    throw AbiError(VXG_ATTN_ERR_INTERNAL, "context poisoned by an earlier device error: " + c.poison);
  check(cudaSetDevice(c.device), "cudaSetDevice");
  return c;
}

Kv& use_kv(Ctx& c, void* h) {
  require(h != nullptr, VXG_ATTN_ERR_NULL_PTR, "null KV pool");
  Kv& kv = *static_cast<Kv*>(h);
  require(kv.device == c.device, VXG_ATTN_ERR_INVALID_OPTION,
          "the KV pool lives on another device than this context");
  return kv;
}
Kv& use_q8(Ctx& c, void* h) {
  Kv& kv = use_kv(c, h);
  require(!kv.f32, VXG_ATTN_ERR_INVALID_OPTION, "this operation needs a Q8_0 KV pool");
  return kv;
}
Kv& use_f32(Ctx& c, void* h) {
  Kv& kv = use_kv(c, h);
  require(kv.f32, VXG_ATTN_ERR_INVALID_OPTION, "this operation needs an fp32 KV pool");
  return kv;
}

// Runs `body` with the reference's error discipline.
template <class F>
int guarded(void* ctx, void* stream, char* err, size_t cap, F&& body) {
  try {
    return body();
  } catch (const AbiError& e) {
    if (ctx) {
      Ctx* c = static_cast<Ctx*>(ctx);
      cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
      // A failed call must never leave a copy targeting caller memory (native/cuda.cu:62-65).
      cudaError_t se = st ? cudaStreamSynchronize(st) : cudaSuccess;
      for (cudaStream_t cs : {c->up_stream, c->down_stream}) {
        const cudaError_t ce = cs ? cudaStreamSynchronize(cs) : cudaSuccess;
        if (se == cudaSuccess) se = ce;
      }
      if (e.code == VXG_ATTN_ERR_INTERNAL || se != cudaSuccess) {
        c->poisoned = true;
        c->poison = e.what();
      }
    }
    set_msg(err, cap, e.what());
    return e.code;
  } catch (const std::exception& e) {
    set_msg(err, cap, e.what());
    return VXG_ATTN_ERR_INTERNAL;
  }
}

// Reads and clears the device status word (stream already synchronised) and maps it to a code.
int collect_status(Ctx& c, cudaStream_t st) {
  check(cudaMemcpyAsync(c.h_status, c.d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost, st),
        "status readback");
  check(cudaMemsetAsync(c.d_status, 0, sizeof(uint32_t), st), "status reset");
  check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  const uint32_t s = *c.h_status;
  if (s & vxg::kStatusTimeout)
    throw AbiError(VXG_ATTN_ERR_INTERNAL, "a device-side bounded wait gave up");
  if (s & vxg::kStatusBadIndex)
    throw AbiError(VXG_ATTN_ERR_INVALID_OPTION,
                   "a sequence id or position was outside the KV pool; that entry was skipped");
  if (s & vxg::kStatusNonFinite) return VXG_ATTN_WARN_NONFINITE;
  return VXG_ATTN_OK;
}

// Outcome of a device status word, with the codes collect_status maps it to.
int status_outcome(uint32_t s, std::string* msg) {
  if (s & vxg::kStatusTimeout) {
    *msg = "a device-side bounded wait gave up";
    return VXG_ATTN_ERR_INTERNAL;
  }
  if (s & vxg::kStatusBadIndex) {
    *msg = "a sequence id or position was outside the KV pool; that entry was skipped";
    return VXG_ATTN_ERR_INVALID_OPTION;
  }
  if (s & vxg::kStatusNonFinite) return VXG_ATTN_WARN_NONFINITE;
  return VXG_ATTN_OK;
}

// Streams, events and pinned status words of the overlapped host-memory path (first use).
void ensure_overlap(Ctx& c) {
  if (c.down_stream) return;
  for (auto& sl : c.slot) {
    for (cudaEvent_t* e : {&sl.up, &sl.done, &sl.down})
      if (!*e) check(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate");
    if (!sl.h_status) {
      check(cudaMallocHost(&sl.h_status, sizeof(uint32_t)), "cudaMallocHost status");
      *sl.h_status = 0;
    }
  }
  if (!c.up_stream)
    check(cudaStreamCreateWithFlags(&c.up_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  check(cudaStreamCreateWithFlags(&c.down_stream, cudaStreamNonBlocking), "cudaStreamCreate");
}

// Waits for the step held by `sl` (output and status word back on the host) and files its
// outcome under its ticket.
void collect_slot(Ctx& c, Ctx::Slot& sl) {
  if (!sl.open) return;
  check(cudaEventSynchronize(sl.down), "cudaEventSynchronize");
  Ctx::Outcome o;
  o.code = status_outcome(*sl.h_status, &o.msg);
  c.outcomes[sl.ticket] = o;
  sl.open = false;
  while (c.outcomes.size() > 4096) c.outcomes.erase(c.outcomes.begin());  // never waited for
}

// Stages host inputs into the context's device staging buffer.
struct Stager {
  Ctx& c;
  cudaStream_t st;
  bool host;
  Carver carve;
  struct In { const void* src; size_t bytes; size_t off; };
  struct Out { void* dst; size_t bytes; size_t off; };
  std::vector<In> ins;
  std::vector<Out> outs;
  std::vector<std::pair<const void**, size_t>> in_slots;
  std::vector<std::pair<void**, size_t>> out_slots;

  Stager(Ctx& c_, cudaStream_t st_, bool host_) : c(c_), st(st_), host(host_) {}
  template <class T>
  void in(const T*& p, size_t bytes) {
    if (!host || !p || bytes == 0) return;
    const size_t off = carve.take(bytes);
    ins.push_back({p, bytes, off});
    in_slots.push_back({reinterpret_cast<const void**>(&p), off});
  }
  // In-out buffers (state) are both uploaded and downloaded.
  template <class T>
  void inout(T*& p, size_t bytes) {
    if (!host || !p || bytes == 0) return;
    const size_t off = carve.take(bytes);
    ins.push_back({p, bytes, off});
    outs.push_back({p, bytes, off});
    out_slots.push_back({reinterpret_cast<void**>(&p), off});
  }
  template <class T>
  void out(T*& p, size_t bytes) {
    if (!host || !p || bytes == 0) return;
    const size_t off = carve.take(bytes);
    outs.push_back({p, bytes, off});
    out_slots.push_back({reinterpret_cast<void**>(&p), off});
  }
  void upload() {
    if (!host) return;
    c.io.reserve(carve.off, "cudaMalloc staging");
    uint8_t* base = static_cast<uint8_t*>(c.io.p);
    for (auto& i : ins)
      check(cudaMemcpyAsync(base + i.off, i.src, i.bytes, cudaMemcpyHostToDevice, st), "upload");
    for (auto& s : in_slots) *s.first = base + s.second;
    for (auto& s : out_slots) *s.first = base + s.second;
  }
  void download() {
    if (!host) return;
    uint8_t* base = static_cast<uint8_t*>(c.io.p);
    for (auto& o : outs)
      check(cudaMemcpyAsync(o.dst, base + o.off, o.bytes, cudaMemcpyDeviceToHost, st), "download");
  }
};

cudaStream_t pick_stream(Ctx& c, void* stream) { return stream ? (cudaStream_t)stream : c.stream; }

int finish(Ctx& c, void* stream, cudaStream_t st) {
  if (stream) return VXG_ATTN_OK;  // asynchronous: status is collected by vxg_attn_cuda_sync
  return collect_status(c, st);
}

void record_timing(Ctx& c, cudaEvent_t* e0, cudaEvent_t* e1) {
  *e0 = *e1 = nullptr;
  if (!c.timing) return;
  if (c.ev_used + 2 > c.ev.size()) {
    // keep at most 4096 timed passes; older ones are folded away by a reset
    if (c.ev.size() >= 8192) return;
    for (int i = 0; i < 256; ++i) {
      cudaEvent_t e;
      check(cudaEventCreate(&e), "cudaEventCreate");
      c.ev.push_back(e);
    }
  }
  *e0 = c.ev[c.ev_used];
  *e1 = c.ev[c.ev_used + 1];
  c.ev_used += 2;
}

vxg::DecodeArgs decode_args(Kv& kv, uint32_t n_batch, uint32_t n_head, const int32_t* seq_ids,
                            const int32_t* kv_begin, const int32_t* kv_end, int end_add,
                            const float* q, float scale, uint32_t max_ctx, uint32_t* status) {
  vxg::DecodeArgs a{};
  a.seq_ids = seq_ids;
  a.kv_begin = kv_begin;
  a.kv_end = kv_end;
  a.end_add = end_add;
  a.q = q;
  a.k_pool = kv.k;
  a.v_pool = kv.v;
  a.n_batch = (int)n_batch;
  a.n_seq = (int)kv.n_seq;
  a.cap = (int)kv.cap;
  a.n_head = (int)n_head;
  a.n_kv = (int)kv.n_kv;
  a.nb = (int)(kv.hd / 32);
  a.max_ctx = (int)((max_ctx == 0 || max_ctx > kv.cap) ? kv.cap : max_ctx);
  a.scale = scale;
  a.status = status;
  a.kv_f32 = kv.f32 ? 1 : 0;
  return a;
}

// The split-KV scratch of the context; a new allocation starts with zeroed split-pass state
// (cleared on the stream the call's kernels use).
vxg::Partials carve_partials(Ctx& c, const vxg::DecodeArgs& a, cudaStream_t st) {
  const size_t floats = vxg::decode_partial_floats(a, c.sm_count);
  const size_t had = c.part.n;
  c.part.reserve(floats * sizeof(float), "cudaMalloc partials");
  if (c.part.n != had)
    check(cudaMemsetAsync(c.part.p, 0, sizeof(vxg::FastState), st), "partials state reset");
  return vxg::carve_partials(static_cast<float*>(c.part.p), a, c.sm_count);
}

void check_decode_shape(const Kv& kv, uint32_t n_batch, uint32_t n_head) {
  require(n_head > 0 && n_head % kv.n_kv == 0, VXG_ATTN_ERR_INVALID_OPTION,
          "n_head must be a positive multiple of n_head_kv");
  require(n_batch <= (1u << 20), VXG_ATTN_ERR_INVALID_OPTION, "n_batch too large");
}

void check_host_positions(const Kv& kv, uint32_t n_batch, const int32_t* seq_ids,
                          const int32_t* pos, uint32_t n_tok) {
  for (uint32_t b = 0; b < n_batch; ++b) {
    if (seq_ids[b] < 0 || (uint32_t)seq_ids[b] >= kv.n_seq)
      throw AbiError(VXG_ATTN_ERR_INVALID_OPTION, "sequence id out of range");
    if (pos[b] < 0 || (uint64_t)pos[b] + n_tok > kv.cap)
      throw AbiError(VXG_ATTN_ERR_BUFFER_TOO_SMALL,
                     "position beyond the KV capacity (grow it with vxg_attn_cuda_kv_reserve)");
  }
}

// Device arrays are read and written with 8- and 16-byte vector accesses and bulk copies, so
// device-memory calls take them 16-byte aligned (cudaMalloc and torch allocations are 256-byte
// aligned; a sub-view stays aligned when it starts at a multiple of 4 floats).  Host-memory
// calls stage through aligned buffers and take any alignment.
void require_aligned16(bool host, std::initializer_list<std::pair<const void*, const char*>> arrays) {
  if (host) return;
  for (const auto& x : arrays)
    if (x.first && (reinterpret_cast<uintptr_t>(x.first) & 15u))
      throw AbiError(VXG_ATTN_ERR_INVALID_OPTION,
                     std::string(x.second) + " must be 16-byte aligned in device memory");
}

}  // namespace

// =============================================================================================
extern "C" {

const char* vxg_attn_cuda_version(void) { return kVersion; }

void* vxg_attn_cuda_create(char* err, size_t cap) {
  Ctx* c = nullptr;
  try {
    c = new Ctx();
    if (const char* env = std::getenv("VXG_CUDA_DEVICE")) c->device = std::atoi(env);
    else check(cudaGetDevice(&c->device), "cudaGetDevice");
    check(cudaSetDevice(c->device), "cudaSetDevice");
    cudaDeviceProp prop{};
    check(cudaGetDeviceProperties(&prop, c->device), "cudaGetDeviceProperties");
    if (prop.major < 10)
      throw AbiError(VXG_ATTN_ERR_UNSUPPORTED, std::string("device ") + prop.name +
                                                   " is not sm_100 class; this library is built "
                                                   "for sm_100a only");
    c->sm_count = prop.multiProcessorCount;
    check(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaMalloc(&c->d_status, sizeof(uint32_t)), "cudaMalloc status");
    check(cudaMemset(c->d_status, 0, sizeof(uint32_t)), "cudaMemset status");
    check(cudaMallocHost(&c->h_status, sizeof(uint32_t)), "cudaMallocHost status");
    set_msg(err, cap, prop.name);
    return c;
  } catch (const std::exception& e) {
    set_msg(err, cap, e.what());
    if (c) vxg_attn_cuda_destroy(c);
    return nullptr;
  }
}

void vxg_attn_cuda_destroy(void* h) {
  if (!h) return;
  Ctx* c = static_cast<Ctx*>(h);
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (Kv* kv : c->pools) kv->ctx = nullptr;  // pools outlive the context as plain memory
  c->pools.clear();
  for (auto e : c->ev) cudaEventDestroy(e);
  c->part.release();
  c->io.release();
  c->aux.release();
  c->aux2.release();
  c->pre.release();
  if (c->up_stream) cudaStreamSynchronize(c->up_stream);
  if (c->down_stream) cudaStreamSynchronize(c->down_stream);
  for (auto& sl : c->slot) {
    sl.buf.release();
    if (sl.h_status) cudaFreeHost(sl.h_status);
    for (cudaEvent_t e : {sl.up, sl.done, sl.down})
      if (e) cudaEventDestroy(e);
  }
  if (c->up_stream) cudaStreamDestroy(c->up_stream);
  if (c->down_stream) cudaStreamDestroy(c->down_stream);
  if (c->d_status) cudaFree(c->d_status);
  if (c->h_status) cudaFreeHost(c->h_status);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

int vxg_attn_cuda_sync(void* ctx, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    return collect_status(c, pick_stream(c, stream));
  });
}

int vxg_attn_cuda_sm_count(void* ctx) { return ctx ? static_cast<Ctx*>(ctx)->sm_count : 0; }

int vxg_attn_cuda_set_timing(void* ctx, int enable) {
  if (!ctx) return VXG_ATTN_ERR_NULL_PTR;
  Ctx* c = static_cast<Ctx*>(ctx);
  c->timing = enable != 0;
  c->ev_used = 0;
  return VXG_ATTN_OK;
}

// Sum of the device time of the split passes timed since the last vxg_attn_cuda_set_timing
// call (waits for the last one); -1 if none.
double vxg_attn_cuda_last_split_ms(void* ctx) {
  if (!ctx) return -1.0;
  Ctx* c = static_cast<Ctx*>(ctx);
  if (c->ev_used < 2) return -1.0;
  cudaSetDevice(c->device);
  if (cudaEventSynchronize(c->ev[c->ev_used - 1]) != cudaSuccess) return -1.0;
  double total = 0.0;
  for (size_t i = 0; i + 1 < c->ev_used; i += 2) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, c->ev[i], c->ev[i + 1]) != cudaSuccess) return -1.0;
    total += ms;
  }
  return total;
}

int vxg_attn_cuda_force_generic(void* ctx, int enable) {
  if (!ctx) return VXG_ATTN_ERR_NULL_PTR;
  static_cast<Ctx*>(ctx)->force_generic = enable != 0;
  return VXG_ATTN_OK;
}

void* vxg_attn_cuda_malloc(void* ctx, size_t bytes, char* err, size_t cap) {
  void* p = nullptr;
  int rc = guarded(ctx, nullptr, err, cap, [&] {
    use_ctx(ctx);
    check(cudaMalloc(&p, bytes ? bytes : 1), "cudaMalloc");
    return VXG_ATTN_OK;
  });
  return rc == VXG_ATTN_OK ? p : nullptr;
}

void vxg_attn_cuda_free(void* ctx, void* dptr) {
  if (!ctx || !dptr) return;
  cudaSetDevice(static_cast<Ctx*>(ctx)->device);
  cudaFree(dptr);
}

void* vxg_attn_cuda_host_alloc(void* ctx, size_t bytes, char* err, size_t cap) {
  void* p = nullptr;
  int rc = guarded(ctx, nullptr, err, cap, [&] {
    use_ctx(ctx);
    check(cudaMallocHost(&p, bytes ? bytes : 1), "cudaMallocHost");
    return VXG_ATTN_OK;
  });
  return rc == VXG_ATTN_OK ? p : nullptr;
}

void vxg_attn_cuda_host_free(void* ctx, void* hptr) {
  if (!ctx || !hptr) return;
  cudaSetDevice(static_cast<Ctx*>(ctx)->device);
  cudaFreeHost(hptr);
}

int vxg_attn_cuda_memcpy(void* ctx, void* dst, const void* src, size_t bytes, int kind, char* err,
                         size_t cap) {
  return guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    require(dst && src, VXG_ATTN_ERR_NULL_PTR, "null pointer");
    require(kind >= 0 && kind <= 2, VXG_ATTN_ERR_INVALID_OPTION, "bad copy kind");
    const cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice
                             : kind == 1 ? cudaMemcpyDeviceToHost
                                         : cudaMemcpyDeviceToDevice;
    check(cudaMemcpyAsync(dst, src, bytes, k, c.stream), "cudaMemcpyAsync");
    check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    return VXG_ATTN_OK;
  });
}

// ---------------------------------------------------------------- KV pool ----------------------
static void* kv_create(void* ctx, uint32_t n_seq, uint32_t n_head_kv, uint32_t head_dim,
                       uint32_t cap_tokens, bool f32, char* err, size_t cap) {
  Kv* kv = nullptr;
  int rc = guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    require(n_seq > 0 && n_head_kv > 0 && cap_tokens > 0, VXG_ATTN_ERR_INVALID_OPTION,
            "n_seq, n_head_kv and cap_tokens must be positive");
    require(head_dim > 0 && head_dim % 32 == 0, VXG_ATTN_ERR_UNSUPPORTED,
            f32 ? "head_dim must be a multiple of 32" : "Q8_0 KV needs head_dim % 32 == 0 (llm.rs:291)");
    require(head_dim <= 256, VXG_ATTN_ERR_UNSUPPORTED, "head_dim above 256 is not supported");
    require((uint64_t)n_seq * cap_tokens < (1ull << 31), VXG_ATTN_ERR_INVALID_OPTION,
            "n_seq * cap_tokens too large");
    kv = new Kv();
    kv->ctx = &c;
    kv->device = c.device;
    c.pools.insert(kv);
    kv->n_seq = n_seq;
    kv->n_kv = n_head_kv;
    kv->hd = head_dim;
    kv->cap = cap_tokens;
    kv->f32 = f32;
    const size_t bytes = (size_t)n_seq * kv->seq_bytes();
    check(cudaMalloc(&kv->k, bytes), "cudaMalloc K pool");
    check(cudaMalloc(&kv->v, bytes), "cudaMalloc V pool");
    check(cudaMemsetAsync(kv->k, 0, bytes, c.stream), "cudaMemset K pool");
    check(cudaMemsetAsync(kv->v, 0, bytes, c.stream), "cudaMemset V pool");
    check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    return VXG_ATTN_OK;
  });
  if (rc != VXG_ATTN_OK) {
    if (kv) vxg_attn_cuda_kv_destroy(kv);
    return nullptr;
  }
  return kv;
}

void* vxg_attn_cuda_kv_create(void* ctx, uint32_t n_seq, uint32_t n_head_kv, uint32_t head_dim,
                              uint32_t cap_tokens, char* err, size_t cap) {
  return kv_create(ctx, n_seq, n_head_kv, head_dim, cap_tokens, false, err, cap);
}

void* vxg_attn_cuda_kv_create_f32(void* ctx, uint32_t n_seq, uint32_t n_head_kv,
                                  uint32_t head_dim, uint32_t cap_tokens, char* err, size_t cap) {
  return kv_create(ctx, n_seq, n_head_kv, head_dim, cap_tokens, true, err, cap);
}

void vxg_attn_cuda_kv_destroy(void* h) {
  if (!h) return;
  Kv* kv = static_cast<Kv*>(h);
  cudaSetDevice(kv->device);
  if (kv->ctx) {
    cudaStreamSynchronize(kv->ctx->stream);
    kv->ctx->pools.erase(kv);
  }
  if (kv->k) cudaFree(kv->k);
  if (kv->v) cudaFree(kv->v);
  delete kv;
}

size_t vxg_attn_cuda_kv_bytes(void* h) {
  if (!h) return 0;
  Kv* kv = static_cast<Kv*>(h);
  return 2 * (size_t)kv->n_seq * kv->seq_bytes();
}

uint32_t vxg_attn_cuda_kv_capacity(void* h) { return h ? static_cast<Kv*>(h)->cap : 0; }

int vxg_attn_cuda_kv_reserve(void* h, uint32_t cap_tokens, char* err, size_t cap) {
  Kv* kv = static_cast<Kv*>(h);
  return guarded(kv ? kv->ctx : nullptr, nullptr, err, cap, [&] {
    require(kv != nullptr, VXG_ATTN_ERR_NULL_PTR, "null KV pool");
    require(kv->ctx != nullptr, VXG_ATTN_ERR_NULL_PTR, "the KV pool's context was destroyed");
    Ctx& c = use_ctx(kv->ctx);
    if (cap_tokens <= kv->cap) return VXG_ATTN_OK;
    // doubling with headroom, as native/metal_cb4_fast.h:174-191
    uint64_t nc = std::max<uint64_t>((uint64_t)kv->cap * 2, (uint64_t)cap_tokens + 256);
    require(nc * kv->n_seq < (1ull << 31), VXG_ATTN_ERR_INVALID_OPTION, "capacity too large");
    const size_t tb = kv->tok_bytes();
    const size_t old_pitch = (size_t)kv->cap * tb, new_pitch = (size_t)nc * tb;
    uint8_t *nk = nullptr, *nv = nullptr;
    check(cudaMalloc(&nk, new_pitch * kv->n_seq), "cudaMalloc K pool");
    cudaError_t e = cudaMalloc(&nv, new_pitch * kv->n_seq);
    if (e != cudaSuccess) {
      cudaFree(nk);
      check(e, "cudaMalloc V pool");
    }
    check(cudaMemsetAsync(nk, 0, new_pitch * kv->n_seq, c.stream), "cudaMemset");
    check(cudaMemsetAsync(nv, 0, new_pitch * kv->n_seq, c.stream), "cudaMemset");
    check(cudaMemcpy2DAsync(nk, new_pitch, kv->k, old_pitch, old_pitch, kv->n_seq,
                            cudaMemcpyDeviceToDevice, c.stream), "copy K pool");
    check(cudaMemcpy2DAsync(nv, new_pitch, kv->v, old_pitch, old_pitch, kv->n_seq,
                            cudaMemcpyDeviceToDevice, c.stream), "copy V pool");
    check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    cudaFree(kv->k);
    cudaFree(kv->v);
    kv->k = nk;
    kv->v = nv;
    kv->cap = (uint32_t)nc;
    return VXG_ATTN_OK;
  });
}

int vxg_attn_cuda_kv_device_ptrs(void* h, void** k_pool, void** v_pool, size_t* seq_stride) {
  if (!h) return VXG_ATTN_ERR_NULL_PTR;
  Kv* kv = static_cast<Kv*>(h);
  if (k_pool) *k_pool = kv->k;
  if (v_pool) *v_pool = kv->v;
  if (seq_stride) *seq_stride = kv->seq_bytes();
  return VXG_ATTN_OK;
}

static int kv_copy(void* ctx, void* h, uint32_t seq, uint32_t tok_begin, uint32_t n_tok,
                   const void* kin, const void* vin, void* kout, void* vout, int memkind,
                   char* err, size_t cap) {
  return guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_kv(c, h);
    require(seq < kv.n_seq, VXG_ATTN_ERR_INVALID_OPTION, "sequence id out of range");
    require((uint64_t)tok_begin + n_tok <= kv.cap, VXG_ATTN_ERR_BUFFER_TOO_SMALL,
            "token range beyond the KV capacity");
    const size_t off = (size_t)seq * kv.seq_bytes() + (size_t)tok_begin * kv.tok_bytes();
    const size_t bytes = (size_t)n_tok * kv.tok_bytes();
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    if (kin || vin) {
      const cudaMemcpyKind k = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
      if (kin) check(cudaMemcpyAsync(kv.k + off, kin, bytes, k, c.stream), "import K");
      if (vin) check(cudaMemcpyAsync(kv.v + off, vin, bytes, k, c.stream), "import V");
    } else {
      const cudaMemcpyKind k = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
      if (kout) check(cudaMemcpyAsync(kout, kv.k + off, bytes, k, c.stream), "export K");
      if (vout) check(cudaMemcpyAsync(vout, kv.v + off, bytes, k, c.stream), "export V");
    }
    check(cudaStreamSynchronize(c.stream), "cudaStreamSynchronize");
    return VXG_ATTN_OK;
  });
}

int vxg_attn_cuda_kv_import(void* ctx, void* kv, uint32_t seq, uint32_t tok_begin, uint32_t n_tok,
                            const void* k_blocks, const void* v_blocks, int memkind, char* err,
                            size_t cap) {
  if (!k_blocks && !v_blocks) {
    set_msg(err, cap, "null block pointers");
    return VXG_ATTN_ERR_NULL_PTR;
  }
  return kv_copy(ctx, kv, seq, tok_begin, n_tok, k_blocks, v_blocks, nullptr, nullptr, memkind,
                 err, cap);
}

int vxg_attn_cuda_kv_export(void* ctx, void* kv, uint32_t seq, uint32_t tok_begin, uint32_t n_tok,
                            void* k_blocks, void* v_blocks, int memkind, char* err, size_t cap) {
  if (!k_blocks && !v_blocks) {
    set_msg(err, cap, "null block pointers");
    return VXG_ATTN_ERR_NULL_PTR;
  }
  return kv_copy(ctx, kv, seq, tok_begin, n_tok, nullptr, nullptr, k_blocks, v_blocks, memkind,
                 err, cap);
}

// ---------------------------------------------------------------- ops --------------------------
int vxg_attn_cuda_state_checkpoint(void* ctx, uint32_t n_buffers, void* const* states,
                                   void* const* backups, const size_t* bytes, uint32_t restore,
                                   void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (n_buffers == 0) return VXG_ATTN_OK;
    require(states && backups && bytes, VXG_ATTN_ERR_NULL_PTR, "null buffer list");
    cudaStream_t st = pick_stream(c, stream);
    for (uint32_t i = 0; i < n_buffers; ++i) {
      if (bytes[i] == 0) continue;
      require(states[i] && backups[i], VXG_ATTN_ERR_NULL_PTR, "null state or backup buffer");
      check(cudaMemcpyAsync(restore ? states[i] : backups[i], restore ? backups[i] : states[i],
                            bytes[i], cudaMemcpyDeviceToDevice, st),
            "checkpoint copy");
    }
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_q8_append(void* ctx, void* h, uint32_t n_batch, uint32_t n_tok,
                            const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                            const float* v_new, int memkind, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_q8(c, h);
    if (n_batch == 0 || n_tok == 0) return VXG_ATTN_OK;
    require(seq_ids && pos && k_new && v_new, VXG_ATTN_ERR_NULL_PTR, "null input");
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{k_new, "k_new"}, {v_new, "v_new"}});
    if (host) check_host_positions(kv, n_batch, seq_ids, pos, n_tok);
    cudaStream_t st = pick_stream(c, stream);
    const size_t kvd = (size_t)n_batch * n_tok * kv.n_kv * kv.hd * sizeof(float);
    Stager sg(c, st, host);
    sg.in(seq_ids, n_batch * sizeof(int32_t));
    sg.in(pos, n_batch * sizeof(int32_t));
    sg.in(k_new, kvd);
    sg.in(v_new, kvd);
    sg.upload();
    check(vxg::launch_q8_append(seq_ids, pos, k_new, v_new, kv.k, kv.v, (int)n_batch, (int)n_tok,
                                (int)kv.n_seq, (int)kv.cap, (int)kv.n_kv, (int)(kv.hd / 32),
                                c.d_status, st),
          "q8_append launch");
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_q8_decode(void* ctx, void* h, uint32_t n_batch, uint32_t n_head,
                            const int32_t* seq_ids, const int32_t* pos, const float* q,
                            const float* k_new, const float* v_new, const float* q_gate,
                            float scale, uint32_t max_ctx, float* out, int memkind, void* stream,
                            char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_q8(c, h);
    if (n_batch == 0) return VXG_ATTN_OK;
    require(seq_ids && pos && q && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require((k_new == nullptr) == (v_new == nullptr), VXG_ATTN_ERR_NULL_PTR,
            "k_new and v_new must both be given or both be NULL");
    check_decode_shape(kv, n_batch, n_head);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{q, "q"}, {k_new, "k_new"}, {v_new, "v_new"}, {q_gate, "q_gate"},
                             {out, "out"}});
    if (host) check_host_positions(kv, n_batch, seq_ids, pos, 1);
    cudaStream_t st = pick_stream(c, stream);
    const size_t qb = (size_t)n_batch * n_head * kv.hd * sizeof(float);
    const size_t kvd = (size_t)n_batch * kv.n_kv * kv.hd * sizeof(float);
    Stager sg(c, st, host);
    sg.in(seq_ids, n_batch * sizeof(int32_t));
    sg.in(pos, n_batch * sizeof(int32_t));
    sg.in(q, qb);
    sg.in(k_new, kvd);
    sg.in(v_new, kvd);
    sg.in(q_gate, qb);
    sg.out(out, qb);
    sg.upload();
    if (k_new)
      check(vxg::launch_q8_append(seq_ids, pos, k_new, v_new, kv.k, kv.v, (int)n_batch, 1,
                                  (int)kv.n_seq, (int)kv.cap, (int)kv.n_kv, (int)(kv.hd / 32),
                                  c.d_status, st),
            "q8_append launch");
    vxg::DecodeArgs a = decode_args(kv, n_batch, n_head, seq_ids, nullptr, pos, 1, q, scale,
                                    max_ctx, c.d_status);
    vxg::Partials p = carve_partials(c, a, st);
    cudaEvent_t e0, e1;
    record_timing(c, &e0, &e1);
    check(vxg::launch_decode(a, p, q_gate, out, c.sm_count, c.force_generic, st, e0, e1),
          "decode launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_q8_decode_host_async(void* ctx, void* h, uint32_t n_batch, uint32_t n_head,
                                       const int32_t* seq_ids, const int32_t* pos,
                                       const float* q, const float* k_new, const float* v_new,
                                       const float* q_gate, float scale, uint32_t max_ctx,
                                       float* out, uint64_t* ticket, char* err, size_t cap) {
  return guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_q8(c, h);
    require(ticket != nullptr, VXG_ATTN_ERR_NULL_PTR, "null ticket");
    *ticket = 0;
    if (n_batch == 0) return VXG_ATTN_OK;
    require(seq_ids && pos && q && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require((k_new == nullptr) == (v_new == nullptr), VXG_ATTN_ERR_NULL_PTR,
            "k_new and v_new must both be given or both be NULL");
    check_decode_shape(kv, n_batch, n_head);
    check_host_positions(kv, n_batch, seq_ids, pos, 1);
    ensure_overlap(c);
    const uint64_t t = c.next_ticket++;
    Ctx::Slot& sl = c.slot[t & 1];
    collect_slot(c, sl);  // the step two back is done with this slot's buffers
    const size_t ib = (size_t)n_batch * sizeof(int32_t);
    const size_t qb = (size_t)n_batch * n_head * kv.hd * sizeof(float);
    const size_t kvd = (size_t)n_batch * kv.n_kv * kv.hd * sizeof(float);
    Carver cv;
    const size_t o_seq = cv.take(ib), o_pos = cv.take(ib), o_q = cv.take(qb);
    const size_t o_k = k_new ? cv.take(kvd) : 0, o_v = v_new ? cv.take(kvd) : 0;
    const size_t o_g = q_gate ? cv.take(qb) : 0, o_out = cv.take(qb);
    const size_t o_st = cv.take(sizeof(uint32_t));
    sl.buf.reserve(cv.off, "cudaMalloc overlapped staging");
    uint8_t* base = static_cast<uint8_t*>(sl.buf.p);
    auto up = [&](size_t off, const void* src, size_t bytes) -> const void* {
      if (!src) return nullptr;
      check(cudaMemcpyAsync(base + off, src, bytes, cudaMemcpyHostToDevice, c.up_stream),
            "upload");
      return base + off;
    };
    const int32_t* dseq = static_cast<const int32_t*>(up(o_seq, seq_ids, ib));
    const int32_t* dpos = static_cast<const int32_t*>(up(o_pos, pos, ib));
    const float* dq = static_cast<const float*>(up(o_q, q, qb));
    const float* dk = static_cast<const float*>(up(o_k, k_new, kvd));
    const float* dv = static_cast<const float*>(up(o_v, v_new, kvd));
    const float* dg = static_cast<const float*>(up(o_g, q_gate, qb));
    float* dout = reinterpret_cast<float*>(base + o_out);
    uint32_t* dst = reinterpret_cast<uint32_t*>(base + o_st);
    check(cudaEventRecord(sl.up, c.up_stream), "cudaEventRecord");
    check(cudaStreamWaitEvent(c.stream, sl.up, 0), "cudaStreamWaitEvent");
    check(cudaMemsetAsync(dst, 0, sizeof(uint32_t), c.stream), "status reset");
    if (dk)
      check(vxg::launch_q8_append(dseq, dpos, dk, dv, kv.k, kv.v, (int)n_batch, 1, (int)kv.n_seq,
                                  (int)kv.cap, (int)kv.n_kv, (int)(kv.hd / 32), dst, c.stream),
            "q8_append launch");
    vxg::DecodeArgs a = decode_args(kv, n_batch, n_head, dseq, nullptr, dpos, 1, dq, scale,
                                    max_ctx, dst);
    vxg::Partials p = carve_partials(c, a, c.stream);
    cudaEvent_t e0, e1;
    record_timing(c, &e0, &e1);
    check(vxg::launch_decode(a, p, dg, dout, c.sm_count, c.force_generic, c.stream, e0, e1),
          "decode launch");
    check(cudaEventRecord(sl.done, c.stream), "cudaEventRecord");
    check(cudaStreamWaitEvent(c.down_stream, sl.done, 0), "cudaStreamWaitEvent");
    check(cudaMemcpyAsync(out, dout, qb, cudaMemcpyDeviceToHost, c.down_stream), "download");
    check(cudaMemcpyAsync(sl.h_status, dst, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                          c.down_stream),
          "status download");
    check(cudaEventRecord(sl.down, c.down_stream), "cudaEventRecord");
    sl.ticket = t;
    sl.open = true;
    *ticket = t;
    return VXG_ATTN_OK;
  });
}

int vxg_attn_cuda_ticket_wait(void* ctx, uint64_t ticket, char* err, size_t cap) {
  return guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (ticket == 0) return VXG_ATTN_OK;
    require(ticket < c.next_ticket, VXG_ATTN_ERR_INVALID_OPTION, "unknown ticket");
    for (auto& sl : c.slot)
      if (sl.open && sl.ticket == ticket) collect_slot(c, sl);
    auto it = c.outcomes.find(ticket);
    if (it == c.outcomes.end()) return VXG_ATTN_OK;  // waited for before
    const Ctx::Outcome o = it->second;
    c.outcomes.erase(it);
    if (o.code < 0) throw AbiError(o.code, o.msg);
    return o.code;
  });
}

int vxg_attn_cuda_q8_prefill(void* ctx, void* h, uint32_t n_batch, uint32_t n_tok,
                             uint32_t n_head, const int32_t* seq_ids, const int32_t* pos,
                             const void* q, const void* k_new, const void* v_new,
                             const void* q_gate, int dtype, float scale, uint32_t max_ctx,
                             float* out, int memkind, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_q8(c, h);
    if (n_batch == 0 || n_tok == 0) return VXG_ATTN_OK;
    require(seq_ids && pos && q && k_new && v_new && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require(dtype == VXG_ATTN_DTYPE_F32 || dtype == VXG_ATTN_DTYPE_BF16,
            VXG_ATTN_ERR_INVALID_OPTION, "dtype must be VXG_ATTN_DTYPE_F32 or _BF16");
    check_decode_shape(kv, n_batch, n_head);
    require(vxg::prefill_supported((int)n_head, (int)kv.n_kv, (int)kv.hd),
            VXG_ATTN_ERR_UNSUPPORTED,
            "prefill needs head_dim 64/128/256 and n_head/n_head_kv dividing 128");
    require((uint64_t)n_tok * (n_head / kv.n_kv) <= 65535ull * 128, VXG_ATTN_ERR_INVALID_OPTION,
            "n_tok too large for one prefill call");
    require(n_tok <= kv.cap, VXG_ATTN_ERR_BUFFER_TOO_SMALL, "n_tok beyond the KV capacity");
    const uint32_t lmax = (max_ctx == 0 || max_ctx > kv.cap) ? kv.cap : max_ctx;
    require(n_tok <= lmax, VXG_ATTN_ERR_INVALID_OPTION, "max_ctx below n_tok");
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{q, "q"}, {k_new, "k_new"}, {v_new, "v_new"}, {q_gate, "q_gate"},
                             {out, "out"}});
    if (host) {
      check_host_positions(kv, n_batch, seq_ids, pos, n_tok);
      for (uint32_t b = 0; b < n_batch; ++b)
        require((uint64_t)pos[b] + n_tok <= lmax, VXG_ATTN_ERR_INVALID_OPTION,
                "pos + n_tok beyond max_ctx");
    }
    cudaStream_t st = pick_stream(c, stream);
    const size_t es = dtype == VXG_ATTN_DTYPE_BF16 ? 2 : 4;
    const size_t bt = (size_t)n_batch * n_tok;
    const size_t qb = bt * n_head * kv.hd * es;
    const size_t kvd = bt * kv.n_kv * kv.hd * es;
    Stager sg(c, st, host);
    sg.in(seq_ids, n_batch * sizeof(int32_t));
    sg.in(pos, n_batch * sizeof(int32_t));
    sg.in(q, qb);
    sg.in(k_new, kvd);
    sg.in(v_new, kvd);
    sg.in(q_gate, qb);
    sg.out(out, bt * n_head * kv.hd * sizeof(float));
    sg.upload();
    vxg::PrefillArgs a{};
    a.seq_ids = seq_ids;
    a.pos_base = pos;
    a.q = q;
    a.k_new = k_new;
    a.v_new = v_new;
    a.gate = q_gate;
    a.k_pool = kv.k;
    a.v_pool = kv.v;
    a.out = out;
    a.n_batch = (int)n_batch;
    a.n_tok = (int)n_tok;
    a.n_seq = (int)kv.n_seq;
    a.cap = (int)kv.cap;
    a.n_head = (int)n_head;
    a.n_kv = (int)kv.n_kv;
    a.hd = (int)kv.hd;
    a.lmax = (int)lmax;
    a.scale = scale;
    a.status = c.d_status;
    const int bf16 = dtype == VXG_ATTN_DTYPE_BF16;
    const int allow_tc = !c.force_generic;
    if (!(allow_tc && vxg::prefill_tc_supported((int)n_head, (int)kv.n_kv, (int)kv.hd, bf16)))
      c.pre.reserve(vxg::prefill_scratch_bytes(a), "cudaMalloc prefill scratch");
    cudaEvent_t e0, e1;
    record_timing(c, &e0, &e1);
    check(vxg::launch_prefill(a, c.pre.p, bf16, allow_tc, st, e0, e1), "prefill launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_f32_append(void* ctx, void* h, uint32_t n_batch, uint32_t n_tok,
                             const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                             const float* v_new, int memkind, void* stream, char* err,
                             size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_f32(c, h);
    if (n_batch == 0 || n_tok == 0) return VXG_ATTN_OK;
    require(seq_ids && pos && k_new && v_new, VXG_ATTN_ERR_NULL_PTR, "null input");
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{k_new, "k_new"}, {v_new, "v_new"}});
    if (host) check_host_positions(kv, n_batch, seq_ids, pos, n_tok);
    cudaStream_t st = pick_stream(c, stream);
    const size_t kvd = (size_t)n_batch * n_tok * kv.n_kv * kv.hd * sizeof(float);
    Stager sg(c, st, host);
    sg.in(seq_ids, n_batch * sizeof(int32_t));
    sg.in(pos, n_batch * sizeof(int32_t));
    sg.in(k_new, kvd);
    sg.in(v_new, kvd);
    sg.upload();
    check(vxg::launch_f32_append(seq_ids, pos, k_new, v_new, reinterpret_cast<float*>(kv.k),
                                 reinterpret_cast<float*>(kv.v), (int)n_batch, (int)n_tok,
                                 (int)kv.n_seq, (int)kv.cap, (int)kv.n_kv, (int)kv.hd,
                                 c.d_status, st),
          "f32 append launch");
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_f32_decode(void* ctx, void* h, uint32_t n_batch, uint32_t n_head,
                             const int32_t* seq_ids, const int32_t* pos, const float* q,
                             const float* k_new, const float* v_new, const float* q_gate,
                             float scale, uint32_t max_ctx, float* out, int memkind, void* stream,
                             char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_f32(c, h);
    if (n_batch == 0) return VXG_ATTN_OK;
    require(seq_ids && pos && q && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require((k_new == nullptr) == (v_new == nullptr), VXG_ATTN_ERR_NULL_PTR,
            "k_new and v_new must both be given or both be NULL");
    check_decode_shape(kv, n_batch, n_head);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{q, "q"}, {k_new, "k_new"}, {v_new, "v_new"}, {q_gate, "q_gate"},
                             {out, "out"}});
    if (host) check_host_positions(kv, n_batch, seq_ids, pos, 1);
    cudaStream_t st = pick_stream(c, stream);
    const size_t qb = (size_t)n_batch * n_head * kv.hd * sizeof(float);
    const size_t kvd = (size_t)n_batch * kv.n_kv * kv.hd * sizeof(float);
    Stager sg(c, st, host);
    sg.in(seq_ids, n_batch * sizeof(int32_t));
    sg.in(pos, n_batch * sizeof(int32_t));
    sg.in(q, qb);
    sg.in(k_new, kvd);
    sg.in(v_new, kvd);
    sg.in(q_gate, qb);
    sg.out(out, qb);
    sg.upload();
    if (k_new)
      check(vxg::launch_f32_append(seq_ids, pos, k_new, v_new, reinterpret_cast<float*>(kv.k),
                                   reinterpret_cast<float*>(kv.v), (int)n_batch, 1,
                                   (int)kv.n_seq, (int)kv.cap, (int)kv.n_kv, (int)kv.hd,
                                   c.d_status, st),
            "f32 append launch");
    vxg::DecodeArgs a = decode_args(kv, n_batch, n_head, seq_ids, nullptr, pos, 1, q, scale,
                                    max_ctx, c.d_status);
    vxg::Partials p = carve_partials(c, a, st);
    cudaEvent_t e0, e1;
    record_timing(c, &e0, &e1);
    check(vxg::launch_decode(a, p, q_gate, out, c.sm_count, 1, st, e0, e1), "decode launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_q8_decode_partial(void* ctx, void* h, uint32_t n_batch, uint32_t n_head,
                                    const int32_t* seq_ids, const int32_t* kv_begin,
                                    const int32_t* kv_end, const float* q, float scale,
                                    uint32_t max_ctx, float* m, float* l, float* o, int memkind,
                                    void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_q8(c, h);
    if (n_batch == 0) return VXG_ATTN_OK;
    require(seq_ids && kv_begin && kv_end && q && m && l && o, VXG_ATTN_ERR_NULL_PTR,
            "null input");
    check_decode_shape(kv, n_batch, n_head);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{q, "q"}, {m, "m"}, {l, "l"}, {o, "o"}});
    if (host)
      for (uint32_t b = 0; b < n_batch; ++b)
        require(seq_ids[b] >= 0 && (uint32_t)seq_ids[b] < kv.n_seq && kv_begin[b] >= 0 &&
                    kv_begin[b] <= kv_end[b] && (uint32_t)kv_end[b] <= kv.cap,
                VXG_ATTN_ERR_INVALID_OPTION, "sequence id or token range out of range");
    cudaStream_t st = pick_stream(c, stream);
    const size_t rows = (size_t)n_batch * n_head;
    Stager sg(c, st, host);
    sg.in(seq_ids, n_batch * sizeof(int32_t));
    sg.in(kv_begin, n_batch * sizeof(int32_t));
    sg.in(kv_end, n_batch * sizeof(int32_t));
    sg.in(q, rows * kv.hd * sizeof(float));
    sg.out(m, rows * sizeof(float));
    sg.out(l, rows * sizeof(float));
    sg.out(o, rows * kv.hd * sizeof(float));
    sg.upload();
    vxg::DecodeArgs a = decode_args(kv, n_batch, n_head, seq_ids, kv_begin, kv_end, 0, q, scale,
                                    max_ctx, c.d_status);
    vxg::Partials p = carve_partials(c, a, st);
    cudaEvent_t e0, e1;
    record_timing(c, &e0, &e1);
    check(vxg::launch_decode_partial(a, p, m, l, o, c.sm_count, c.force_generic, st, e0, e1),
          "decode partial launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_lse_combine(void* ctx, uint32_t n_parts, uint32_t n_rows, uint32_t head_dim,
                              const float* m, const float* l, const float* o, const float* gate,
                              float* out, int memkind, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (n_rows == 0) return VXG_ATTN_OK;
    require(m && l && o && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_parts > 0 && head_dim > 0, VXG_ATTN_ERR_INVALID_OPTION, "empty combine");
    cudaStream_t st = pick_stream(c, stream);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{m, "m"}, {l, "l"}, {o, "o"}, {gate, "gate"}, {out, "out"}});
    const size_t pr = (size_t)n_parts * n_rows;
    Stager sg(c, st, host);
    sg.in(m, pr * sizeof(float));
    sg.in(l, pr * sizeof(float));
    sg.in(o, pr * head_dim * sizeof(float));
    sg.in(gate, (size_t)n_rows * head_dim * sizeof(float));
    sg.out(out, (size_t)n_rows * head_dim * sizeof(float));
    sg.upload();
    check(vxg::launch_lse_combine((int)n_parts, (int)n_rows, (int)head_dim, m, l, o, gate, out,
                                  c.d_status, st),
          "lse combine launch");
    sg.download();
    return finish(c, stream, st);
  });
}

size_t vxg_attn_cuda_peer_buffer_bytes(uint32_t world, uint32_t n_rows, uint32_t head_dim) {
  return vxg::peer_buffer_bytes((int)world, (int)(n_rows * (head_dim + 2)));
}

void* vxg_attn_cuda_peer_alloc(void* ctx, uint32_t world, uint32_t n_rows, uint32_t head_dim,
                               void* ipc_handle, char* err, size_t cap) {
  void* p = nullptr;
  int rc = guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    require(ipc_handle != nullptr, VXG_ATTN_ERR_NULL_PTR, "null ipc_handle");
    require(world >= 1 && world <= 8 && n_rows > 0 && head_dim > 0, VXG_ATTN_ERR_INVALID_OPTION,
            "need 1 <= world <= 8 and a non-empty partial");
    const size_t bytes = vxg_attn_cuda_peer_buffer_bytes(world, n_rows, head_dim);
    check(cudaMalloc(&p, bytes), "cudaMalloc peer buffer");
    check(cudaMemset(p, 0, bytes), "cudaMemset peer buffer");
    cudaIpcMemHandle_t h;
    check(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
    std::memcpy(ipc_handle, &h, sizeof(h));
    (void)c;
    return VXG_ATTN_OK;
  });
  if (rc != VXG_ATTN_OK && p) {
    cudaFree(p);
    p = nullptr;
  }
  return p;
}

void* vxg_attn_cuda_peer_open(void* ctx, const void* ipc_handle, char* err, size_t cap) {
  void* p = nullptr;
  int rc = guarded(ctx, nullptr, err, cap, [&] {
    use_ctx(ctx);
    require(ipc_handle != nullptr, VXG_ATTN_ERR_NULL_PTR, "null ipc_handle");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    return VXG_ATTN_OK;
  });
  return rc == VXG_ATTN_OK ? p : nullptr;
}

void vxg_attn_cuda_peer_close(void* ctx, void* mapped) {
  if (!ctx || !mapped) return;
  cudaSetDevice(static_cast<Ctx*>(ctx)->device);
  cudaIpcCloseMemHandle(mapped);
}

void vxg_attn_cuda_peer_free(void* ctx, void* buf) { vxg_attn_cuda_free(ctx, buf); }

int vxg_attn_cuda_peer_step(void* ctx, void* const* bufs, uint32_t world, uint32_t rank,
                            uint32_t n_rows, uint32_t head_dim, const float* send,
                            const float* gate, float* out, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    require(bufs && send && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require(world >= 1 && world <= 8 && rank < world, VXG_ATTN_ERR_INVALID_OPTION,
            "need 1 <= world <= 8 and rank < world");
    require(n_rows > 0 && head_dim > 0, VXG_ATTN_ERR_INVALID_OPTION, "empty partial");
    vxg::PeerTable t{};
    for (uint32_t r = 0; r < world; ++r) {
      require(bufs[r] != nullptr, VXG_ATTN_ERR_NULL_PTR, "null peer buffer");
      t.buf[r] = static_cast<float*>(bufs[r]);
    }
    require_aligned16(false, {{send, "send"}, {gate, "gate"}, {out, "out"}, {bufs[rank], "buffer"}});
    cudaStream_t st = pick_stream(c, stream);
    const int per = (int)(n_rows * (head_dim + 2));
    check(vxg::launch_peer_push(send, per, t, (int)world, (int)rank, t.buf[rank], st),
          "peer push launch");
    check(vxg::launch_peer_combine(t.buf[rank], (int)world, (int)n_rows, (int)head_dim, gate, out,
                                   c.d_status, st),
          "peer combine launch");
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_lse_combine_packed(void* ctx, uint32_t n_parts, uint32_t n_rows,
                                     uint32_t head_dim, const float* packed, const float* gate,
                                     float* out, int memkind, void* stream, char* err,
                                     size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (n_rows == 0) return VXG_ATTN_OK;
    require(packed && out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_parts > 0 && head_dim > 0, VXG_ATTN_ERR_INVALID_OPTION, "empty combine");
    cudaStream_t st = pick_stream(c, stream);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{packed, "packed"}, {gate, "gate"}, {out, "out"}});
    Stager sg(c, st, host);
    sg.in(packed, (size_t)n_parts * n_rows * (head_dim + 2) * sizeof(float));
    sg.in(gate, (size_t)n_rows * head_dim * sizeof(float));
    sg.out(out, (size_t)n_rows * head_dim * sizeof(float));
    sg.upload();
    check(vxg::launch_lse_combine_packed((int)n_parts, (int)n_rows, (int)head_dim, packed, gate,
                                         out, c.d_status, st),
          "lse combine launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_step_full_gqa_q8(void* ctx, void* h, uint32_t seq, const float* q_raw,
                                   float* k_cur, const float* v_cur, const float* q_norm,
                                   const float* k_norm, int gated_q, uint32_t n_head,
                                   uint32_t n_head_kv, uint32_t head_dim, uint32_t pos,
                                   uint32_t rope_pos, uint32_t rope_dim, float rope_freq_base,
                                   int rope_neox, float eps, float* attn_out, char* err,
                                   size_t cap) {
  return guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_q8(c, h);
    require(q_raw && k_cur && v_cur && attn_out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_head_kv == kv.n_kv && head_dim == kv.hd, VXG_ATTN_ERR_INVALID_OPTION,
            "n_head_kv / head_dim differ from the KV pool's");
    check_decode_shape(kv, 1, n_head);
    require(seq < kv.n_seq, VXG_ATTN_ERR_INVALID_OPTION, "sequence id out of range");
    require(pos < kv.cap, VXG_ATTN_ERR_BUFFER_TOO_SMALL,
            "position beyond the KV capacity (grow it with vxg_attn_cuda_kv_reserve)");
    cudaStream_t st = c.stream;
    // RoPE table with the C library, as apply_rope does (llm_ops.rs:81-101)
    const uint32_t rdim = rope_dim < head_dim ? rope_dim : head_dim;
    const uint32_t half = rdim / 2;
    std::vector<float> cs(2 * (size_t)(half ? half : 1));
    for (uint32_t i = 0; i < half; ++i) {
      volatile float e = -(2.0f * (float)i) / (float)rdim;
      const float freq = powf(rope_freq_base, e);
      const float theta = (float)rope_pos * freq;
      cs[2 * i] = cosf(theta);
      cs[2 * i + 1] = sinf(theta);
    }
    const size_t hdb = head_dim * sizeof(float);
    const size_t qraw_b = (size_t)n_head * (gated_q ? 2 : 1) * hdb;
    Carver cv;
    const size_t o_qraw = cv.take(qraw_b), o_k = cv.take(n_head_kv * hdb),
                 o_v = cv.take(n_head_kv * hdb), o_qn = cv.take(hdb), o_kn = cv.take(hdb),
                 o_cs = cv.take(cs.size() * sizeof(float)), o_q = cv.take(n_head * hdb),
                 o_g = cv.take(n_head * hdb), o_out = cv.take(n_head * hdb),
                 o_ids = cv.take(2 * sizeof(int32_t));
    c.aux.reserve(cv.off, "cudaMalloc step buffers");
    uint8_t* base = static_cast<uint8_t*>(c.aux.p);
    auto up = [&](size_t off, const void* src, size_t bytes) {
      check(cudaMemcpyAsync(base + off, src, bytes, cudaMemcpyHostToDevice, st), "upload");
    };
    up(o_qraw, q_raw, qraw_b);
    up(o_k, k_cur, n_head_kv * hdb);
    up(o_v, v_cur, n_head_kv * hdb);
    if (q_norm) up(o_qn, q_norm, hdb);
    if (k_norm) up(o_kn, k_norm, hdb);
    if (half) up(o_cs, cs.data(), cs.size() * sizeof(float));
    const int32_t ids[2] = {(int32_t)seq, (int32_t)pos};
    up(o_ids, ids, sizeof(ids));
    float* dk = reinterpret_cast<float*>(base + o_k);
    float* dq = reinterpret_cast<float*>(base + o_q);
    float* dg = gated_q ? reinterpret_cast<float*>(base + o_g) : nullptr;
    check(vxg::launch_gqa_prep(reinterpret_cast<const float*>(base + o_qraw), dk,
                               q_norm ? reinterpret_cast<const float*>(base + o_qn) : nullptr,
                               k_norm ? reinterpret_cast<const float*>(base + o_kn) : nullptr,
                               gated_q ? 1 : 0, (int)n_head, (int)n_head_kv, (int)head_dim,
                               reinterpret_cast<const float2*>(base + o_cs), (int)half,
                               rope_neox ? 1 : 0, eps, dq, dg, st),
          "prep launch");
    const int32_t* d_seq = reinterpret_cast<const int32_t*>(base + o_ids);
    const int32_t* d_pos = d_seq + 1;
    check(vxg::launch_q8_append(d_seq, d_pos, dk, reinterpret_cast<const float*>(base + o_v), kv.k,
                                kv.v, 1, 1, (int)kv.n_seq, (int)kv.cap, (int)kv.n_kv,
                                (int)(kv.hd / 32), c.d_status, st),
          "q8_append launch");
    const float scale = 1.0f / sqrtf((float)head_dim);
    vxg::DecodeArgs a = decode_args(kv, 1, n_head, d_seq, nullptr, d_pos, 1, dq, scale, pos + 1,
                                    c.d_status);
    vxg::Partials p = carve_partials(c, a, st);
    float* dout = reinterpret_cast<float*>(base + o_out);
    check(vxg::launch_decode(a, p, dg, dout, c.sm_count, c.force_generic, st, nullptr, nullptr),
          "decode launch");
    check(cudaMemcpyAsync(attn_out, dout, n_head * hdb, cudaMemcpyDeviceToHost, st), "download");
    check(cudaMemcpyAsync(k_cur, dk, n_head_kv * hdb, cudaMemcpyDeviceToHost, st), "download k");
    return collect_status(c, st);
  });
}

int vxg_attn_cuda_step_full_gqa(void* ctx, void* h, uint32_t seq, const float* q_raw,
                                float* k_cur, const float* v_cur, const float* q_norm,
                                const float* k_norm, int gated_q, uint32_t n_head,
                                uint32_t n_head_kv, uint32_t head_dim, uint32_t pos,
                                uint32_t rope_dim, float rope_freq_base, int rope_neox, float eps,
                                float* att_cat, char* err, size_t cap) {
  const uint32_t rope_pos = pos;  // step_full_gqa ropes at the cache position (llm_ops.rs:235-251)
  float* attn_out = att_cat;
  return guarded(ctx, nullptr, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    Kv& kv = use_f32(c, h);
    require(q_raw && k_cur && v_cur && attn_out, VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_head_kv == kv.n_kv && head_dim == kv.hd, VXG_ATTN_ERR_INVALID_OPTION,
            "n_head_kv / head_dim differ from the KV pool's");
    check_decode_shape(kv, 1, n_head);
    require(seq < kv.n_seq, VXG_ATTN_ERR_INVALID_OPTION, "sequence id out of range");
    require(pos < kv.cap, VXG_ATTN_ERR_BUFFER_TOO_SMALL,
            "position beyond the KV capacity (grow it with vxg_attn_cuda_kv_reserve)");
    cudaStream_t st = c.stream;
    // RoPE table with the C library, as apply_rope does (llm_ops.rs:81-101)
    const uint32_t rdim = rope_dim < head_dim ? rope_dim : head_dim;
    const uint32_t half = rdim / 2;
    std::vector<float> cs(2 * (size_t)(half ? half : 1));
    for (uint32_t i = 0; i < half; ++i) {
      volatile float e = -(2.0f * (float)i) / (float)rdim;
      const float freq = powf(rope_freq_base, e);
      const float theta = (float)rope_pos * freq;
      cs[2 * i] = cosf(theta);
      cs[2 * i + 1] = sinf(theta);
    }
    const size_t hdb = head_dim * sizeof(float);
    const size_t qraw_b = (size_t)n_head * (gated_q ? 2 : 1) * hdb;
    Carver cv;
    const size_t o_qraw = cv.take(qraw_b), o_k = cv.take(n_head_kv * hdb),
                 o_v = cv.take(n_head_kv * hdb), o_qn = cv.take(hdb), o_kn = cv.take(hdb),
                 o_cs = cv.take(cs.size() * sizeof(float)), o_q = cv.take(n_head * hdb),
                 o_g = cv.take(n_head * hdb), o_out = cv.take(n_head * hdb),
                 o_ids = cv.take(2 * sizeof(int32_t));
    c.aux.reserve(cv.off, "cudaMalloc step buffers");
    uint8_t* base = static_cast<uint8_t*>(c.aux.p);
    auto up = [&](size_t off, const void* src, size_t bytes) {
      check(cudaMemcpyAsync(base + off, src, bytes, cudaMemcpyHostToDevice, st), "upload");
    };
    up(o_qraw, q_raw, qraw_b);
    up(o_k, k_cur, n_head_kv * hdb);
    up(o_v, v_cur, n_head_kv * hdb);
    if (q_norm) up(o_qn, q_norm, hdb);
    if (k_norm) up(o_kn, k_norm, hdb);
    if (half) up(o_cs, cs.data(), cs.size() * sizeof(float));
    const int32_t ids[2] = {(int32_t)seq, (int32_t)pos};
    up(o_ids, ids, sizeof(ids));
    float* dk = reinterpret_cast<float*>(base + o_k);
    float* dq = reinterpret_cast<float*>(base + o_q);
    float* dg = gated_q ? reinterpret_cast<float*>(base + o_g) : nullptr;
    check(vxg::launch_gqa_prep(reinterpret_cast<const float*>(base + o_qraw), dk,
                               q_norm ? reinterpret_cast<const float*>(base + o_qn) : nullptr,
                               k_norm ? reinterpret_cast<const float*>(base + o_kn) : nullptr,
                               gated_q ? 1 : 0, (int)n_head, (int)n_head_kv, (int)head_dim,
                               reinterpret_cast<const float2*>(base + o_cs), (int)half,
                               rope_neox ? 1 : 0, eps, dq, dg, st),
          "prep launch");
    const int32_t* d_seq = reinterpret_cast<const int32_t*>(base + o_ids);
    const int32_t* d_pos = d_seq + 1;
    check(vxg::launch_f32_append(d_seq, d_pos, dk, reinterpret_cast<const float*>(base + o_v),
                                 reinterpret_cast<float*>(kv.k), reinterpret_cast<float*>(kv.v),
                                 1, 1, (int)kv.n_seq, (int)kv.cap, (int)kv.n_kv, (int)kv.hd,
                                 c.d_status, st),
          "f32 append launch");
    const float scale = 1.0f / sqrtf((float)head_dim);
    vxg::DecodeArgs a = decode_args(kv, 1, n_head, d_seq, nullptr, d_pos, 1, dq, scale, pos + 1,
                                    c.d_status);
    vxg::Partials p = carve_partials(c, a, st);
    float* dout = reinterpret_cast<float*>(base + o_out);
    check(vxg::launch_decode(a, p, dg, dout, c.sm_count, 1, st, nullptr, nullptr),
          "decode launch");
    check(cudaMemcpyAsync(attn_out, dout, n_head * hdb, cudaMemcpyDeviceToHost, st), "download");
    check(cudaMemcpyAsync(k_cur, dk, n_head_kv * hdb, cudaMemcpyDeviceToHost, st), "download k");
    return collect_status(c, st);
  });
}

int vxg_attn_cuda_deltanet_step(void* ctx, uint32_t n_batch, uint32_t n_kh, uint32_t n_vh,
                                uint32_t dk, uint32_t dv, const float* q, const float* k,
                                const float* v, const float* beta_raw, const float* alpha_raw,
                                const float* ssm_a, const float* dt_bias, float q_scale, float eps,
                                float* state, float* o, int memkind, void* stream, char* err,
                                size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (n_batch == 0) return VXG_ATTN_OK;
    require(q && k && v && beta_raw && alpha_raw && ssm_a && dt_bias && state && o,
            VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_kh > 0 && n_vh > 0 && n_vh % n_kh == 0, VXG_ATTN_ERR_INVALID_OPTION,
            "n_vh must be a positive multiple of n_kh");
    require(dk == 64 || dk == 128 || dk == 256, VXG_ATTN_ERR_UNSUPPORTED,
            "dk must be 64, 128 or 256");
    require(dv > 0 && dv % 32 == 0, VXG_ATTN_ERR_UNSUPPORTED, "dv must be a multiple of 32");
    cudaStream_t st = pick_stream(c, stream);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{q, "q"}, {k, "k"}, {v, "v"}, {state, "state"}, {o, "o"}});
    Stager sg(c, st, host);
    sg.in(q, (size_t)n_batch * n_kh * dk * sizeof(float));
    sg.in(k, (size_t)n_batch * n_kh * dk * sizeof(float));
    sg.in(v, (size_t)n_batch * n_vh * dv * sizeof(float));
    sg.in(beta_raw, (size_t)n_batch * n_vh * sizeof(float));
    sg.in(alpha_raw, (size_t)n_batch * n_vh * sizeof(float));
    sg.in(ssm_a, n_vh * sizeof(float));
    sg.in(dt_bias, n_vh * sizeof(float));
    sg.inout(state, (size_t)n_batch * n_vh * dv * dk * sizeof(float));
    sg.out(o, (size_t)n_batch * n_vh * dv * sizeof(float));
    sg.upload();
    vxg::DeltaNetArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.beta_raw = beta_raw;
    a.alpha_raw = alpha_raw;
    a.ssm_a = ssm_a;
    a.dt_bias = dt_bias;
    a.state = state;
    a.o = o;
    a.q_bs = a.k_bs = (long long)n_kh * dk;
    a.v_bs = a.o_bs = (long long)n_vh * dv;
    a.g_bs = n_vh;
    a.n_batch = (int)n_batch;
    a.n_tok = 1;
    a.n_kh = (int)n_kh;
    a.n_vh = (int)n_vh;
    a.dk = (int)dk;
    a.dv = (int)dv;
    a.eps = eps;
    a.q_scale = q_scale;
    a.status = c.d_status;
    check(vxg::launch_deltanet_step(a, st), "deltanet launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_deltanet_prefill(void* ctx, uint32_t n_batch, uint32_t n_tok, uint32_t n_kh,
                                   uint32_t n_vh, uint32_t dk, uint32_t dv, const float* q,
                                   const float* k, const float* v, const float* beta_raw,
                                   const float* alpha_raw, const float* ssm_a,
                                   const float* dt_bias, float q_scale, float eps, float* state,
                                   float* o, int memkind, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (n_batch == 0 || n_tok == 0) return VXG_ATTN_OK;
    require(q && k && v && beta_raw && alpha_raw && ssm_a && dt_bias && state && o,
            VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_kh > 0 && n_vh > 0 && n_vh % n_kh == 0, VXG_ATTN_ERR_INVALID_OPTION,
            "n_vh must be a positive multiple of n_kh");
    require(dk == 64 || dk == 128 || dk == 256, VXG_ATTN_ERR_UNSUPPORTED,
            "dk must be 64, 128 or 256");
    require(dv > 0 && dv % 32 == 0, VXG_ATTN_ERR_UNSUPPORTED, "dv must be a multiple of 32");
    cudaStream_t st = pick_stream(c, stream);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{q, "q"}, {k, "k"}, {v, "v"}, {state, "state"}, {o, "o"}});
    const size_t bt = (size_t)n_batch * n_tok;
    Stager sg(c, st, host);
    sg.in(q, bt * n_kh * dk * sizeof(float));
    sg.in(k, bt * n_kh * dk * sizeof(float));
    sg.in(v, bt * n_vh * dv * sizeof(float));
    sg.in(beta_raw, bt * n_vh * sizeof(float));
    sg.in(alpha_raw, bt * n_vh * sizeof(float));
    sg.in(ssm_a, n_vh * sizeof(float));
    sg.in(dt_bias, n_vh * sizeof(float));
    sg.inout(state, (size_t)n_batch * n_vh * dv * dk * sizeof(float));
    sg.out(o, bt * n_vh * dv * sizeof(float));
    sg.upload();
    vxg::DeltaNetArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.beta_raw = beta_raw;
    a.alpha_raw = alpha_raw;
    a.ssm_a = ssm_a;
    a.dt_bias = dt_bias;
    a.state = state;
    a.o = o;
    a.q_ts = a.k_ts = (long long)n_kh * dk;
    a.q_bs = a.k_bs = (long long)n_tok * n_kh * dk;
    a.v_ts = a.o_ts = (long long)n_vh * dv;
    a.v_bs = a.o_bs = (long long)n_tok * n_vh * dv;
    a.g_ts = n_vh;
    a.g_bs = (long long)n_tok * n_vh;
    a.n_batch = (int)n_batch;
    a.n_tok = (int)n_tok;
    a.n_kh = (int)n_kh;
    a.n_vh = (int)n_vh;
    a.dk = (int)dk;
    a.dv = (int)dv;
    a.eps = eps;
    a.q_scale = q_scale;
    a.status = c.d_status;
    c.aux2.reserve(vxg::deltanet_prefill_scratch_bytes(a), "cudaMalloc deltanet scratch");
    check(vxg::launch_deltanet_prefill(a, c.aux2.p, !c.force_generic, st),
          "deltanet prefill launch");
    sg.download();
    return finish(c, stream, st);
  });
}

int vxg_attn_cuda_step_deltanet_recurrent(
    void* ctx, uint32_t n_batch, const float* qkv_mixed, uint32_t conv_ch, const float* z,
    const float* alpha_raw, const float* beta_raw, const float* ssm_conv1d, const float* ssm_a,
    const float* ssm_dt_bias, const float* ssm_norm, float* conv_state, float* ssm_state,
    uint32_t n_kh, uint32_t n_vh, uint32_t dk, uint32_t dv, uint32_t k_sz, float eps,
    float* y_concat, int memkind, void* stream, char* err, size_t cap) {
  return guarded(ctx, stream, err, cap, [&] {
    Ctx& c = use_ctx(ctx);
    if (n_batch == 0) return VXG_ATTN_OK;
    require(qkv_mixed && z && alpha_raw && beta_raw && ssm_conv1d && ssm_a && ssm_dt_bias &&
                ssm_norm && conv_state && ssm_state && y_concat,
            VXG_ATTN_ERR_NULL_PTR, "null input");
    require(n_kh > 0 && n_vh > 0 && n_vh % n_kh == 0, VXG_ATTN_ERR_INVALID_OPTION,
            "n_vh must be a positive multiple of n_kh");
    require(dk == 64 || dk == 128 || dk == 256, VXG_ATTN_ERR_UNSUPPORTED,
            "dk must be 64, 128 or 256");
    require(dv > 0 && dv % 32 == 0 && dv <= 256, VXG_ATTN_ERR_UNSUPPORTED,
            "dv must be a multiple of 32, at most 256");
    require(k_sz >= 2, VXG_ATTN_ERR_INVALID_OPTION, "k_sz must be at least 2");
    require(conv_ch == 2 * n_kh * dk + n_vh * dv, VXG_ATTN_ERR_INVALID_OPTION,
            "conv_ch must equal 2 * n_kh * dk + n_vh * dv (llm_ops.rs:139-143)");
    cudaStream_t st = pick_stream(c, stream);
    const bool host = memkind == VXG_ATTN_MEM_HOST;
    require_aligned16(host, {{qkv_mixed, "qkv_mixed"}, {z, "z"}, {conv_state, "conv_state"},
                             {ssm_state, "ssm_state"}, {y_concat, "y_concat"}});
    if (!host)
      require(((uintptr_t)ssm_state % 16) == 0, VXG_ATTN_ERR_INVALID_OPTION,
              "ssm_state must be 16-byte aligned");
    const size_t ydim = (size_t)n_vh * dv;
    Stager sg(c, st, host);
    sg.in(qkv_mixed, (size_t)n_batch * conv_ch * sizeof(float));
    sg.in(z, n_batch * ydim * sizeof(float));
    sg.in(alpha_raw, (size_t)n_batch * n_vh * sizeof(float));
    sg.in(beta_raw, (size_t)n_batch * n_vh * sizeof(float));
    sg.in(ssm_conv1d, (size_t)conv_ch * k_sz * sizeof(float));
    sg.in(ssm_a, n_vh * sizeof(float));
    sg.in(ssm_dt_bias, n_vh * sizeof(float));
    sg.in(ssm_norm, dv * sizeof(float));
    sg.inout(conv_state, (size_t)n_batch * (k_sz - 1) * conv_ch * sizeof(float));
    sg.inout(ssm_state, (size_t)n_batch * n_vh * dv * dk * sizeof(float));
    sg.out(y_concat, n_batch * ydim * sizeof(float));
    sg.upload();
    c.aux2.reserve((size_t)n_batch * conv_ch * sizeof(float) + 256, "cudaMalloc conv scratch");
    float* conv_out = static_cast<float*>(c.aux2.p);
    check(vxg::launch_deltanet_conv(qkv_mixed, ssm_conv1d, conv_state, conv_out, (int)n_batch,
                                    (int)conv_ch, (int)k_sz, st),
          "conv launch");
    const size_t qk_dim = (size_t)n_kh * dk;
    vxg::DeltaNetArgs a{};
    a.q = conv_out;
    a.k = conv_out + qk_dim;
    a.v = conv_out + 2 * qk_dim;
    a.beta_raw = beta_raw;
    a.alpha_raw = alpha_raw;
    a.ssm_a = ssm_a;
    a.dt_bias = ssm_dt_bias;
    a.state = ssm_state;
    a.o = nullptr;
    a.z = z;
    a.ssm_norm = ssm_norm;
    a.y = y_concat;
    a.q_bs = a.k_bs = a.v_bs = conv_ch;
    a.o_bs = (long long)ydim;
    a.g_bs = n_vh;
    a.n_batch = (int)n_batch;
    a.n_tok = 1;
    a.n_kh = (int)n_kh;
    a.n_vh = (int)n_vh;
    a.dk = (int)dk;
    a.dv = (int)dv;
    a.eps = eps;
    a.q_scale = 1.0f / sqrtf((float)dk);
    a.status = c.d_status;
    check(vxg::launch_deltanet_step(a, st), "deltanet launch");
    sg.download();
    return finish(c, stream, st);
  });
}

}  // extern "C"
