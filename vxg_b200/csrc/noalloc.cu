// Batched Q8 decode attention that allocates no device memory.
//
// Some callers cannot call cudaMalloc: an engine whose device memory is owned by a budgeted
// pool or another framework's caching allocator (allocating behind its back can fail or
// fragment the pool), and decode loops that must not stall, because cudaMalloc may
// synchronise the device.  This entry point serves them.  The caller passes every input and
// output as device memory (including the KV pools); the split-KV partials and the device
// status word live in one file-scope __device__ array of fixed size that every GPU loading
// this library holds until the process exits.
//
// Limits and sharing:
//  * the array is kScratchBytes (32 MiB); a call whose partials do not fit is rejected with
//    VXG_ATTN_ERR_BUFFER_TOO_SMALL before anything is launched.  At 16 query / 2 KV heads,
//    head_dim 256 the partials take ((SMs + n) * 6 * 16 * 258 + n + SMs + 64) floats for n >= 32
//    entries (a little more below 32, where the combine splits slots), so a 148-SM B200 takes up
//    to 190 batch entries per call.  Other shapes run the generic split kernel, whose partials
//    grow with cap_tokens (n * ceil(cap_tokens / 512) * n_head * (head_dim + 2) floats): there
//    the batch limit shrinks as the pools' capacity grows;
//  * every call on a device uses the same array, so calls that overlap on the GPU (different
//    streams, or several host threads) race and must be serialised by the caller;
//  * each call clears the status word it needs; the partials are fully written by a call before
//    that call reads them, so leftovers from the previous call do no harm.
//
// The first call on a device does a one-time set-up with that device current: it looks up the
// array's device address with cudaGetSymbolAddress (host code cannot use the array's name as a
// device address) and the SM count.  Make that first call before any stream capture.  The
// address is cached per device index, which assumes every call on a device runs in that
// device's primary context (the CUDA runtime's default); a caller that makes its own driver-API
// contexts must not call this entry point from more than one context per device.
#include "vxg_attn_cuda.h"
#include "kernels.h"

#include <cstdio>
#include <mutex>
#include <string>

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;
constexpr size_t kStatusBytes = 256;  // the status word, padded to keep the partials aligned
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceScratch {
  unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this device
  int sm_count = 0;
};
DeviceScratch g_dev[kMaxDevices];
std::mutex g_setup_mu;

void put(char* err, size_t cap, const std::string& m) {
  if (err && cap) std::snprintf(err, cap, "%s", m.c_str());
}

// One-time per-device set-up (the current device must be `dev`).
int setup(int dev, DeviceScratch* out, char* err, size_t cap) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_dev[dev].base) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      put(err, cap, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      return VXG_ATTN_ERR_INTERNAL;
    }
    int sm = 0;
    e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      put(err, cap, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
      return VXG_ATTN_ERR_INTERNAL;
    }
    g_dev[dev].sm_count = sm;
    g_dev[dev].base = static_cast<unsigned char*>(p);
  }
  *out = g_dev[dev];
  return VXG_ATTN_OK;
}

}  // namespace

extern "C" int vxg_attn_cuda_q8_decode_noalloc(
    void* k_pool, void* v_pool, uint32_t n_seq, uint32_t cap_tokens,
    uint32_t n_head_kv, uint32_t head_dim, uint32_t n_batch, uint32_t n_head,
    const int32_t* seq_ids, const int32_t* pos, const float* q, const float* k_new,
    const float* v_new, const float* q_gate, float scale, float* out, void* stream, char* err,
    size_t cap) {
  if (!k_pool || !v_pool || !seq_ids || !pos || !q || !out) {
    put(err, cap, "null pointer");
    return VXG_ATTN_ERR_NULL_PTR;
  }
  if ((k_new == nullptr) != (v_new == nullptr)) {
    put(err, cap, "k_new and v_new must both be given or both be NULL");
    return VXG_ATTN_ERR_NULL_PTR;
  }
  // bulk copies and vector accesses need 16-byte aligned arrays
  const void* arrays[] = {k_pool, v_pool, q, k_new, v_new, q_gate, out};
  for (const void* p : arrays)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15u)) {
      put(err, cap, "device arrays must be 16-byte aligned");
      return VXG_ATTN_ERR_INVALID_OPTION;
    }
  if (head_dim == 0 || head_dim % 32 || head_dim > 256) {
    put(err, cap, "head_dim must be a multiple of 32, at most 256");
    return VXG_ATTN_ERR_UNSUPPORTED;
  }
  if (n_head_kv == 0 || n_head == 0 || n_head % n_head_kv || n_seq == 0 || cap_tokens == 0 ||
      (uint64_t)n_seq * cap_tokens >= (1ull << 31)) {
    put(err, cap, "bad shape (n_head must be a multiple of n_head_kv; pool sizes positive)");
    return VXG_ATTN_ERR_INVALID_OPTION;
  }
  if (n_batch == 0) return VXG_ATTN_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    put(err, cap, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return VXG_ATTN_ERR_INTERNAL;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    put(err, cap, "device index " + std::to_string(dev) + " is beyond the " +
                      std::to_string(kMaxDevices) + " devices this entry point keeps set-up for");
    return VXG_ATTN_ERR_UNSUPPORTED;
  }
  DeviceScratch ds;
  int rc = setup(dev, &ds, err, cap);
  if (rc != VXG_ATTN_OK) return rc;

  vxg::DecodeArgs a{};
  a.seq_ids = seq_ids;
  a.kv_begin = nullptr;
  a.kv_end = pos;
  a.end_add = 1;  // attend to [0, pos[b]]
  a.q = q;
  a.k_pool = static_cast<const uint8_t*>(k_pool);
  a.v_pool = static_cast<const uint8_t*>(v_pool);
  a.n_batch = (int)n_batch;
  a.n_seq = (int)n_seq;
  a.cap = (int)cap_tokens;
  a.n_head = (int)n_head;
  a.n_kv = (int)n_head_kv;
  a.nb = (int)(head_dim / 32);
  a.max_ctx = (int)cap_tokens;
  a.scale = scale;
  const size_t floats = vxg::decode_partial_floats(a, ds.sm_count);
  if (kStatusBytes + floats * sizeof(float) > kScratchBytes) {
    put(err, cap, "this batch needs " + std::to_string(floats * sizeof(float)) +
                      " bytes of split-KV scratch; the built-in array holds " +
                      std::to_string(kScratchBytes - kStatusBytes) +
                      " (split the batch, or use vxg_attn_cuda_q8_decode)");
    return VXG_ATTN_ERR_BUFFER_TOO_SMALL;
  }
  uint32_t* status = reinterpret_cast<uint32_t*>(ds.base);
  a.status = status;
  vxg::Partials part =
      vxg::carve_partials(reinterpret_cast<float*>(ds.base + kStatusBytes), a, ds.sm_count);

  // NULL stream: run on the legacy default stream and wait, so the status can be reported.
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
  auto fail = [&](cudaError_t ce, const char* what) {
    cudaStreamSynchronize(st);
    put(err, cap, std::string(what) + ": " + cudaGetErrorString(ce));
    return VXG_ATTN_ERR_INTERNAL;
  };
  if ((e = cudaMemsetAsync(status, 0, sizeof(uint32_t), st)) != cudaSuccess)
    return fail(e, "status clear");
  if (k_new &&
      (e = vxg::launch_q8_append(seq_ids, pos, k_new, v_new, static_cast<uint8_t*>(k_pool),
                                 static_cast<uint8_t*>(v_pool), (int)n_batch, 1, (int)n_seq,
                                 (int)cap_tokens, (int)n_head_kv, a.nb, status, st)) != cudaSuccess)
    return fail(e, "q8_append launch");
  if ((e = vxg::launch_decode(a, part, q_gate, out, ds.sm_count, 0, st, nullptr, nullptr)) !=
      cudaSuccess)
    return fail(e, "decode launch");
  if (stream) return VXG_ATTN_OK;  // asynchronous: the device status word is not collected
  uint32_t s = 0;
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return fail(e, "cudaStreamSynchronize");
  if ((e = cudaMemcpy(&s, status, sizeof(s), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return fail(e, "status readback");
  if (s & vxg::kStatusTimeout) {
    put(err, cap, "a device-side bounded wait gave up");
    return VXG_ATTN_ERR_INTERNAL;
  }
  if (s & vxg::kStatusBadIndex) {
    put(err, cap, "a sequence id or position was outside the KV pool; that entry was skipped");
    return VXG_ATTN_ERR_INVALID_OPTION;
  }
  return (s & vxg::kStatusNonFinite) ? VXG_ATTN_WARN_NONFINITE : VXG_ATTN_OK;
}
