// Internal launch interface between the C-ABI host layer (abi.cu) and the kernels.
#pragma once
#include <utility>

#include "common.cuh"

namespace vxg {

// Launch with programmatic stream serialisation: the kernel may start before the previous
// kernel of the stream completes; it must call grid_dep_wait() before it reads anything that
// kernel wrote (and before it reads anything written earlier in the stream).
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// q8_append.cu -----------------------------------------------------------------------------
// For batch entry b and token t < n_tok: quantise k_new/v_new[b][t][n_kv][32*nb] into
// sequence seq_ids[b] at position pos[b] + t.
cudaError_t launch_q8_append(const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                             const float* v_new, uint8_t* k_pool, uint8_t* v_pool, int n_batch,
                             int n_tok, int n_seq, int cap, int n_kv, int nb, uint32_t* status,
                             cudaStream_t stream);
// Same with bf16 inputs (k_new / v_new are __nv_bfloat16; bf16 -> f32 is exact).
cudaError_t launch_q8_append_bf16(const int32_t* seq_ids, const int32_t* pos, const void* k_new,
                                  const void* v_new, uint8_t* k_pool, uint8_t* v_pool, int n_batch,
                                  int n_tok, int n_seq, int cap, int n_kv, int nb, uint32_t* status,
                                  cudaStream_t stream);

// Copy of fp32 K/V tokens into fp32 pools: k_new/v_new[b][t][n_kv][hd] -> sequence seq_ids[b]
// at position pos[b] + t (the reference's k_cache.extend_from_slice, llm_ops.rs:256-257).
cudaError_t launch_f32_append(const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                              const float* v_new, float* k_pool, float* v_pool, int n_batch,
                              int n_tok, int n_seq, int cap, int n_kv, int hd, uint32_t* status,
                              cudaStream_t stream);

// decode_attn.cu ---------------------------------------------------------------------------
struct DecodeArgs {
  const int32_t* seq_ids;  // [n_batch]
  const int32_t* kv_begin; // [n_batch] first token attended (nullptr -> 0)
  const int32_t* kv_end;   // [n_batch] one past the last token attended
  const float* q;          // [n_batch][n_head][hd] prepared queries
  const uint8_t* k_pool;   // [n_seq][cap][n_kv][nb] blocks
  const uint8_t* v_pool;
  int n_batch, n_seq, cap, n_head, n_kv, nb;
  int end_add;             // effective end of entry b = kv_end[b] + end_add (decode: pos + 1)
  int max_ctx;             // upper bound of (end - begin) over the batch (host-known)
  float scale;             // softmax scale (1/sqrt(hd) in the reference)
  uint32_t* status;
  int kv_f32;              // pools hold fp32 K/V [n_seq][cap][n_kv][hd] (portable kernel only)
};

// Partial (m, l, o) buffers for the split-KV pass: m, l in log2 units, o unnormalised.
// State of the fast split pass that outlives a call, at the front of the split-KV scratch
// (zero when the scratch is new): the measured units per microsecond of each CTA's range in the
// last call, in two buffers.  The split pass reads buffer `cur` to size its CTAs' unit ranges
// and writes the other; the last of its CTAs to finish (counted in `done`) flips `cur`, after
// every CTA has read it.  Every CTA of one call thus reads the same rates, and any rates give
// a valid partition of the units.
struct FastState {
  int cur;
  unsigned done;
  int pad[30];
  float rate[2][512];
};
constexpr size_t kFastStateFloats = sizeof(FastState) / sizeof(float);

struct Partials {
  FastState* state;  // the split pass's cross-call state (front of the scratch)
  float* m;   // [n_slot][n_head]
  float* l;   // [n_slot][n_head]
  float* o;   // [n_slot][n_head][hd]
  float* inter; // second-level merge scratch of the fast combine
  int* prefix;  // unit prefix over the batch, published by the fast split pass
  int n_slot; // slots available
};

// Floats of partial storage the split-KV pass needs for these args, and its carving.
size_t decode_partial_floats(const DecodeArgs& a, int sm_count);
Partials carve_partials(float* base, const DecodeArgs& a, int sm_count);

// Split-KV pass then LSE combine into out[n_batch][n_head][hd] (gate optional, same shape).
// `force_generic` selects the portable kernel even when the fast path applies.
cudaError_t launch_decode(const DecodeArgs& a, const Partials& part, const float* gate,
                          float* out, int sm_count, int force_generic, cudaStream_t stream,
                          cudaEvent_t ev_split_begin, cudaEvent_t ev_split_end);

// Split-KV pass only, leaving one combined (m, l, o) per (batch, head): m_out/l_out
// [n_batch][n_head], o_out [n_batch][n_head][hd] (o unnormalised, m in log2 units).
cudaError_t launch_decode_partial(const DecodeArgs& a, const Partials& part, float* m_out,
                                  float* l_out, float* o_out, int sm_count, int force_generic,
                                  cudaStream_t stream, cudaEvent_t ev_split_begin,
                                  cudaEvent_t ev_split_end);

// Log-sum-exp merge of n_parts partial results: m,l [n_parts][n_rows], o [n_parts][n_rows][hd]
// -> out [n_rows][hd] (normalised, gate optional [n_rows][hd]).
cudaError_t launch_lse_combine(int n_parts, int n_rows, int hd, const float* m, const float* l,
                               const float* o, const float* gate, float* out, uint32_t* status,
                               cudaStream_t stream);
// Same merge over packed parts: packed[k] = [m (n_rows) | l (n_rows) | o (n_rows*hd)].
cudaError_t launch_lse_combine_packed(int n_parts, int n_rows, int hd, const float* packed,
                                      const float* gate, float* out, uint32_t* status,
                                      cudaStream_t stream);

// deltanet.cu ------------------------------------------------------------------------------
struct DeltaNetArgs {
  // Element (b, t, head, i) of q / k is at q + b*q_bs + t*q_ts + head*dk + i (k likewise);
  // v, o, z, y use (v_bs, v_ts) / (o_bs, o_ts) with head*dv; beta_raw, alpha_raw use (g_bs, g_ts).
  const float* q;          // before L2 norm
  const float* k;
  const float* v;
  const float* beta_raw;
  const float* alpha_raw;
  const float* ssm_a;      // [n_vh]
  const float* dt_bias;    // [n_vh]
  float* state;            // [n_batch][n_vh][dv][dk] updated in place
  float* o;                // S_new q (not written by the decode step when y != nullptr)
  const float* z;          // epilogue gate input (optional, with y)
  const float* ssm_norm;   // [dv] RMSNorm weight (with y)
  float* y;                // optional: RMSNorm(o) * ssm_norm * SiLU(z)
  long long q_bs, q_ts, k_bs, k_ts, v_bs, v_ts, g_bs, g_ts, o_bs, o_ts;
  int n_batch, n_tok, n_kh, n_vh, dk, dv;
  float eps, q_scale;
  uint32_t* status;
};
// One token per sequence (t = 0), state streamed from / to HBM.
cudaError_t launch_deltanet_step(const DeltaNetArgs& a, cudaStream_t stream);
// n_tok tokens per sequence with the state held on chip; needs deltanet_prefill_scratch_bytes of
// device scratch.  Writes o (y is not used: the prefill returns o before the epilogue).
// allow_chunk: dk 128 and dv a multiple of 64 with at least 64 tokens run the chunked (WY)
// form (deltanet_tc.cu for dv = 128, deltanet_chunk.cu otherwise); other shapes, or
// allow_chunk = 0, the sequential on-chip recurrence.
size_t deltanet_prefill_scratch_bytes(const DeltaNetArgs& a);
cudaError_t launch_deltanet_prefill(const DeltaNetArgs& a, void* scratch, int allow_chunk,
                                    cudaStream_t stream);
// deltanet_chunk.cu: qn / kn normalised q, k [b][t][n_kh][128], gates (beta, decay) and lgs
// (log decay) [b][t][n_vh] from the prep kernel.
bool deltanet_chunk_supported(const DeltaNetArgs& a);
size_t deltanet_chunk_smem_bytes();
cudaError_t launch_deltanet_chunk(const DeltaNetArgs& a, const float* qn, const float* kn,
                                  const float2* gates, const float* lgs, cudaStream_t stream);
// deltanet_tc.cu: the same chunked form on tcgen05 / TMEM for dk = dv = 128 (one CTA per
// (sequence, v head) with the whole state in tensor memory); reads the raw arguments (norms
// and gates on chip), so it needs no preparation pass and no scratch.
bool deltanet_chunk_tc_supported(const DeltaNetArgs& a);
size_t deltanet_chunk_tc_smem_bytes();
cudaError_t launch_deltanet_chunk_tc(const DeltaNetArgs& a, cudaStream_t stream);
// conv1d + SiLU over the rolling history (llm_ops.rs:122-137), batched.
cudaError_t launch_deltanet_conv(const float* x, const float* w, float* conv_state, float* out,
                                 int n_batch, int conv_ch, int k_sz, cudaStream_t stream);

// prefill_attn.cu --------------------------------------------------------------------------
struct PrefillArgs {
  const int32_t* seq_ids;  // [n_batch]
  const int32_t* pos_base; // [n_batch] cache position of prompt token 0
  const void* q;           // [n_batch][n_tok][n_head][hd] (f32 or bf16) prepared queries
  const void* k_new;       // [n_batch][n_tok][n_kv][hd] appended to the cache first
  const void* v_new;
  const void* gate;        // optional sigmoid gate, q's shape and type
  const uint8_t* k_pool;   // [n_seq][cap][n_kv][hd/32] blocks (written by the append)
  const uint8_t* v_pool;
  float* out;              // [n_batch][n_tok][n_head][hd]
  __half* kd[2];           // dequantised cache, hi and lo f16 planes [n_batch][lmax][n_kv][hd]
  __half* vd[2];           // (carved from scratch by launch_prefill)
  int n_batch, n_tok, n_seq, cap, n_head, n_kv, hd;
  int lmax;                // >= pos_base[b] + n_tok for every b (host-known)
  float scale;
  uint32_t* status;
};
// Append + causal attention of n_tok prompt tokens per sequence (hd = 256, n_head = 8 * n_kv).
size_t prefill_scratch_bytes(const PrefillArgs& a);
size_t prefill_smem_bytes();
bool prefill_supported(int n_head, int n_kv, int hd);
// ev_attn_begin / ev_attn_end (nullable) bracket the attention kernel.  With allow_tc, bf16
// inputs at head_dim 256 run the tcgen05/TMEM kernel (prefill_tc.cu, no scratch used); everything
// else runs the mma.sync kernel over the dequantised f16 planes.
cudaError_t launch_prefill(const PrefillArgs& a, void* scratch, int bf16, int allow_tc,
                           cudaStream_t stream, cudaEvent_t ev_attn_begin,
                           cudaEvent_t ev_attn_end);
// prefill_tc.cu
bool prefill_tc_supported(int n_head, int n_kv, int hd, int bf16);
size_t prefill_tc_smem_bytes();
cudaError_t launch_prefill_tc(const PrefillArgs& a, cudaStream_t stream);

// prep.cu ----------------------------------------------------------------------------------
// q/k prologue of step_full_gqa_q8 for one token: rope_cs = host-computed (cos, sin) pairs.
cudaError_t launch_gqa_prep(const float* q_raw, float* k_cur, const float* q_norm,
                            const float* k_norm, int gated, int n_head, int n_kv, int hd,
                            const float2* rope_cs, int rope_half, int neox, float eps,
                            float* q_out, float* gate_out, cudaStream_t stream);

// peer.cu: long-context partials exchanged over NVLink peer memory
struct PeerTable {
  float* buf[8];  // exchange buffer of rank r, as mapped on this GPU (own buffer at `rank`)
};
size_t peer_buffer_bytes(int world, int per);
cudaError_t launch_peer_push(const float* send, int per, const PeerTable& peers, int world,
                             int rank, float* local_buf, cudaStream_t stream);
cudaError_t launch_peer_combine(const float* local_buf, int world, int n_rows, int hd,
                                const float* gate, float* out, uint32_t* status,
                                cudaStream_t stream);

}  // namespace vxg
