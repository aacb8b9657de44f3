/*
 * avqa_b200 -- C ABI of the B200 AVQ-attention kernels.
 *
 * Every entry point takes raw device pointers, plain integer sizes and a
 * CUDA stream (as void*), enqueues its kernels on that stream and returns an
 * int status: 0 = AVQ_OK, otherwise an error code; avq_last_error() returns
 * the message of the calling thread's last failure.  Nothing here allocates
 * device memory: scratch space is the caller's `workspace`, sized by the
 * matching *_workspace_size() query.
 *
 * dtype: 0 = fp32, 1 = bf16, 2 = fp16.  Tensors in "dtype" hold elements of
 * that type; counts and indices are int32.  Strides are in elements: element
 * (b, h, s, d) of a 4-D operand is at b*stride[0] + h*stride[1] + s*stride[2] + d
 * (so module layout [B, S, H*D] is {S*H*D, D, H*D} and head layout
 * [B, H, S, D] is {H*S*D, S*D, D}).
 *
 * Reference interfaces replaced (paths in sachncs/avqa):
 *   avq_prepare_codebook  attention_module.py:344-348 (codebook cast to the
 *                         input dtype) + the squared norms of quantizer.py:208,224
 *   avq_quantize          Backend.quantize / TorchBackend.quantize, backend.py:216-237
 *                         -> EuclideanHierarchicalQuantizer.precompute, quantizer.py:166-278
 *   avq_forward           run_pipeline stages 6-11, pipeline.py:322-393, with
 *                         AVQAttention.refine_and_output, attention_module.py:471-544
 *   avq_append            resolve_kv_cache + KVCache.append, attention_module.py:350-367,
 *                         cache.py:246-260, plus the re-quantization of the grown key
 *                         set (quantizer.py:166-278) done incrementally
 *   avq_reduce_min        the budget's min over (b,h) of valid parents, pipeline.py:341-342
 *   avq_codeword_presence the user / causal mask's codeword visibility, pipeline.py:82-106,
 *                         attention_module.py:210-223, 369-390
 *   avq_bcar_update       online_codebook_adaptation, online_adaptation.py:37-127
 *   avq_stream_extend     StreamingVQBuffer.extend, streaming_vq.py:109-229
 *   avq_dense_attention   TorchBackend.naive_attention / online_softmax_attention,
 *                         backend.py:105-156, 190-203
 *   avq_device_fault      no counterpart: device-side fault record of the bounded waits
 *   avq_quantize_noalloc  no counterpart: avq_quantize with its scratch in a fixed
 *                         device array, for hosts that cannot allocate
 */
#ifndef AVQA_B200_H
#define AVQA_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AVQ_OK 0
#define AVQ_ERR_ARG 1
#define AVQ_ERR_CUDA 2
#define AVQ_ERR_UNSUPPORTED 3
#define AVQ_ERR_WORKSPACE 4

/* Library version string. */
const char* avq_version(void);

/* Copy the calling thread's last error message into buf (NUL-terminated);
 * returns its full length. */
int avq_last_error(char* buf, int len);

/* Cast the fp32 master codebook to `dtype` and compute the dtype-rounded
 * squared norms.  parents32 [H,M0,D], children32 [H,M0,C,D] (fp32);
 * outputs parents_dt [H,M0,D], children_dt [H,M0,C,D] (dtype),
 * p_sq [H,M0], c_sq [H,M0,C] (fp32 holding dtype values). */
int avq_prepare_codebook(int dtype, const float* parents32, const float* children32, int H, int M0, int C, int D,
                         void* parents_dt, void* children_dt, float* p_sq, float* c_sq, void* stream);

size_t avq_quantize_workspace_size(int B, int H, int S, int M0);

/* Hierarchical VQ of S keys per (b,h) against the (b,h)'s head codebook.
 * keys/values: dtype with strides key_strides/value_strides (3 longs each).
 * Outputs (G = B*H): passign, cassign [G,S]; pagg [G,M0,D] and cagg
 * [G,M0,C,D] in dtype; pacc/cacc the fp32 sums before narrowing (may be
 * NULL); pcnt [G,M0], ccnt [G,M0,C] exact counts; nvalid [G] non-empty
 * parents; gmin_valid (may be NULL) receives atomicMin(nvalid) -- the caller
 * initialises it (e.g. to INT_MAX). */
int avq_quantize(int dtype, const void* keys, const long long* key_strides, const void* values,
                 const long long* value_strides, int B, int H, int S, int D, int M0, int C, const void* parents_dt,
                 const float* p_sq, const void* children_dt, const float* c_sq, int* passign, int* cassign,
                 void* pagg, void* cagg, float* pacc, float* cacc, int* pcnt, int* ccnt, int* nvalid,
                 int* gmin_valid, void* workspace, size_t workspace_bytes, void* stream);

/* Size in bytes of the fixed scratch array behind avq_quantize_noalloc: one
 * array per device, 16 MiB.  A call needs avq_quantize_workspace_size(B, H,
 * S, M0) bytes of it (12.3 MiB for B=4, H=32, S=8192, M0=512). */
#define AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)

/* avq_quantize for callers that cannot supply a device workspace.  No
 * counterpart in the reference, whose torch quantizer allocates through the
 * torch caching allocator on every call.
 *
 * Arguments, outputs and results are those of avq_quantize (same kernels);
 * only `workspace`/`workspace_bytes` are gone.  The quantizer's scratch --
 * bucket histograms, key order, bucket offsets, a work counter -- lives in a file-scope
 * device array compiled into the library, so the call allocates nothing.
 *
 * Who needs it: a host whose device memory is owned by someone else -- a
 * serving runtime that reserved the GPU's memory for its own pool up front,
 * or a foreign-language host (cgo, JNI) with no device allocator of its own
 * -- where a cudaMalloc would fail, or take memory the pool counts on, and a
 * cudaFree would synchronize the device in the middle of a prefill.
 *
 * Limits and rules:
 *  - Requests needing more than AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES fail with
 *    AVQ_ERR_WORKSPACE before anything is enqueued; use avq_quantize then.
 *  - The scratch need not start zeroed: every call writes each scratch byte
 *    before reading it.  gmin_valid, as for avq_quantize, must be initialised
 *    by the caller.
 *  - The array is shared by every call on a device: calls that overlap on one
 *    device (two streams, or two host threads without ordering) race on it.
 *    Issue them in order on one stream.
 *  - The first call in each CUDA context (the context current at the call:
 *    the device's primary context for a runtime-API host, the host's own
 *    context for a driver-API host) does a one-time setup: it looks up the
 *    array's device address with cudaGetSymbolAddress, which may load the
 *    library's device code into that context.  Make that first call before
 *    any stream capture begins on the device.  The address is cached per
 *    context handle; a host that destroys a context and creates another one
 *    under the same handle (cudaDeviceReset) must not call this entry point
 *    afterwards. */
int avq_quantize_noalloc(int dtype, const void* keys, const long long* key_strides, const void* values,
                         const long long* value_strides, int B, int H, int S, int D, int M0, int C,
                         const void* parents_dt, const float* p_sq, const void* children_dt, const float* c_sq,
                         int* passign, int* cassign, void* pagg, void* cagg, float* pacc, float* cacc, int* pcnt,
                         int* ccnt, int* nvalid, int* gmin_valid, void* stream);

/* Dense softmax attention, the reference's naive path (backend.py:190-203,
 * the online-softmax form of :105-156; used by execution.mode="reference",
 * by refinement disabled and by the budget-0 fallback, pipeline.py:261-273,
 * 310-345): out = softmax(mask(DT(DT(q k^T) * D^-1/2))) v in the input dtype.
 * q [B,H,T,D], k and v [B,H,N,D] (strides as avq_quantize), out [B,H,T,D]
 * (out_strides).  mask NULL, or uint8 (nonzero = attend) with element strides
 * {b, h, t} and unit key stride (zero strides broadcast).  A query with every
 * key masked gets NaN, as softmax over -inf does. */
int avq_dense_attention(int dtype, const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                        const void* v, const long long* v_strides, int B, int H, int T, int N, int D,
                        const unsigned char* mask, const long long* mask_strides, void* out,
                        const long long* out_strides, void* stream);

size_t avq_bcar_workspace_size(int B, int H, int M0, int C, int D);

/* BCAR online codebook adaptation (online_adaptation.py:37-127, run by
 * run_vq_precompute, attention_module.py:420-428): one EMA step of the child
 * codebook toward the mean of the keys assigned to each child cell,
 * children' = c + DT(w * DT(mean - c)) with w = DT(1 - decay) where the cell
 * got keys, averaged over the batch (the reference tiles the codebook with
 * repeat_interleave(B) while groups are ordered b*H + h; that pairing is
 * kept), then parents' = mean of their children.  keys [B,H,S,D] (strides as
 * avq_quantize), passign/cassign [B*H, S] from avq_quantize; children_in
 * [H,M0,C,D] in dtype; writes children_out (must not alias children_in) and
 * parents_out [H,M0,D].  workspace: avq_bcar_workspace_size bytes. */
int avq_bcar_update(int dtype, const void* keys, const long long* key_strides, const int* passign, const int* cassign,
                    int B, int H, int S, int D, int M0, int C, float decay, const void* children_in, void* children_out,
                    void* parents_out, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes for avq_stream_extend with B new keys (0 for bad sizes). */
size_t avq_stream_workspace_size(int B, int H, int M0, int C);

/* Streaming VQ extend (StreamingVQBuffer.extend, streaming_vq.py:109-229):
 * B new keys [B, D] (row stride key_row_stride elements, unit inner stride),
 * the same keys for every head, are assigned against parents [H,M0,D] by the
 * distance DT(DT(k_sq - 2 k.p) + p_sq) and against the assigned parent's
 * children [H,M0,C,D] by sum DT((k - c)^2) (first argmin, a NaN wins).
 * Writes parent_out / child_out [B,H] int64; when parent_record is not NULL
 * also appends them to the running records [H, record_stride] laid out as the
 * reference's assign.reshape(1, H, B): flat result i at row i / B, column
 * record_size + i % B.  Then adds the keys into the running sums
 * parent_aggregates [H,M0,D] / child_aggregates [H,M0,C,D] (dtype) and the
 * int64 counts [H,M0] / [H,M0,C] as the reference's index_add_ does: flat
 * row i adds key i / H to head i / B; the rows of one call accumulate in
 * fp32 in row order from the stored value and narrow once.  D <= 512.
 * All buffers are contiguous device memory; keys, codebook and aggregates
 * share `dtype`.  workspace: avq_stream_workspace_size bytes.  B = 0 is a
 * no-op. */
int avq_stream_extend(int dtype, const void* keys, long long key_row_stride, int B, int H, int M0, int C, int D,
                      const void* parents, const void* children, long long* parent_out, long long* child_out,
                      long long* parent_record, long long* child_record, long long record_stride,
                      long long record_size, long long* parent_counts, long long* child_counts,
                      void* parent_aggregates, void* child_aggregates, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Words per (b,h, query) row of the codeword visibility bits: ceil(M0 / 32). */
int avq_presence_words(int M0);

/* Codeword visibility under a mask (pipeline.py:82-106 with the causal mask
 * of attention_module.py:210-223, 369-390): parent p is visible to query t of
 * (b,h) when at least one key assigned to it is allowed by the mask.  Bit
 * p % 32 of present[((b*H + h)*T + t)*W + p/32] (W = avq_presence_words(M0),
 * present holds B*H*T*W words) is set for a visible parent.
 * mask NULL: the causal mask, query t sees keys 0 .. t + causal_offset (the
 * reference uses causal_offset = S - T: the cached prefix is visible to every
 * query).  Otherwise mask is uint8 (nonzero = attend) with element strides
 * mask_strides {b, h, t} (the key stride is 1; zero strides broadcast, so a
 * [T, S] mask passes {0, 0, S}).  passign [state_batch*H, S] are the parent
 * assignments of avq_quantize; state_batch is B or 1 as in avq_forward.
 * workspace: avq_presence_workspace_size bytes for the causal path (may be
 * NULL with a user mask). */
int avq_codeword_presence(const int* passign, int B, int H, int S, int M0, int T, int state_batch,
                          const unsigned char* mask, const long long* mask_strides, int causal_offset,
                          unsigned int* present, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes of avq_codeword_presence's causal path (mask NULL): the first
 * key position of every (key set, parent).  A user mask needs none. */
size_t avq_presence_workspace_size(int H, int M0, int state_batch);

/* Number of int32 slots per (b,h) in the `selected` output of avq_forward:
 * the sum of the per-pass budget caps for base budget P. */
int avq_selection_stride(int P, int passes, float pass_decay);

size_t avq_forward_workspace_size(int dtype, int B, int H, int T, int D, int M0, int C, int P, int passes,
                                  float pass_decay, int hvaq);

/* AVQ attention of T queries per (b,h) over a quantized key set.
 * q: dtype with q_strides; out: fp32 with out_strides (module layout
 * [B,T,H*D] -> {T*H*D, D, H*D}).  state_batch: the batch of the quantized
 * state (pagg, cagg, pcnt, ccnt): B, or 1 when one key set serves all B query
 * batches (query chunks of one sequence over keys quantized once; each chunk
 * is routed on its own, as a separate reference call over the same keys would
 * be).  min_valid: device int, the minimum over every (b,h) of the call (or
 * of all ranks) of non-empty parents; the routing budget is
 * min(P, *min_valid).  min_valid_ready: NULL, or a cudaEvent_t recorded by
 * whatever produces *min_valid (e.g. a cross-rank all-reduce on another
 * stream): `stream` waits on it only before the routing kernel, so the
 * parent-attention kernel overlaps the reduction.  present: NULL, or the
 * codeword visibility bits of avq_codeword_presence for these B*H*T query
 * rows (a masked parent's logit is -inf for that query).  hvaq: 0 off, 1 entropy schedule,
 * 2 linear schedule; beta0 the base temperature (1/sqrt(D) when the config
 * says 0), alpha the linear slope.  importance_out [G,M0] fp32, selected_out
 * [G, avq_selection_stride()] int32 and pass_counts_out [passes] int32 are
 * optional diagnostics (NULL to skip). */
int avq_forward(int dtype, const void* q, const long long* q_strides, int B, int H, int T, int D, int M0, int C,
                const void* parents_dt, const void* children_dt, const void* pagg, const void* cagg, const int* pcnt,
                const int* ccnt, int state_batch, const int* min_valid, void* min_valid_ready,
                const unsigned int* present, int P, int passes, float pass_decay, int hvaq, float beta0,
                float alpha, float* out, const long long* out_strides, float* importance_out, int* selected_out,
                int* pass_counts_out, void* workspace, size_t workspace_bytes, void* stream);

size_t avq_append_workspace_size(int B, int H, int Tn);

/* Append Tn new tokens per (b,h) to a quantized key set, in order:
 * assign each new key, add its value to the fp32 bucket sums pacc/cacc,
 * refresh pagg/cagg, bump pcnt/ccnt/nvalid.  When kpage/vpage are not NULL
 * the raw k/v are also written to page slots slot0.. (page_strides).
 * workspace: avq_append_workspace_size(B, H, Tn) bytes (the new keys'
 * parents, found on the tensor cores as the prefill quantizer finds them). */
int avq_append(int dtype, const void* k, const long long* k_strides, const void* v, const long long* v_strides,
               int B, int H, int Tn, int D, int M0, int C, const void* parents_dt, const float* p_sq,
               const void* children_dt, const float* c_sq, float* pacc, float* cacc, void* pagg, void* cagg,
               int* pcnt, int* ccnt, int* nvalid, void* kpage, void* vpage, const long long* page_strides, int slot0,
               void* workspace, size_t workspace_bytes, void* stream);

/* *out = min(v[0..n)). */
int avq_reduce_min(const int* v, int n, int* out, void* stream);

/* Read and clear the device-side fault record, after synchronizing `stream`.
 * *code receives 0, or a nonzero bit set by a kernel that abandoned a
 * bounded wait (about one second) on one of its own barriers; the kernel
 * then released its resources and returned with undefined outputs.  No
 * counterpart in the reference (its CPU kernels have no asynchronous waits). */
int avq_device_fault(int* code, void* stream);

/* Per-kernel device timing (no counterpart in the reference; measurement
 * support).  avq_profile_begin() starts recording a CUDA event pair around
 * every kernel the library launches; avq_profile_end() waits for them and
 * writes, per kernel name (names joined by '\n'), the summed milliseconds and
 * the launch count; returns the number of kernels (or -1 on error). */
int avq_profile_begin(void);
int avq_profile_end(char* names, int names_len, float* total_ms, int* launches, int max_kernels);

#ifdef __cplusplus
}
#endif

#endif /* AVQA_B200_H */
