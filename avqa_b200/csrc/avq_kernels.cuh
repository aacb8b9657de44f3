// Internal declarations shared by the kernel translation units and the C-ABI.
#pragma once

#include "avq_common.cuh"
#include "avq_profile.cuh"

namespace avq {

// Element (b, h, s, d) of a 4-D tensor lives at b*b_ + h*h_ + s*s_ + d.
struct Strides3 {
  long b, h, s;
};

inline size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

// Row pitch, in elements, of the per-64-query exponential slices that the
// parent-attention kernels write and the routing kernel re-reads: M0 rounded up
// to 16, plus 16, so that every row of a 16-bit slice starts on a 32-byte
// boundary.
__host__ __device__ inline int exp_slice_pitch(int M0) { return ((M0 + 15) & ~15) + 16; }

struct QuantizeArgs {
  const void* keys;
  Strides3 ks;
  const void* values;
  Strides3 vs;
  int B, H, S, D, M0, C;
  const void* parents_dt;
  const float* p_sq;
  const void* children_dt;
  const float* c_sq;
  int* passign;
  int* cassign;
  void* pagg;
  void* cagg;
  float* pacc;  // optional fp32 accumulators (needed for incremental decode)
  float* cacc;
  int* pcnt;
  int* ccnt;
  int* nvalid;
  int* gmin_valid;  // optional: atomicMin of nvalid (caller initialises it)
  void* workspace;
  size_t workspace_bytes;
};

struct ForwardArgs {
  const void* q;
  Strides3 qs;
  int B, H, T, D, M0, C;
  const void* parents_dt;
  const void* children_dt;
  const void* pagg;
  const void* cagg;
  const int* pcnt;
  const int* ccnt;
  const int* min_valid;  // device scalar: min over all (b,h) of non-empty parents
  int P;
  int passes;
  float pass_decay;
  int hvaq;  // 0 off, 1 entropy, 2 linear
  float beta0;
  float alpha;
  float* out;  // fp32
  Strides3 os;
  float* importance_out;  // optional [G, M0] pre-HVAQ importance (dtype values)
  int* selected_out;      // optional [G, sel_stride] selections of every pass
  int* pass_counts_out;   // optional [passes]
  void* workspace;
  size_t workspace_bytes;
  // Groups (b,h) of the quantized state: B*H, or H when one state (batch 1)
  // serves every query batch -- query chunks over one cached key set.  The
  // state of query group g is g % state_groups.  0 means B*H.
  int state_groups = 0;
  void* min_valid_ready = nullptr;  // optional cudaEvent_t awaited before routing
  // optional codeword visibility under a mask: bit p % 32 of word
  // present[(g T + t) W + p / 32], W = presence_words(M0), for query group g
  const unsigned int* present = nullptr;
};

struct AppendArgs {
  const void* k;
  Strides3 ks;
  const void* v;
  Strides3 vs;
  int B, H, Tn, D, M0, C;
  const void* parents_dt;
  const float* p_sq;
  const void* children_dt;
  const float* c_sq;
  float* pacc;
  float* cacc;
  void* pagg;
  void* cagg;
  int* pcnt;
  int* ccnt;
  int* nvalid;
  void* kpage;  // optional paged K/V destination
  void* vpage;
  Strides3 pgs;
  int slot0;
  void* workspace = nullptr;  // append_workspace_bytes(B, H, Tn): the new keys' parents
  size_t workspace_bytes = 0;
};

// Parent-attention pass of the tensor-core path (avq_attention_mma.cu).
struct PAArgs {
  const void* q;
  Strides3 qs;
  int B, H, T, D, M0;
  float sqrtD;
  const void* parents;
  const void* pagg;
  const int* pcnt;
  int mode;            // 0 plain, 1 HVAQ rescale of the stored logits
  int keep_logits;     // mode 0 only: leave the logits in sglobal for a later HVAQ pass
  void* sglobal;       // logits scratch when they do not fit in shared memory
  bool s_in_smem;
  float *m, *l, *z;    // [G,T]
  void* a;             // [G,T,D] dtype
  float* colpart;      // [G, nqt, M0] fp32 column sums of probs per 64-query tile
  const int* sel0;
  int sel_stride;
  const int* pass_cnt;
  int hvaq;
  float beta0, alpha;
  float* beta;         // [G,T]
  int sG = 0;          // state groups: the state of query group g is g % sG
  const unsigned int* present = nullptr;  // optional mask bits (see ForwardArgs)
};

// Importance from fp32 per-tile column partials, with the exact fallback
// reading the parent-attention tiles (see route_kernel).
struct RouteExact {
  const float* colpart;  // nullptr: the fp64 partials path
  const void* scratch;   // dtype tiles [G][nqt][64][exp_slice_pitch(M0)]
  int scr_logits;        // tiles hold logits (exponentials recomputed from m)
  const float* m;        // [G,T]
  const float* z;        // [G,T]
  int T;
};

struct PassOffsets {
  int off[8];
};

struct CorrArgs {
  const void* q;
  Strides3 qs;
  int B, H, T, D, M0, C;
  float sqrtD;
  const void* parents;
  const void* children;
  const void* pagg;
  const void* cagg;
  const int* pcnt;
  const int* ccnt;
  const float *m, *l, *z, *beta;  // beta: HVAQ temperatures or nullptr
  const void* a;                  // [G,T,D] dtype
  const int* sel;
  int sel_stride;
  const int* pass_cnt;
  int npass;
  int pass_off[8];
  int multipass;
  float* out;
  Strides3 os;
  int sG = 0;  // state groups: the state of query group g is g % sG
  const unsigned int* present = nullptr;  // optional mask bits (see ForwardArgs)
};

template <int DT>
int launch_parent_attn_mma(const PAArgs& a, cudaStream_t st);
template <int DT>
int launch_correct_mma(const CorrArgs& a, cudaStream_t st);
size_t parent_attn_mma_smem(int D, int M0, bool s_in_smem, int dt_bytes);
bool parent_attn_mma_ok(int dt, int D, int M0);
bool parent_attn_mma_smem_mode(int D, int M0);
size_t parent_attn_mma_scratch(int G, int T, int M0, int dt_bytes);
constexpr int PM_ROWS_PUBLIC = 64;

// tcgen05 parent attention (first pass without HVAQ): same outputs, scratch
// slices and 64-query importance partials as launch_parent_attn_mma.
bool parent_attn_tc_ok(int dt, int D, int M0);
// The HVAQ rescaling pass on tcgen05 (mode 1): the first pass's budget P
// must fit one gathered 64-row tile.
bool parent_attn_tc_hvaq_ok(int dt, int D, int M0, int P);
size_t parent_attn_tc_table_bytes();
template <int DT>
int launch_parent_attn_tc(const PAArgs& a, void* exptab, cudaStream_t st);
// The bf16 exponential table of the tcgen05 kernels (DT(exp(-x)) for every
// bf16 x in [2^-9, 128], then 0), parent_attn_tc_table_bytes() bytes.
void launch_exp_table(void* tab, cudaStream_t st);
// tcgen05 child correction (bf16, fp16): same output as launch_correct_mma.
bool correct_tc_ok(int dt, int D, int C);
size_t correct_tc_desc_bytes(int G, int sel_stride, int C);
template <int DT>
int launch_correct_tc(const CorrArgs& a, const void* exptab, void* desc, cudaStream_t st);
// tcgen05 key assignment (parent argmin + child argmin), same outputs as the
// assign kernels of avq_quantize.cu.
bool assign_tc_ok(int dt, int D, int M0);
template <int DT>
int launch_assign_tc(const QuantizeArgs& a, cudaStream_t st);
// the child assignment of a launch_assign_tc pass, after the sort by parent
template <int DT>
int launch_child_bucket(const QuantizeArgs& a, const int* order, cudaStream_t st);
// Reads and clears the device fault record (stream-synchronous): the OR of
// the fault words of the tcgen05 kernel files.
int read_device_fault(int* code, cudaStream_t st);
int read_fault_assign(int* code, cudaStream_t st);
int read_fault_correct(int* code, cudaStream_t st);

// Dense softmax attention (avq_dense.cu): the reference's naive path.
template <int DT>
int launch_dense_attention(const void* q, Strides3 qs, const void* k, Strides3 ks, const void* v, Strides3 vs, int B,
                           int H, int T, int N, int D, const unsigned char* mask, const long long* mask_strides,
                           void* out, Strides3 os, cudaStream_t st);

// BCAR online codebook adaptation (avq_bcar.cu).
size_t bcar_workspace_bytes(int G, int M0, int C, int D);

// Dense attention on the tcgen05 parent-attention kernel (no mask; bf16 / fp16,
// D in {64, 128}, N <= 8192 keys, N % 8 == 0); AVQ_ERR_UNSUPPORTED otherwise.
template <int DT>
int launch_dense_tc(const void* q, Strides3 qs, const void* k, Strides3 ks, const void* v, Strides3 vs, int B, int H,
                    int T, int N, int D, float scale, void* out, Strides3 os, cudaStream_t st);

// Streaming VQ extend (avq_stream.cu).
int stream_max_head_dim();
size_t stream_workspace_bytes(int B, int H, int M0, int C);
template <int DT>
int launch_stream_extend(const void* keys, long long kstride, int B, int H, int M0, int C, int D, const void* parents,
                         const void* children, long long* pout, long long* cout_, long long* prec, long long* crec,
                         long long rec_stride, long long rec_size, long long* pcnt, long long* ccnt, void* pagg,
                         void* cagg, void* workspace, cudaStream_t st);
template <int DT>
int launch_bcar(const void* keys, Strides3 ks, const int* passign, const int* cassign, int B, int H, int S, int D,
                int M0, int C, float decay, const void* ch_in, void* ch_out, void* parents_out, void* workspace,
                cudaStream_t st);

// Codeword visibility bits under a causal (mask == nullptr) or user mask
// (avq_mask.cu).
int presence_words(int M0);
size_t presence_workspace_bytes(int sG, int M0);
int launch_presence(const int* passign, int B, int H, int S, int M0, int T, const unsigned char* mask,
                    const long long* mask_strides, int causal_offset, int sG, unsigned int* present, void* scratch,
                    cudaStream_t st);

// The mask bit of parent p for row (g, t) (all present when there is no mask).
__device__ __forceinline__ bool present_bit(const unsigned int* present, int W, long gt, int p) {
  return !present || ((present[gt * W + (p >> 5)] >> (p & 31)) & 1u);
}

template <int DT>
int launch_append(const AppendArgs& a, cudaStream_t st);
size_t append_workspace_bytes(int B, int H, int Tn);
// Decode step (one query per (b,h), one routing pass, no HVAQ): per-head
// logits on mma.sync, then one CTA per (b,h) for softmax, routing and the
// child correction (avq_decode_attn.cu).
bool decode_forward_ok(int dt, int T, int D, int M0, int C, int P, int passes, int hvaq);
size_t decode_work_bytes(int G, int M0, int P);
template <int DT>
int launch_decode_forward(const ForwardArgs& a, void* work, const void* exptab, int* sel, int sel_stride,
                          int* pass_cnt, float* importance, cudaStream_t st);
int launch_reduce_min(const int* v, int n, int* out, cudaStream_t st);

template <int DT>
int launch_prep_codebook(const float* parents32, const float* children32, int H, int M0, int C, int D,
                         void* parents_dt, void* children_dt, float* p_sq, float* c_sq, cudaStream_t st);
template <int DT>
int launch_quantize(const QuantizeArgs& a, cudaStream_t st);
size_t quantize_workspace_bytes(int G, int S, int M0);

template <int DT>
int launch_forward(const ForwardArgs& a, cudaStream_t st);
size_t forward_workspace_bytes(int dtype, int G, int T, int D, int M0, int C, int P, int passes, float decay, int hvaq);
bool forward_uses_mma(int dtype, int D, int M0, int C);
int selection_stride(int P, int passes, float decay);
void pass_budget_caps(int P, int passes, float decay, int* caps);

}  // namespace avq
