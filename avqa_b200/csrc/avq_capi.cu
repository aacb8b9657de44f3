// extern "C" entry points (include/avqa_b200.h): argument checks, dtype
// dispatch and error reporting around the kernel launchers.
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>

#include "../../include/avqa_b200.h"
#include "avq_kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int finish(int rc, const char* what) {
  if (rc == AVQ_OK) {
    const cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess) return fail(AVQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return AVQ_OK;
  }
  if (rc == AVQ_ERR_UNSUPPORTED) return fail(rc, "%s: unsupported size (D <= 256, C <= 8, M0 <= 8192, passes <= 8)", what);
  if (rc == AVQ_ERR_WORKSPACE) return fail(rc, "%s: workspace too small", what);
  const cudaError_t e = cudaGetLastError();
  return fail(rc, "%s: %s", what, cudaGetErrorString(e));
}

avq::Strides3 st3(const long long* s) { return avq::Strides3{(long)s[0], (long)s[1], (long)s[2]}; }

struct ProfRecord {
  const char* name;
  cudaEvent_t e0, e1;
};
std::mutex g_prof_mu;
std::vector<ProfRecord> g_prof;
bool g_prof_on = false;

}  // namespace

namespace avq {

ProfileScope::ProfileScope(const char* n, cudaStream_t s) : name(n), st(s), e0(nullptr), on(false) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof_on) return;
  if (cudaEventCreate(&e0) != cudaSuccess) return;
  cudaEventRecord(e0, st);
  on = true;
}

ProfileScope::~ProfileScope() {
  if (!on) return;
  cudaEvent_t e1;
  if (cudaEventCreate(&e1) != cudaSuccess) return;
  cudaEventRecord(e1, st);
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof.push_back({name, e0, e1});
}

}  // namespace avq

namespace {

bool bad_dtype(int dt) { return dt < 0 || dt > 2; }

// B * H (the number of (b,h) groups) must stay an int: every kernel indexes
// groups with int arithmetic.  Checked in 64 bits before any size is derived.
bool too_many_groups(int B, int H) { return (long long)B * (long long)H > (long long)INT_MAX; }

}  // namespace

extern "C" {

const char* avq_version(void) { return "avqa_b200 0.1.0 (sm_100a)"; }

int avq_last_error(char* buf, int len) {
  if (buf && len > 0) {
    std::strncpy(buf, g_last_error.c_str(), (size_t)len - 1);
    buf[len - 1] = 0;
  }
  return (int)g_last_error.size();
}

int avq_prepare_codebook(int dtype, const float* parents32, const float* children32, int H, int M0, int C, int D,
                         void* parents_dt, void* children_dt, float* p_sq, float* c_sq, void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_prepare_codebook: bad dtype %d", dtype);
  if (H <= 0 || M0 <= 0 || C <= 0 || D <= 0) return fail(AVQ_ERR_ARG, "avq_prepare_codebook: sizes must be > 0");
  if (!parents32 || !children32 || !parents_dt || !children_dt || !p_sq || !c_sq)
    return fail(AVQ_ERR_ARG, "avq_prepare_codebook: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  switch (dtype) {
    case 0: rc = avq::launch_prep_codebook<avq::DT_F32>(parents32, children32, H, M0, C, D, parents_dt, children_dt, p_sq, c_sq, st); break;
    case 1: rc = avq::launch_prep_codebook<avq::DT_BF16>(parents32, children32, H, M0, C, D, parents_dt, children_dt, p_sq, c_sq, st); break;
    default: rc = avq::launch_prep_codebook<avq::DT_F16>(parents32, children32, H, M0, C, D, parents_dt, children_dt, p_sq, c_sq, st); break;
  }
  return finish(rc, "avq_prepare_codebook");
}

size_t avq_quantize_workspace_size(int B, int H, int S, int M0) {
  if (B < 0 || H <= 0 || S < 0 || M0 <= 0 || too_many_groups(B, H)) return 0;
  return avq::quantize_workspace_bytes(B * H, S, M0);
}

int avq_quantize(int dtype, const void* keys, const long long* key_strides, const void* values,
                 const long long* value_strides, int B, int H, int S, int D, int M0, int C, const void* parents_dt,
                 const float* p_sq, const void* children_dt, const float* c_sq, int* passign, int* cassign,
                 void* pagg, void* cagg, float* pacc, float* cacc, int* pcnt, int* ccnt, int* nvalid,
                 int* gmin_valid, void* workspace, size_t workspace_bytes, void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_quantize: bad dtype %d", dtype);
  if (B < 0 || H <= 0 || S < 0 || D <= 0 || M0 <= 0 || C <= 0) return fail(AVQ_ERR_ARG, "avq_quantize: bad sizes");
  if (!key_strides || !value_strides || !parents_dt || !p_sq || !children_dt || !c_sq || !pagg || !cagg || !pcnt ||
      !ccnt || !nvalid)
    return fail(AVQ_ERR_ARG, "avq_quantize: null pointer");
  if (S > 0 && (!keys || !values || !passign || !cassign)) return fail(AVQ_ERR_ARG, "avq_quantize: null key pointer");
  if ((pacc == nullptr) != (cacc == nullptr)) return fail(AVQ_ERR_ARG, "avq_quantize: pacc and cacc go together");
  if (too_many_groups(B, H)) return fail(AVQ_ERR_ARG, "avq_quantize: B*H = %lld exceeds INT_MAX", (long long)B * H);
  const size_t need = avq::quantize_workspace_bytes(B * H, S, M0);
  if (workspace_bytes < need || (need && !workspace))
    return fail(AVQ_ERR_WORKSPACE, "avq_quantize: workspace %zu < %zu bytes", workspace_bytes, need);
  if (B == 0) return AVQ_OK;
  avq::QuantizeArgs a{keys, st3(key_strides), values, st3(value_strides), B, H, S, D, M0, C, parents_dt, p_sq,
                      children_dt, c_sq, passign, cassign, pagg, cagg, pacc, cacc, pcnt, ccnt, nvalid, gmin_valid,
                      workspace, workspace_bytes};
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  switch (dtype) {
    case 0: rc = avq::launch_quantize<avq::DT_F32>(a, st); break;
    case 1: rc = avq::launch_quantize<avq::DT_BF16>(a, st); break;
    default: rc = avq::launch_quantize<avq::DT_F16>(a, st); break;
  }
  return finish(rc, "avq_quantize");
}

int avq_selection_stride(int P, int passes, float pass_decay) {
  if (P <= 0 || passes <= 0 || passes > 8) return fail(AVQ_ERR_ARG, "avq_selection_stride: bad P/passes"), -1;
  return avq::selection_stride(P, passes, pass_decay);
}

size_t avq_forward_workspace_size(int dtype, int B, int H, int T, int D, int M0, int C, int P, int passes,
                                  float pass_decay, int hvaq) {
  if (bad_dtype(dtype) || P <= 0 || passes <= 0 || passes > 8 || B < 0 || H <= 0 || too_many_groups(B, H)) return 0;
  return avq::forward_workspace_bytes(dtype, B * H, T, D, M0, C, P, passes, pass_decay, hvaq);
}

int avq_dense_attention(int dtype, const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                        const void* v, const long long* v_strides, int B, int H, int T, int N, int D,
                        const unsigned char* mask, const long long* mask_strides, void* out,
                        const long long* out_strides, void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_dense_attention: bad dtype %d", dtype);
  if (B < 0 || H <= 0 || T < 0 || N < 0 || D <= 0) return fail(AVQ_ERR_ARG, "avq_dense_attention: bad sizes");
  if (too_many_groups(B, H)) return fail(AVQ_ERR_ARG, "avq_dense_attention: B*H exceeds INT_MAX");
  if (!q_strides || !k_strides || !v_strides || !out_strides || (mask && !mask_strides) ||
      ((long long)B * T > 0 && (!q || !out)) || ((long long)B * N > 0 && (!k || !v)))
    return fail(AVQ_ERR_ARG, "avq_dense_attention: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  switch (dtype) {
    case 0: rc = avq::launch_dense_attention<avq::DT_F32>(q, st3(q_strides), k, st3(k_strides), v, st3(v_strides), B, H, T, N, D, mask, mask_strides, out, st3(out_strides), st); break;
    case 1: rc = avq::launch_dense_attention<avq::DT_BF16>(q, st3(q_strides), k, st3(k_strides), v, st3(v_strides), B, H, T, N, D, mask, mask_strides, out, st3(out_strides), st); break;
    default: rc = avq::launch_dense_attention<avq::DT_F16>(q, st3(q_strides), k, st3(k_strides), v, st3(v_strides), B, H, T, N, D, mask, mask_strides, out, st3(out_strides), st); break;
  }
  return finish(rc, "avq_dense_attention");
}

size_t avq_bcar_workspace_size(int B, int H, int M0, int C, int D) {
  if (B < 0 || H <= 0 || M0 <= 0 || C <= 0 || D <= 0 || too_many_groups(B, H)) return 0;
  return avq::bcar_workspace_bytes(B * H, M0, C, D);
}

int avq_bcar_update(int dtype, const void* keys, const long long* key_strides, const int* passign, const int* cassign,
                    int B, int H, int S, int D, int M0, int C, float decay, const void* children_in, void* children_out,
                    void* parents_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_bcar_update: bad dtype %d", dtype);
  if (B <= 0 || H <= 0 || S < 0 || D <= 0 || M0 <= 0 || C <= 0) return fail(AVQ_ERR_ARG, "avq_bcar_update: bad sizes");
  if (too_many_groups(B, H)) return fail(AVQ_ERR_ARG, "avq_bcar_update: B*H exceeds INT_MAX");
  if (!(decay >= 0.f && decay < 1.f))
    return fail(AVQ_ERR_ARG, "avq_bcar_update: decay must be in [0, 1), got %g", (double)decay);
  if (!key_strides || !children_in || !children_out || !parents_out || (S > 0 && (!keys || !passign || !cassign)))
    return fail(AVQ_ERR_ARG, "avq_bcar_update: null pointer");
  if (children_out == children_in)
    return fail(AVQ_ERR_ARG, "avq_bcar_update: children_out must not alias children_in");
  const size_t need = avq::bcar_workspace_bytes(B * H, M0, C, D);
  if (workspace_bytes < need || !workspace)
    return fail(AVQ_ERR_WORKSPACE, "avq_bcar_update: workspace %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  switch (dtype) {
    case 0: rc = avq::launch_bcar<avq::DT_F32>(keys, st3(key_strides), passign, cassign, B, H, S, D, M0, C, decay, children_in, children_out, parents_out, workspace, st); break;
    case 1: rc = avq::launch_bcar<avq::DT_BF16>(keys, st3(key_strides), passign, cassign, B, H, S, D, M0, C, decay, children_in, children_out, parents_out, workspace, st); break;
    default: rc = avq::launch_bcar<avq::DT_F16>(keys, st3(key_strides), passign, cassign, B, H, S, D, M0, C, decay, children_in, children_out, parents_out, workspace, st); break;
  }
  return finish(rc, "avq_bcar_update");
}

size_t avq_stream_workspace_size(int B, int H, int M0, int C) {
  if (B < 0 || H <= 0 || M0 <= 0 || C <= 0 || too_many_groups(B, H) || (long long)H * M0 * C > INT_MAX) return 0;
  return avq::stream_workspace_bytes(B, H, M0, C);
}

int avq_stream_extend(int dtype, const void* keys, long long key_row_stride, int B, int H, int M0, int C, int D,
                      const void* parents, const void* children, long long* parent_out, long long* child_out,
                      long long* parent_record, long long* child_record, long long record_stride,
                      long long record_size, long long* parent_counts, long long* child_counts,
                      void* parent_aggregates, void* child_aggregates, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_stream_extend: bad dtype %d", dtype);
  if (B < 0 || H <= 0 || M0 <= 0 || C <= 0 || D <= 0) return fail(AVQ_ERR_ARG, "avq_stream_extend: bad sizes");
  if (too_many_groups(B, H) || (long long)H * M0 * C > INT_MAX)
    return fail(AVQ_ERR_ARG, "avq_stream_extend: B*H or H*M0*C exceeds INT_MAX");
  if (D > avq::stream_max_head_dim())
    return fail(AVQ_ERR_UNSUPPORTED, "avq_stream_extend: head_dim %d > %d", D, avq::stream_max_head_dim());
  if (B == 0) return AVQ_OK;
  if (!keys || !parents || !children || !parent_out || !child_out || !parent_counts || !child_counts ||
      !parent_aggregates || !child_aggregates || (!parent_record) != (!child_record))
    return fail(AVQ_ERR_ARG, "avq_stream_extend: null pointer");
  if (key_row_stride < D) return fail(AVQ_ERR_ARG, "avq_stream_extend: key row stride %lld < D", key_row_stride);
  if (parent_record && (record_size < 0 || record_stride < record_size + B))
    return fail(AVQ_ERR_ARG, "avq_stream_extend: record stride %lld < size %lld + B %d", record_stride,
                record_size, B);
  const size_t need = avq::stream_workspace_bytes(B, H, M0, C);
  if (workspace_bytes < need || !workspace)
    return fail(AVQ_ERR_WORKSPACE, "avq_stream_extend: workspace %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
#define AVQ_STREAM_CALL(DT)                                                                                      \
  avq::launch_stream_extend<DT>(keys, key_row_stride, B, H, M0, C, D, parents, children, parent_out, child_out, \
                                parent_record, child_record, record_stride, record_size, parent_counts,          \
                                child_counts, parent_aggregates, child_aggregates, workspace, st)
  switch (dtype) {
    case 0: rc = AVQ_STREAM_CALL(avq::DT_F32); break;
    case 1: rc = AVQ_STREAM_CALL(avq::DT_BF16); break;
    default: rc = AVQ_STREAM_CALL(avq::DT_F16); break;
  }
#undef AVQ_STREAM_CALL
  return finish(rc, "avq_stream_extend");
}

int avq_presence_words(int M0) { return M0 > 0 ? avq::presence_words(M0) : 0; }

size_t avq_presence_workspace_size(int H, int M0, int state_batch) {
  if (H <= 0 || M0 <= 0 || state_batch <= 0 || too_many_groups(state_batch, H)) return 0;
  return avq::presence_workspace_bytes(state_batch * H, M0);
}

int avq_codeword_presence(const int* passign, int B, int H, int S, int M0, int T, int state_batch,
                          const unsigned char* mask, const long long* mask_strides, int causal_offset,
                          unsigned int* present, void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || H <= 0 || S < 0 || M0 <= 0 || T < 0 || M0 > 8192)
    return fail(AVQ_ERR_ARG, "avq_codeword_presence: bad sizes");
  if (too_many_groups(B, H)) return fail(AVQ_ERR_ARG, "avq_codeword_presence: B*H exceeds INT_MAX");
  if (state_batch != B && state_batch != 1)
    return fail(AVQ_ERR_ARG, "avq_codeword_presence: state_batch must be B (%d) or 1, got %d", B, state_batch);
  if (!present || (S > 0 && !passign) || (mask && !mask_strides))
    return fail(AVQ_ERR_ARG, "avq_codeword_presence: null pointer");
  const size_t need = avq::presence_workspace_bytes(state_batch * H, M0);
  if (!mask && (workspace_bytes < need || !workspace))
    return fail(AVQ_ERR_WORKSPACE, "avq_codeword_presence: workspace %zu < %zu bytes", workspace_bytes, need);
  return finish(avq::launch_presence(passign, B, H, S, M0, T, mask, mask_strides, causal_offset, state_batch * H,
                                     present, workspace, (cudaStream_t)stream),
                "avq_codeword_presence");
}

int avq_forward(int dtype, const void* q, const long long* q_strides, int B, int H, int T, int D, int M0, int C,
                const void* parents_dt, const void* children_dt, const void* pagg, const void* cagg, const int* pcnt,
                const int* ccnt, int state_batch, const int* min_valid, void* min_valid_ready,
                const unsigned int* present, int P, int passes, float pass_decay, int hvaq, float beta0,
                float alpha, float* out, const long long* out_strides, float* importance_out, int* selected_out,
                int* pass_counts_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_forward: bad dtype %d", dtype);
  if (B < 0 || H <= 0 || T < 0 || D <= 0 || M0 <= 0 || C <= 0) return fail(AVQ_ERR_ARG, "avq_forward: bad sizes");
  if (state_batch != B && state_batch != 1)
    return fail(AVQ_ERR_ARG, "avq_forward: state_batch must be B (%d) or 1, got %d", B, state_batch);
  if (P <= 0) return fail(AVQ_ERR_ARG, "avq_forward: budget must be > 0, got %d", P);
  if (P > M0) return fail(AVQ_ERR_ARG, "avq_forward: budget (%d) exceeds number of parents (%d)", P, M0);
  if (passes <= 0 || passes > 8) return fail(AVQ_ERR_ARG, "avq_forward: passes must be in [1, 8], got %d", passes);
  if (passes > 1 && !(pass_decay > 0.f && pass_decay <= 1.f))
    return fail(AVQ_ERR_ARG, "avq_forward: decay must be in (0, 1], got %g", (double)pass_decay);
  if (hvaq < 0 || hvaq > 2) return fail(AVQ_ERR_ARG, "avq_forward: hvaq must be 0, 1 or 2");
  if (hvaq && !(beta0 > 0.f)) return fail(AVQ_ERR_ARG, "avq_forward: beta_init must be > 0");
  if (!q_strides || !out_strides || !parents_dt || !children_dt || !pagg || !cagg || !pcnt || !ccnt || !min_valid)
    return fail(AVQ_ERR_ARG, "avq_forward: null pointer");
  if (too_many_groups(B, H)) return fail(AVQ_ERR_ARG, "avq_forward: B*H = %lld exceeds INT_MAX", (long long)B * H);
  if ((long long)B * T > 0 && (!q || !out)) return fail(AVQ_ERR_ARG, "avq_forward: null q/out");
  const size_t need = avq::forward_workspace_bytes(dtype, B * H, T, D, M0, C, P, passes, pass_decay, hvaq);
  if (workspace_bytes < need || !workspace)
    return fail(AVQ_ERR_WORKSPACE, "avq_forward: workspace %zu < %zu bytes", workspace_bytes, need);
  avq::ForwardArgs a{q, st3(q_strides), B, H, T, D, M0, C, parents_dt, children_dt, pagg, cagg, pcnt, ccnt, min_valid,
                     P, passes, pass_decay, hvaq, beta0, alpha, out, st3(out_strides), importance_out, selected_out,
                     pass_counts_out, workspace, workspace_bytes, state_batch * H, min_valid_ready, present};
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  switch (dtype) {
    case 0: rc = avq::launch_forward<avq::DT_F32>(a, st); break;
    case 1: rc = avq::launch_forward<avq::DT_BF16>(a, st); break;
    default: rc = avq::launch_forward<avq::DT_F16>(a, st); break;
  }
  return finish(rc, "avq_forward");
}

size_t avq_append_workspace_size(int B, int H, int Tn) {
  if (B < 0 || H <= 0 || Tn < 0 || too_many_groups(B, H)) return 0;
  return avq::append_workspace_bytes(B, H, Tn);
}

int avq_append(int dtype, const void* k, const long long* k_strides, const void* v, const long long* v_strides,
               int B, int H, int Tn, int D, int M0, int C, const void* parents_dt, const float* p_sq,
               const void* children_dt, const float* c_sq, float* pacc, float* cacc, void* pagg, void* cagg,
               int* pcnt, int* ccnt, int* nvalid, void* kpage, void* vpage, const long long* page_strides, int slot0,
               void* workspace, size_t workspace_bytes, void* stream) {
  if (bad_dtype(dtype)) return fail(AVQ_ERR_ARG, "avq_append: bad dtype %d", dtype);
  if (B < 0 || H <= 0 || Tn < 0 || D <= 0 || M0 <= 0 || C <= 0) return fail(AVQ_ERR_ARG, "avq_append: bad sizes");
  if (!k || !v || !k_strides || !v_strides || !parents_dt || !p_sq || !children_dt || !c_sq || !pacc || !cacc ||
      !pagg || !cagg || !pcnt || !ccnt || !nvalid)
    return fail(AVQ_ERR_ARG, "avq_append: null pointer");
  if ((kpage == nullptr) != (vpage == nullptr) || (kpage && !page_strides))
    return fail(AVQ_ERR_ARG, "avq_append: kpage, vpage and page_strides go together");
  if (too_many_groups(B, H)) return fail(AVQ_ERR_ARG, "avq_append: B*H = %lld exceeds INT_MAX", (long long)B * H);
  if (workspace_bytes < avq::append_workspace_bytes(B, H, Tn) || !workspace)
    return fail(AVQ_ERR_WORKSPACE, "avq_append: workspace %zu < %zu bytes", workspace_bytes,
                avq::append_workspace_bytes(B, H, Tn));
  avq::AppendArgs a{k, st3(k_strides), v, st3(v_strides), B, H, Tn, D, M0, C, parents_dt, p_sq, children_dt, c_sq,
                    pacc, cacc, pagg, cagg, pcnt, ccnt, nvalid, kpage, vpage,
                    kpage ? st3(page_strides) : avq::Strides3{0, 0, 0}, slot0, workspace, workspace_bytes};
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  switch (dtype) {
    case 0: rc = avq::launch_append<avq::DT_F32>(a, st); break;
    case 1: rc = avq::launch_append<avq::DT_BF16>(a, st); break;
    default: rc = avq::launch_append<avq::DT_F16>(a, st); break;
  }
  return finish(rc, "avq_append");
}

int avq_profile_begin(void) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& r : g_prof) {
    cudaEventDestroy(r.e0);
    cudaEventDestroy(r.e1);
  }
  g_prof.clear();
  g_prof_on = true;
  return AVQ_OK;
}

int avq_profile_end(char* names, int names_len, float* total_ms, int* launches, int max_kernels) {
  std::vector<ProfRecord> recs;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_on = false;
    recs.swap(g_prof);
  }
  std::map<std::string, std::pair<double, int>> agg;
  int rc = AVQ_OK;
  for (auto& r : recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.e1) != cudaSuccess || cudaEventElapsedTime(&ms, r.e0, r.e1) != cudaSuccess)
      rc = fail(AVQ_ERR_CUDA, "avq_profile_end: %s", cudaGetErrorString(cudaGetLastError()));
    auto& a = agg[r.name];
    a.first += ms;
    a.second += 1;
    cudaEventDestroy(r.e0);
    cudaEventDestroy(r.e1);
  }
  std::string joined;
  int k = 0;
  for (auto& kv : agg) {
    if (k >= max_kernels) break;
    if (total_ms) total_ms[k] = (float)kv.second.first;
    if (launches) launches[k] = kv.second.second;
    joined += kv.first + "\n";
    ++k;
  }
  if (names && names_len > 0) {
    std::strncpy(names, joined.c_str(), (size_t)names_len - 1);
    names[names_len - 1] = 0;
  }
  return rc == AVQ_OK ? k : -1;
}

int avq_reduce_min(const int* v, int n, int* out, void* stream) {
  if (!v || !out || n <= 0) return fail(AVQ_ERR_ARG, "avq_reduce_min: bad arguments");
  return finish(avq::launch_reduce_min(v, n, out, (cudaStream_t)stream), "avq_reduce_min");
}

int avq_device_fault(int* code, void* stream) {
  if (!code) return fail(AVQ_ERR_ARG, "avq_device_fault: null pointer");
  if (avq::read_device_fault(code, (cudaStream_t)stream) != AVQ_OK)
    return fail(AVQ_ERR_CUDA, "avq_device_fault: %s", cudaGetErrorString(cudaGetLastError()));
  return AVQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// avq_quantize_noalloc: the quantizer with its scratch in a fixed device array.
//
// It exists for hosts that may not allocate device memory while they run: a
// serving runtime that carved the whole GPU into its own pool at start-up, or
// a cgo/JNI host that has no device allocator to call.  Such a host cannot
// hand avq_quantize a workspace, and a cudaMalloc inside the library would
// either fail or eat into memory the pool has promised elsewhere (and the
// matching cudaFree would synchronize the whole device).  So the scratch is a
// file-scope __device__ array: it comes with the library's device code, one
// copy per device, and costs AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES of each
// device's memory once the code is loaded there.
//
// Because every call on a device uses the same array, two calls that run at
// the same time on one device corrupt each other's bucket order; callers
// keep them in order on one stream.  No byte of the array needs a known
// starting value: the histogram kernel writes all M0 bins of every segment
// (or a memset zeroes them when S == 0), the scan writes every offset and the
// scatter writes every key position, and the aggregation's work counter is
// zeroed by a memset, before anything reads them.

namespace {

__device__ __align__(256) unsigned char g_quantize_scratch[AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES];

// The array's device address belongs to the CUDA context that loaded the
// library's device code: one address per context, so the cache is keyed by the
// context current at the call (the device's primary context for runtime-API
// hosts; the host's own context for a driver-API host).
struct NoallocEntry {
  void* ctx;
  void* scratch;
};
constexpr int kNoallocMaxContexts = 64;
std::mutex g_noalloc_mu;
NoallocEntry g_noalloc[kNoallocMaxContexts] = {};
int g_noalloc_n = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The current context, through the runtime's driver entry point (the library
// links only the runtime); *ctx is null when none is current yet.
int current_context(void** ctx) {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  if (!fn) return fail(AVQ_ERR_CUDA, "avq_quantize_noalloc: cuCtxGetCurrent is unavailable");
  CUcontext c = nullptr;
  if (fn(&c) != CUDA_SUCCESS) return fail(AVQ_ERR_CUDA, "avq_quantize_noalloc: cuCtxGetCurrent failed");
  *ctx = c;
  return AVQ_OK;
}

// Device address of the scratch array in the current context; looked up once
// per context, with that context current.
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);  // also makes the device's primary context current if none is
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(AVQ_ERR_CUDA, "avq_quantize_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  }
  void* ctx = nullptr;
  int rc = current_context(&ctx);
  if (rc != AVQ_OK) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (ctx) {
    for (int i = 0; i < g_noalloc_n; ++i)
      if (g_noalloc[i].ctx == ctx) {
        *out = g_noalloc[i].scratch;
        return AVQ_OK;
      }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_quantize_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    return fail(AVQ_ERR_CUDA, "avq_quantize_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                cudaGetErrorString(e));
  }
  if (!ctx) {  // the lookup above created the primary context: key by it from now on
    if ((rc = current_context(&ctx)) != AVQ_OK) return rc;
  }
  if (ctx && g_noalloc_n < kNoallocMaxContexts) g_noalloc[g_noalloc_n++] = {ctx, p};
  *out = p;
  return AVQ_OK;
}

}  // namespace

extern "C" int avq_quantize_noalloc(int dtype, const void* keys, const long long* key_strides, const void* values,
                                    const long long* value_strides, int B, int H, int S, int D, int M0, int C,
                                    const void* parents_dt, const float* p_sq, const void* children_dt,
                                    const float* c_sq, int* passign, int* cassign, void* pagg, void* cagg,
                                    float* pacc, float* cacc, int* pcnt, int* ccnt, int* nvalid, int* gmin_valid,
                                    void* stream) {
  // The size check comes first so that an oversized request touches no device.
  if (B < 0 || H <= 0 || S < 0 || M0 <= 0) return fail(AVQ_ERR_ARG, "avq_quantize_noalloc: bad sizes");
  if (too_many_groups(B, H))
    return fail(AVQ_ERR_ARG, "avq_quantize_noalloc: B*H = %lld exceeds INT_MAX", (long long)B * H);
  const size_t need = avq::quantize_workspace_bytes(B * H, S, M0);
  if (need > AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES)
    return fail(AVQ_ERR_WORKSPACE,
                "avq_quantize_noalloc: B=%d H=%d S=%d M0=%d needs %zu scratch bytes but the fixed array holds %zu; "
                "call avq_quantize with a workspace instead",
                B, H, S, M0, need, (size_t)AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != AVQ_OK) return rc;
  return avq_quantize(dtype, keys, key_strides, values, value_strides, B, H, S, D, M0, C, parents_dt, p_sq,
                      children_dt, c_sq, passign, cassign, pagg, cagg, pacc, cacc, pcnt, ccnt, nvalid, gmin_valid,
                      scratch, AVQ_QUANTIZE_NOALLOC_SCRATCH_BYTES, stream);
}
