// plstm_abi.cu — the C ABI (include/plstm.h): validation, backend dispatch,
// workspace layout and the reference-named entry points.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "plstm_common.cuh"

namespace plstm {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

namespace {
std::atomic<int64_t> g_launches{0};
std::atomic<int> g_profile{0};
std::mutex g_prof_mu;
std::vector<std::pair<cudaEvent_t, cudaEvent_t>> g_prof_events;
thread_local cudaEvent_t t_prof_start = nullptr;
}  // namespace

void note_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void profile_begin(cudaStream_t s) {
  if (!g_profile.load(std::memory_order_relaxed)) return;
  cudaEvent_t e;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, s);
  t_prof_start = e;
}

void profile_end(cudaStream_t s) {
  if (t_prof_start == nullptr) return;
  cudaEvent_t e;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, s);
  std::lock_guard<std::mutex> g(g_prof_mu);
  g_prof_events.emplace_back(t_prof_start, e);
  t_prof_start = nullptr;
}

int32_t make_problem(const plstm_desc* d, Problem* p) {
  PLSTM_CHECK_ARG(d != nullptr, "descriptor is NULL");
  PLSTM_CHECK_ARG(d->batch >= 0, "batch must be >= 0");
  PLSTM_CHECK_ARG(d->seq_len >= 0, "seq_len must be >= 0");
  PLSTM_CHECK_ARG(d->input_size > 0, "input_size must be > 0");
  PLSTM_CHECK_ARG(d->hidden_size > 0 && d->hidden_size <= 4096, "hidden_size must be in [1, 4096]");
  PLSTM_CHECK_ARG(d->num_layers > 0 && d->num_layers <= 64, "num_layers must be in [1, 64]");
  PLSTM_CHECK_ARG(d->dtype == PLSTM_F32 || d->dtype == PLSTM_F16 || d->dtype == PLSTM_BF16,
                  "dtype must be PLSTM_F32, PLSTM_F16 or PLSTM_BF16");
  PLSTM_CHECK_ARG(d->w_layout >= PLSTM_W_NATIVE && d->w_layout <= PLSTM_W_KPAIR, "unknown w_layout");
  PLSTM_CHECK_ARG(d->backend >= PLSTM_BACKEND_AUTO && d->backend <= PLSTM_BACKEND_TC, "unknown backend");
  const int outs = ((d->flags & PLSTM_FLAG_OUT_SEQ) ? 1 : 0) + ((d->flags & PLSTM_FLAG_OUT_LAST) ? 1 : 0) +
                   ((d->flags & PLSTM_FLAG_NO_LINEAR) ? 1 : 0);
  PLSTM_CHECK_ARG(outs == 1, "exactly one of PLSTM_FLAG_OUT_SEQ, _OUT_LAST, _NO_LINEAR must be set");
  if (!(d->flags & PLSTM_FLAG_NO_LINEAR))
    PLSTM_CHECK_ARG(d->output_size > 0, "output_size must be > 0 with a Linear head");
  PLSTM_CHECK_ARG(d->timeout_ms >= 0, "timeout_ms must be >= 0");
  p->B = d->batch;
  p->T = d->seq_len;
  p->I = d->input_size;
  p->H = d->hidden_size;
  p->L = d->num_layers;
  p->O = (d->flags & PLSTM_FLAG_NO_LINEAR) ? 0 : d->output_size;
  p->dtype = d->dtype;
  p->flags = d->flags;
  p->timeout_ms = d->timeout_ms > 0 ? d->timeout_ms : default_timeout_ms();
  p->device = d->device;
  return PLSTM_OK;
}

// Bound of every inter-CTA wait when the descriptor leaves it 0: PLSTM_TIMEOUT_MS if set (a
// profiler that replays each launch dozens of times can stretch a step well past 2 s), else 2 s.
int32_t default_timeout_ms() {
  if (const char* e = std::getenv("PLSTM_TIMEOUT_MS")) {
    const long v = std::strtol(e, nullptr, 10);
    if (v > 0 && v <= 3600000) return (int32_t)v;
  }
  return 2000;
}

namespace {

// Picks the backend; fails if the caller forced one that cannot serve `p`.
int32_t pick_backend(const plstm_desc* d, const Problem& p, int* backend) {
  std::string why;
  const bool tc_ok = tc_supported(p, &why);
  if (d->backend == PLSTM_BACKEND_TC) {
    if (!tc_ok) {
      set_error("tensor-core backend cannot serve this problem: " + why);
      return PLSTM_ENOTSUP;
    }
    *backend = PLSTM_BACKEND_TC;
  } else if (d->backend == PLSTM_BACKEND_SIMT) {
    *backend = PLSTM_BACKEND_SIMT;
  } else {
    *backend = tc_ok ? PLSTM_BACKEND_TC : PLSTM_BACKEND_SIMT;
  }
  return PLSTM_OK;
}

size_t backend_ws(int backend, const Problem& p) {
  return backend == PLSTM_BACKEND_TC ? tc_workspace_size(p) : simt_workspace_size(p);
}

// Scratch plstm_forward_packed needs: the backend's, then (PLSTM_FLAG_DEDUPE)
// the row grouping and the distinct-row copies; a multiple of 256 bytes, so the
// packed image plstm_forward places after it stays aligned.
size_t forward_ws(int backend, const Problem& p) {
  const size_t inner = align_up(backend_ws(backend, p), 256);
  return (p.flags & PLSTM_FLAG_DEDUPE) ? align_up(inner + dedupe_scratch_size(p), 256) : inner;
}

struct BackendCtx {
  int backend;
  const void* packed;
};

int32_t run_backend(void* ctx, const Problem& q, const void* x, const int32_t* lengths, const void* h0,
                    const void* c0, void* out, void* h_n, void* c_n, void* ws, cudaStream_t s) {
  const BackendCtx* c = static_cast<const BackendCtx*>(ctx);
  return c->backend == PLSTM_BACKEND_TC ? tc_forward(q, c->packed, x, lengths, h0, c0, out, h_n, c_n, ws, s)
                                        : simt_forward(q, c->packed, x, lengths, h0, c0, out, h_n, c_n, ws, s);
}

int32_t finish(const Problem& p, void* ws, cudaStream_t s) {
  if (!(p.flags & PLSTM_FLAG_SYNC_CHECK)) return PLSTM_OK;
  int32_t st = 0, detail = 0;
  const int32_t rc = plstm_read_status(ws, s, &st, &detail);
  if (rc != PLSTM_OK) return rc;
  if (st == PLSTM_EBOUNDS) {
    set_error("device status " + std::to_string(st) + " (site " + std::to_string(detail) +
              "): the bounds-check build found an index outside its buffer");
    return st;
  }
  if (st != PLSTM_OK) {
    set_error("device status " + std::to_string(st) + " (cta " + std::to_string(detail >> 16) +
              ", step " + std::to_string(detail & 0xffff) + "): a bounded inter-CTA wait gave up");
    return st;
  }
  return PLSTM_OK;
}

}  // namespace
}  // namespace plstm

using namespace plstm;

extern "C" {

int32_t plstm_abi_version(void) { return PLSTM_ABI_VERSION; }

int64_t plstm_launch_count(void) { return g_launches.load(); }

int32_t plstm_profile(int32_t enable) {
  g_profile.store(enable != 0 ? 1 : 0);
  return PLSTM_OK;
}

int32_t plstm_profile_read(float* ms, int32_t* launches) {
  clear_error();
  PLSTM_CHECK_ARG(ms != nullptr, "ms is NULL");
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> evs;
  {
    std::lock_guard<std::mutex> g(g_prof_mu);
    evs.swap(g_prof_events);
  }
  float total = 0.0f;
  int32_t rc = PLSTM_OK;
  for (auto& pr : evs) {
    float v = 0.0f;
    if (rc == PLSTM_OK) {
      cudaError_t e = cudaEventSynchronize(pr.second);
      if (e == cudaSuccess) e = cudaEventElapsedTime(&v, pr.first, pr.second);
      if (e != cudaSuccess) {
        set_error(std::string("profile events: ") + cudaGetErrorString(e));
        rc = PLSTM_ECUDA;
      }
    }
    total += v;
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  *ms = total;
  if (launches != nullptr) *launches = (int32_t)evs.size();
  return rc;
}

const char* plstm_last_error(void) { return g_last_error.c_str(); }

int32_t plstm_select_backend(const plstm_desc* d) {
  Problem p;
  if (make_problem(d, &p) != PLSTM_OK) return -PLSTM_EINVAL;
  int b = 0;
  if (pick_backend(d, p, &b) != PLSTM_OK) return -PLSTM_ENOTSUP;
  return b;
}

int32_t plstm_packed_size(const plstm_desc* d, size_t* bytes) {
  clear_error();
  Problem p;
  int32_t rc = make_problem(d, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(bytes != nullptr, "bytes is NULL");
  int b = 0;
  if ((rc = pick_backend(d, p, &b)) != PLSTM_OK) return rc;
  *bytes = b == PLSTM_BACKEND_TC ? tc_packed_size(p) : simt_packed_size(p);
  return PLSTM_OK;
}

int32_t plstm_workspace_size(const plstm_desc* d, size_t* bytes) {
  clear_error();
  Problem p;
  int32_t rc = make_problem(d, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(bytes != nullptr, "bytes is NULL");
  int b = 0;
  if ((rc = pick_backend(d, p, &b)) != PLSTM_OK) return rc;
  *bytes = forward_ws(b, p);
  return PLSTM_OK;
}

static int32_t pack_impl(const plstm_desc* d, int ih_layout, int hh_layout, const void* const* w_ih,
                         const void* const* w_hh, const void* const* b_ih, const void* const* b_hh,
                         const void* w_lin, const void* b_lin, void* packed, size_t packed_bytes,
                         void* stream) {
  Problem p;
  int32_t rc = make_problem(d, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(w_ih != nullptr && w_hh != nullptr, "w_ih / w_hh arrays are NULL");
  for (int l = 0; l < p.L; ++l)
    PLSTM_CHECK_ARG(w_ih[l] != nullptr && w_hh[l] != nullptr, "a layer weight pointer is NULL");
  if (d->flags & PLSTM_FLAG_BIAS_SUMMED)
    PLSTM_CHECK_ARG(b_hh == nullptr, "PLSTM_FLAG_BIAS_SUMMED requires b_hh == NULL");
  if (p.has_linear()) PLSTM_CHECK_ARG(w_lin != nullptr, "w_lin is NULL");
  PLSTM_CHECK_ARG(packed != nullptr, "packed is NULL");
  PLSTM_CHECK_ARG(aligned16(packed), "packed must be 16-byte aligned");
  int b = 0;
  if ((rc = pick_backend(d, p, &b)) != PLSTM_OK) return rc;
  const size_t need = b == PLSTM_BACKEND_TC ? tc_packed_size(p) : simt_packed_size(p);
  if (packed_bytes < need) {
    set_error("packed buffer too small: need " + std::to_string(need) + " bytes");
    return PLSTM_EWORKSPACE;
  }
  DeviceGuard dev_guard;
  if ((rc = dev_guard.enter(p.device)) != PLSTM_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return b == PLSTM_BACKEND_TC
             ? tc_pack(p, ih_layout, hh_layout, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, packed, s)
             : simt_pack(p, ih_layout, hh_layout, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, packed, s);
}

int32_t plstm_pack(const plstm_desc* d, const void* const* w_ih, const void* const* w_hh,
                   const void* const* b_ih, const void* const* b_hh, const void* w_lin,
                   const void* b_lin, void* packed, size_t packed_bytes, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(d != nullptr, "descriptor is NULL");
  return pack_impl(d, d->w_layout, d->w_layout, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, packed,
                   packed_bytes, stream);
}

int32_t plstm_forward_packed(const plstm_desc* d, const void* packed, const void* x,
                             const int32_t* lengths, const void* h0, const void* c0, void* out,
                             void* h_n, void* c_n, void* workspace, size_t workspace_bytes,
                             void* stream) {
  clear_error();
  Problem p;
  int32_t rc = make_problem(d, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(packed != nullptr, "packed is NULL");
  PLSTM_CHECK_ARG(workspace != nullptr, "workspace is NULL");
  PLSTM_CHECK_ARG(aligned16(packed) && aligned16(workspace), "packed and workspace must be 16-byte aligned");
  PLSTM_CHECK_ARG(p.B == 0 || p.T == 0 || x != nullptr, "x is NULL");
  PLSTM_CHECK_ARG(p.B == 0 || out != nullptr, "out is NULL");
  PLSTM_CHECK_ARG((h0 == nullptr) == (c0 == nullptr), "h0 and c0 must both be given or both be NULL");
  int b = 0;
  if ((rc = pick_backend(d, p, &b)) != PLSTM_OK) return rc;
  const size_t need = forward_ws(b, p);
  if (workspace_bytes < need) {
    set_error("workspace too small: need " + std::to_string(need) + " bytes");
    return PLSTM_EWORKSPACE;
  }
  DeviceGuard dev_guard;
  if ((rc = dev_guard.enter(p.device)) != PLSTM_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((p.flags & PLSTM_FLAG_DEDUPE) && (rc = dedupe_stream_ok(s)) != PLSTM_OK) return rc;
  PLSTM_TRY_CUDA(cudaMemsetAsync(workspace, 0, kStatusBytes, s));
  if (p.B == 0) return PLSTM_OK;
  BackendCtx ctx = {b, packed};
  if ((p.flags & PLSTM_FLAG_DEDUPE) && p.B > 1 && p.T > 0)
    rc = dedupe_forward(p, DedupeInner{run_backend, &ctx}, x, lengths, h0, c0, out, h_n, c_n, workspace,
                        backend_ws(b, p), s);
  else
    rc = run_backend(&ctx, p, x, lengths, h0, c0, out, h_n, c_n, workspace, s);
  if (rc != PLSTM_OK) return rc;
  return finish(p, workspace, s);
}

static int32_t forward_impl(const plstm_desc* d, int ih_layout, int hh_layout, const void* x,
                            const void* const* w_ih, const void* const* w_hh,
                            const void* const* b_ih, const void* const* b_hh, const void* w_lin,
                            const void* b_lin, const int32_t* lengths, const void* h0,
                            const void* c0, void* out, void* h_n, void* c_n, void* workspace,
                            size_t workspace_bytes, void* stream) {
  size_t pk = 0, ws = 0;
  int32_t rc = plstm_packed_size(d, &pk);
  if (rc != PLSTM_OK) return rc;
  if ((rc = plstm_workspace_size(d, &ws)) != PLSTM_OK) return rc;
  pk = align_up(pk, 256);
  if (workspace == nullptr || workspace_bytes < pk + ws) {
    set_error("workspace too small: need " + std::to_string(pk + ws) + " bytes");
    return PLSTM_EWORKSPACE;
  }
  // Layout: [status + scratch of the forward][packed weights].
  char* base = static_cast<char*>(workspace);
  void* packed = base + ws;
  rc = pack_impl(d, ih_layout, hh_layout, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, packed, pk, stream);
  if (rc != PLSTM_OK) return rc;
  return plstm_forward_packed(d, packed, x, lengths, h0, c0, out, h_n, c_n, base, ws, stream);
}

int32_t plstm_forward(const plstm_desc* d, const void* x, const void* const* w_ih,
                      const void* const* w_hh, const void* const* b_ih, const void* const* b_hh,
                      const void* w_lin, const void* b_lin, const int32_t* lengths, const void* h0,
                      const void* c0, void* out, void* h_n, void* c_n, void* workspace,
                      size_t workspace_bytes, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(d != nullptr, "descriptor is NULL");
  return forward_impl(d, d->w_layout, d->w_layout, x, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, lengths,
                      h0, c0, out, h_n, c_n, workspace, workspace_bytes, stream);
}

int32_t plstm_unique_rows_workspace_size(const plstm_desc* d, size_t* bytes) {
  clear_error();
  Problem p;
  int32_t rc = make_problem(d, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(bytes != nullptr, "bytes is NULL");
  *bytes = unique_rows_scratch_size(p);
  return PLSTM_OK;
}

int32_t plstm_unique_rows(const plstm_desc* d, const void* x, const int32_t* lengths, const void* h0,
                          const void* c0, int32_t* row_map, int32_t* unique_index, int32_t* count,
                          void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  Problem p;
  int32_t rc = make_problem(d, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(count != nullptr, "count is NULL");
  PLSTM_CHECK_ARG(p.B == 0 || (row_map != nullptr && unique_index != nullptr), "row_map / unique_index is NULL");
  PLSTM_CHECK_ARG(p.B == 0 || p.T == 0 || x != nullptr, "x is NULL");
  PLSTM_CHECK_ARG((h0 == nullptr) == (c0 == nullptr), "h0 and c0 must both be given or both be NULL");
  PLSTM_CHECK_ARG(aligned16(workspace), "workspace must be 16-byte aligned");
  const size_t need = unique_rows_scratch_size(p);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("workspace too small: need " + std::to_string(need) + " bytes");
    return PLSTM_EWORKSPACE;
  }
  *count = 0;
  if (p.B == 0) return PLSTM_OK;
  DeviceGuard dev_guard;
  if ((rc = dev_guard.enter(p.device)) != PLSTM_OK) return rc;
  return unique_rows(p, x, lengths, h0, c0, row_map, unique_index, count, workspace,
                     static_cast<cudaStream_t>(stream));
}

int32_t plstm_read_status(const void* workspace, void* stream, int32_t* status, int32_t* detail) {
  PLSTM_CHECK_ARG(workspace != nullptr && status != nullptr, "NULL argument");
  int32_t host[2] = {0, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PLSTM_TRY_CUDA(cudaMemcpyAsync(host, workspace, sizeof(host), cudaMemcpyDeviceToHost, s));
  PLSTM_TRY_CUDA(cudaStreamSynchronize(s));
  PLSTM_TRY_CUDA(cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(host), s));
  *status = host[0];
  if (detail != nullptr) *detail = host[1];
  return PLSTM_OK;
}

// ---- persistent_lstm_hip_ext entry points -----------------------------------

static int32_t ref4_desc(int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
                         int32_t output_size, int32_t layout, plstm_desc* d) {
  std::memset(d, 0, sizeof(*d));
  d->batch = batch;
  d->seq_len = seq_len;
  d->input_size = input_size;
  d->hidden_size = hidden_size;
  d->num_layers = 4;
  d->output_size = output_size;
  d->dtype = PLSTM_F16;  // the reference's 4-layer kernels are f16-only (persistent_lstm_hip.cu:1697-1727)
  d->w_layout = layout;
  d->flags = PLSTM_FLAG_OUT_LAST | PLSTM_FLAG_BIAS_SUMMED;
  d->backend = PLSTM_BACKEND_AUTO;
  int dev = 0;
  cudaGetDevice(&dev);
  d->device = dev;
  return PLSTM_OK;
}

int32_t plstm_ref4_workspace_size(int32_t batch, int32_t seq_len, int32_t input_size,
                                  int32_t hidden_size, int32_t output_size, size_t* bytes) {
  plstm_desc d;
  ref4_desc(batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_NATIVE, &d);
  size_t pk = 0, ws = 0;
  int32_t rc = plstm_packed_size(&d, &pk);
  if (rc != PLSTM_OK) return rc;
  if ((rc = plstm_workspace_size(&d, &ws)) != PLSTM_OK) return rc;
  *bytes = align_up(pk, 256) + ws;
  return PLSTM_OK;
}

static int32_t ref4_forward(const void* x, int32_t batch, int32_t seq_len, int32_t input_size,
                            int32_t hidden_size, int32_t output_size, int32_t ih_layout,
                            int32_t hh_layout, const void* const* w_ih4, const void* const* w_hh4,
                            const void* const* bias4, const void* w_lin, const void* b_lin,
                            void* out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(w_ih4 != nullptr && w_hh4 != nullptr && bias4 != nullptr, "NULL weight array");
  plstm_desc d;
  ref4_desc(batch, seq_len, input_size, hidden_size, output_size, ih_layout, &d);
  return forward_impl(&d, ih_layout, hh_layout, x, w_ih4, w_hh4, bias4, nullptr, w_lin, b_lin,
                      nullptr, nullptr, nullptr, out, nullptr, nullptr, workspace, workspace_bytes,
                      stream);
}

int32_t plstm_persistent_lstm4_forward(const void* x, int32_t batch, int32_t seq_len,
                                       int32_t input_size, int32_t hidden_size,
                                       int32_t output_size, const void* const* w_ih4,
                                       const void* const* w_hh4, const void* const* bias4,
                                       const void* w_lin, const void* b_lin, void* out,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  return ref4_forward(x, batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_NATIVE,
                      PLSTM_W_NATIVE, w_ih4, w_hh4, bias4, w_lin, b_lin, out, workspace,
                      workspace_bytes, stream);
}

int32_t plstm_persistent_lstm4_forward_packed(const void* x, int32_t batch, int32_t seq_len,
                                              int32_t input_size, int32_t hidden_size,
                                              int32_t output_size, const void* const* w_ih4_t,
                                              const void* const* w_hh4_t, const void* const* bias4,
                                              const void* w_lin, const void* b_lin, void* out,
                                              void* workspace, size_t workspace_bytes,
                                              void* stream) {
  return ref4_forward(x, batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_TRANSPOSED,
                      PLSTM_W_TRANSPOSED, w_ih4_t, w_hh4_t, bias4, w_lin, b_lin, out, workspace,
                      workspace_bytes, stream);
}

int32_t plstm_persistent_lstm4_forward_interleaved(
    const void* x, int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
    int32_t output_size, const void* const* w_ih4_kpair, const void* const* w_hh4_kpair,
    const void* const* bias4, const void* w_lin, const void* b_lin, void* out, void* workspace,
    size_t workspace_bytes, void* stream) {
  return ref4_forward(x, batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_KPAIR,
                      PLSTM_W_KPAIR, w_ih4_kpair, w_hh4_kpair, bias4, w_lin, b_lin, out, workspace,
                      workspace_bytes, stream);
}

int32_t plstm_persistent_lstm4_forward_monolithic(
    const void* x, int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
    int32_t output_size, const void* const* w_ih4_kpair, const void* const* w_hh4_kpair,
    const void* const* bias4, const void* w_lin, const void* b_lin, void* out, void* workspace,
    size_t workspace_bytes, void* stream) {
  return ref4_forward(x, batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_KPAIR,
                      PLSTM_W_KPAIR, w_ih4_kpair, w_hh4_kpair, bias4, w_lin, b_lin, out, workspace,
                      workspace_bytes, stream);
}

int32_t plstm_persistent_lstm4_forward_projected(
    const void* x, int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
    int32_t output_size, const void* const* w_ih4, const void* const* w_hh4_kpair,
    const void* const* bias4, const void* w_lin, const void* b_lin, void* out, void* workspace,
    size_t workspace_bytes, void* stream) {
  return ref4_forward(x, batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_NATIVE,
                      PLSTM_W_KPAIR, w_ih4, w_hh4_kpair, bias4, w_lin, b_lin, out, workspace,
                      workspace_bytes, stream);
}

int32_t plstm_regressor_forward_generic(const void* x, int32_t batch, int32_t seq_len,
                                        int32_t input_size, int32_t hidden_size,
                                        int32_t num_layers, int32_t output_size,
                                        const void* const* w_ih, const void* const* w_hh,
                                        const void* const* bias, const void* w_lin,
                                        const void* b_lin, void* out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  plstm_desc d;
  ref4_desc(batch, seq_len, input_size, hidden_size, output_size, PLSTM_W_NATIVE, &d);
  d.num_layers = num_layers;
  return plstm_forward(&d, x, w_ih, w_hh, bias, nullptr, w_lin, b_lin, nullptr, nullptr, nullptr,
                       out, nullptr, nullptr, workspace, workspace_bytes, stream);
}

}  // extern "C"
