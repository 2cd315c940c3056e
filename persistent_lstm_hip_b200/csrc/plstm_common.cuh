// plstm_common.cuh — shared definitions of the B200 LSTM + Linear library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/plstm.h"

namespace plstm {

// ---- error reporting -------------------------------------------------------
// Thread-local message of the last failure; plstm_last_error() returns it.
void set_error(const std::string& msg);
void clear_error();

struct Error {
  int32_t code;
  std::string msg;
};

#define PLSTM_TRY_CUDA(expr)                                                          \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    if (_e != cudaSuccess) {                                                          \
      ::plstm::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));         \
      return PLSTM_ECUDA;                                                             \
    }                                                                                 \
  } while (0)

#define PLSTM_CHECK_ARG(cond, msg)           \
  do {                                       \
    if (!(cond)) {                           \
      ::plstm::set_error(std::string(msg));  \
      return PLSTM_EINVAL;                   \
    }                                        \
  } while (0)

// ---- instrumentation ----------------------------------------------------------
// Counts every kernel launch of the library (plstm_launch_count).
void note_launches(int n);
// Records the start / end of the dominant (recurrent) kernel when profiling is on.
void profile_begin(cudaStream_t s);
void profile_end(cudaStream_t s);

// ---- workspace status block ------------------------------------------------
// The first kStatusBytes of every workspace hold the device status the
// kernels write when a bounded wait gives up: word 0 = PLSTM_* code (0 = ok),
// word 1 = detail (cta << 16 | step & 0xffff) of the first failure.
constexpr size_t kStatusBytes = 256;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// Caller buffers are read with 16-byte vector loads and bulk copies.
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline size_t dtype_size(int32_t dt) { return dt == PLSTM_F32 ? 4 : 2; }

// Makes a device current for the lifetime of the guard and puts the caller's
// device back on every return path, so that no entry point leaves the calling
// thread on another device.
class DeviceGuard {
 public:
  DeviceGuard() = default;
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
  ~DeviceGuard() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }
  int32_t enter(int dev) {
    int cur = -1;
    PLSTM_TRY_CUDA(cudaGetDevice(&cur));
    if (cur != dev) {
      PLSTM_TRY_CUDA(cudaSetDevice(dev));
      prev_ = cur;
    }
    return PLSTM_OK;
  }

 private:
  int prev_ = -1;
};

// ---- element conversion ----------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Gate nonlinearities, written with CUDA's accurate expf / tanhf (the
// reference computes sigmoid as 1 / (1 + expf(-x)) and tanh with tanhf,
// persistent_lstm_hip.cu:96-98 and :316-324).
__device__ __forceinline__ float sigmoid_acc(float v) { return 1.0f / (1.0f + expf(-v)); }
__device__ __forceinline__ float tanh_acc(float v) { return tanhf(v); }

// Records the first failure in the workspace status block.
__device__ __forceinline__ void report_status(int* status, int code, int detail) {
  if (status != nullptr && atomicCAS(status, 0, code) == 0) status[1] = detail;
}

// Checked accesses of the bounds-check build (compiled with -DPLSTM_BOUNDS_CHECK, the
// library lib/libplstm_bc.so): each checked site tests its index against its buffer's
// extent; a failure records PLSTM_EBOUNDS with the site number as the detail word and the
// caller skips the access instead of faulting.  In the normal build the test is compiled out.
#ifdef PLSTM_BOUNDS_CHECK
__device__ __forceinline__ bool bc_ok(int* status, bool ok, int site) {
  if (!ok) report_status(status, PLSTM_EBOUNDS, site);
  return ok;
}
#else
__device__ __forceinline__ bool bc_ok(int*, bool, int) { return true; }
#endif

// ---- entry points implemented per backend ---------------------------------
struct Problem {
  int B, T, I, H, L, O;
  int dtype;
  int flags;
  int timeout_ms;
  int device;
  // Batch size that chooses between kernels whose per-row arithmetic differs (-1: B).  The
  // deduplicated forward runs the distinct rows with the full batch's value, so that its
  // results stay bit-identical to the full forward's.
  int route_B = -1;
  int route_batch() const { return route_B >= 0 ? route_B : B; }
  bool has_linear() const { return (flags & PLSTM_FLAG_NO_LINEAR) == 0; }
  bool out_seq() const { return (flags & PLSTM_FLAG_OUT_SEQ) != 0; }
  bool out_last() const { return (flags & PLSTM_FLAG_OUT_LAST) != 0; }
};

// Validates a descriptor and fills the Problem every backend reads (plstm_abi.cu);
// PLSTM_EINVAL with the message set on a bad field.
int32_t make_problem(const plstm_desc* d, Problem* p);
// Default bound of the inter-CTA waits: PLSTM_TIMEOUT_MS, else 2000 ms.
int32_t default_timeout_ms();

// Generic layer-sequential FFMA backend (any shape, f32/f16/bf16).
size_t simt_packed_size(const Problem& p);
size_t simt_workspace_size(const Problem& p);
int32_t simt_pack(const Problem& p, int ih_layout, int hh_layout, const void* const* w_ih, const void* const* w_hh,
                  const void* const* b_ih, const void* const* b_hh, const void* w_lin,
                  const void* b_lin, void* packed, cudaStream_t s);
int32_t simt_forward(const Problem& p, const void* packed, const void* x, const int32_t* lengths,
                     const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                     cudaStream_t s);

// tcgen05 cluster wavefront backend (H = 128, L <= 8, I <= 128, O <= 32, f16/bf16).
bool tc_supported(const Problem& p, std::string* why);
size_t tc_packed_size(const Problem& p);
size_t tc_workspace_size(const Problem& p);
int32_t tc_pack(const Problem& p, int ih_layout, int hh_layout, const void* const* w_ih, const void* const* w_hh,
                const void* const* b_ih, const void* const* b_hh, const void* w_lin,
                const void* b_lin, void* packed, cudaStream_t s);
int32_t tc_forward(const Problem& p, const void* packed, const void* x, const int32_t* lengths,
                   const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                   cudaStream_t s);

// Tile row order shared by the tensor-core backends: perm[tiles * N] = batch row of
// each tile row (-1 = padding), tile_len[tiles] = steps of each tile.  Uniform
// lengths keep batch order; variable lengths sort rows by length, longest first
// (hist / sorted: (T + 1) and B int32 scratch words).
int32_t tc_make_perm(const Problem& p, int N, int tiles, const int32_t* lengths, int32_t* perm, int32_t* tile_len,
                     int32_t* hist, int32_t* sorted, cudaStream_t s);

// x[B][T][I] (I <= kx) -> xp[tiles][T][N rows x kx] 16-bit K-major core matrices
// (8 rows x 16 bytes; K groups 128 bytes apart, 8-row groups kx * 16 bytes apart), rows
// in tile order, zero for padding rows and columns I..kx-1.  kx: multiple of 16.  With
// `choice`, the launch packs only if *choice == N (device-side choice of the tile height).
int32_t tc_xpack(const Problem& p, int N, int tiles, const void* x, const int32_t* perm, uint8_t* xp, int kx,
                 cudaStream_t s, const int* choice = nullptr);

// tcgen05 layer-sequential backend (plstm_tcl.cu) for any H <= 512 (zero-padded to a multiple
// of 64), L <= 16, I <= 128: per layer a projection GEMM and a cluster-wide recurrence; the tc_* entry
// points above forward every shape outside the H = 128 wavefront kernel's envelope to it.
bool tcl_supported(const Problem& p, std::string* why);
size_t tcl_packed_size(const Problem& p);
size_t tcl_workspace_size(const Problem& p);
int32_t tcl_pack(const Problem& p, int ih_layout, int hh_layout, const void* const* w_ih, const void* const* w_hh,
                 const void* const* b_ih, const void* const* b_hh, const void* w_lin, const void* b_lin,
                 void* packed, cudaStream_t s);
int32_t tcl_forward(const Problem& p, const void* packed, const void* x, const int32_t* lengths, const void* h0,
                    const void* c0, void* out, void* h_n, void* c_n, void* ws, cudaStream_t s);

// Duplicate-row elimination (plstm_dedupe.cu).  `inner.run` is the backend
// forward the distinct rows go through (Problem q: batch = distinct count).
struct DedupeInner {
  int32_t (*run)(void* ctx, const Problem& q, const void* x, const int32_t* lengths, const void* h0,
                 const void* c0, void* out, void* h_n, void* c_n, void* ws, cudaStream_t s);
  void* ctx;
};
int32_t dedupe_stream_ok(cudaStream_t s);  // PLSTM_EINVAL (message set) while `s` is capturing
size_t unique_rows_scratch_size(const Problem& p);
size_t dedupe_scratch_size(const Problem& p);
int32_t unique_rows(const Problem& p, const void* x, const int32_t* lengths, const void* h0, const void* c0,
                    int* row_map, int* unique_index, int* count, void* scratch, cudaStream_t s);
// ws = [inner_ws_bytes of backend scratch, 256-aligned][dedupe_scratch_size(p)].
int32_t dedupe_forward(const Problem& p, const DedupeInner& inner, const void* x, const int32_t* lengths,
                       const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                       size_t inner_ws_bytes, cudaStream_t s);

// Hidden update (plstm_hidden_update): recurrence over precomputed input projections.
struct HuProblem {
  int B, T, H, dtype, flags, w_layout, device;
  bool seq_major() const { return (flags & PLSTM_HU_SEQ_MAJOR) != 0; }
  bool write_seq() const { return (flags & PLSTM_HU_WRITE_SEQUENCE) != 0; }
};
bool tcl_hu_supported(const HuProblem& p);
size_t tcl_hu_workspace_size(const HuProblem& p);
int32_t tcl_hidden_update(const HuProblem& p, const void* gate_proj, const void* w_hh, const void* bias, void* h_state,
                          float* c_state, void* out, void* ws, cudaStream_t s);
size_t simt_hu_workspace_size(const HuProblem& p);
int32_t simt_hidden_update(const HuProblem& p, const void* gate_proj, const void* w_hh, const void* bias,
                           void* h_state, float* c_state, void* out, void* ws, cudaStream_t s);

// Reads element (r, k) of a [4H or O][K] weight given in any PLSTM_W_* layout.
__device__ __forceinline__ int64_t weight_src_index(int layout, int rows, int K, int r, int k) {
  if (layout == PLSTM_W_TRANSPOSED) return (int64_t)k * rows + r;
  if (layout == PLSTM_W_KPAIR) return ((int64_t)(k >> 1) * rows + r) * 2 + (k & 1);
  if (layout == PLSTM_W_MMAC) {  // rows = 4K: row = gate * K + unit
    const int gate = r / K, u = r % K, nt = K / 16;
    return (((((int64_t)(u >> 4) * nt + (k >> 4)) * 16 + (k & 15)) * 4 + ((u & 15) >> 2)) * 4 + gate) * 4 + (u & 3);
  }
  return (int64_t)r * K + k;
}

__device__ __forceinline__ float load_any(const void* src, int dtype, int64_t idx) {
  if (dtype == PLSTM_F32) return static_cast<const float*>(src)[idx];
  if (dtype == PLSTM_F16) return __half2float(static_cast<const __half*>(src)[idx]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(src)[idx]);
}

__device__ __forceinline__ void store_any(void* dst, int dtype, int64_t idx, float v) {
  if (dtype == PLSTM_F32)
    static_cast<float*>(dst)[idx] = v;
  else if (dtype == PLSTM_F16)
    static_cast<__half*>(dst)[idx] = __float2half_rn(v);
  else
    static_cast<__nv_bfloat16*>(dst)[idx] = __float2bfloat16_rn(v);
}

}  // namespace plstm
