// plstm_noalloc.cu — a forward entry point for callers that cannot provide a
// device workspace.
//
// Who needs it: hosts that own every device allocation themselves and do not
// let a plugin call cudaMalloc from its execute path (inference-server and
// engine plugin interfaces whose enqueue/execute hook must not allocate), and
// programs that run under a fixed device-memory budget after start-up, where
// an allocation on the hot path could fail or stall the device.  Such a caller
// still passes its inputs and outputs, but the scratch the tensor-core forward
// needs (status word, repacked x tiles, row order, tile lengths, length
// histogram) comes from the array below instead of a caller workspace.
//
// The array is a file-scope device variable: every GPU on which the library is
// loaded holds its kNoAllocScratchBytes for the life of the process.  All
// calls share it and it keeps what the previous call left; the entry point
// clears the status block itself (the only part that must start at zero; every
// other byte a call reads is written by that call first).  Two calls whose GPU
// work overlaps (different streams, or different host threads on one device)
// race on the array and must be serialised by the caller.
#include <mutex>
#include <string>

#include "plstm_common.cuh"

namespace plstm {
namespace {

constexpr size_t kNoAllocScratchBytes = 24u << 20;  // 24 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
int32_t scratch_for_current_device(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("plstm_forward_packed_noalloc: device ordinal out of range");
    return PLSTM_EINVAL;
  }
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(std::string("plstm_forward_packed_noalloc: cudaGetSymbolAddress failed: ") +
                cudaGetErrorString(e));
      return PLSTM_ECUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PLSTM_OK;
}

}  // namespace
}  // namespace plstm

using namespace plstm;

extern "C" int32_t plstm_forward_packed_noalloc(const plstm_desc* d, const void* packed, const void* x,
                                                const int32_t* lengths, const void* h0, const void* c0,
                                                void* out, void* h_n, void* c_n, void* stream) {
  clear_error();
  Problem p;
  int32_t rc = make_problem(d, &p);  // the same argument checks as every other entry point
  if (rc != PLSTM_OK) return rc;
  // What this entry point adds: the 16-bit tensor-core path only, and no option
  // whose scratch lives outside the fixed array.
  PLSTM_CHECK_ARG(d->dtype == PLSTM_F16 || d->dtype == PLSTM_BF16,
                  "plstm_forward_packed_noalloc serves the f16 / bf16 tensor-core path only");
  PLSTM_CHECK_ARG(d->backend == PLSTM_BACKEND_AUTO || d->backend == PLSTM_BACKEND_TC,
                  "plstm_forward_packed_noalloc serves the tensor-core backend only");
  PLSTM_CHECK_ARG(!(d->flags & PLSTM_FLAG_TRACE), "PLSTM_FLAG_TRACE needs a caller workspace");
  PLSTM_CHECK_ARG(!(d->flags & PLSTM_FLAG_DEDUPE), "PLSTM_FLAG_DEDUPE needs a caller workspace");
  PLSTM_CHECK_ARG(packed != nullptr, "packed is NULL");
  PLSTM_CHECK_ARG(aligned16(packed), "packed must be 16-byte aligned");
  PLSTM_CHECK_ARG(p.B == 0 || p.T == 0 || x != nullptr, "x is NULL");
  PLSTM_CHECK_ARG(p.B == 0 || out != nullptr, "out is NULL");
  PLSTM_CHECK_ARG((h0 == nullptr) == (c0 == nullptr), "h0 and c0 must both be given or both be NULL");
  std::string why;
  if (!tc_supported(p, &why)) {
    set_error("plstm_forward_packed_noalloc: tensor-core backend cannot serve this problem: " + why);
    return PLSTM_ENOTSUP;
  }
  const size_t need = tc_workspace_size(p);
  if (need > kNoAllocScratchBytes) {
    set_error("plstm_forward_packed_noalloc: this problem needs " + std::to_string(need) +
              " bytes of scratch, more than the " + std::to_string(kNoAllocScratchBytes) +
              " bytes (24 MiB) the no-allocation entry point holds; use plstm_forward_packed with a workspace");
    return PLSTM_EINVAL;
  }
  DeviceGuard dev_guard;  // the caller's current device is restored on return
  if ((rc = dev_guard.enter(p.device)) != PLSTM_OK) return rc;
  void* ws = nullptr;
  rc = scratch_for_current_device(p.device, &ws);
  if (rc != PLSTM_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PLSTM_TRY_CUDA(cudaMemsetAsync(ws, 0, kStatusBytes, s));
  if (p.B == 0) return PLSTM_OK;
  rc = tc_forward(p, packed, x, lengths, h0, c0, out, h_n, c_n, ws, s);
  if (rc != PLSTM_OK) return rc;
  if (p.flags & PLSTM_FLAG_SYNC_CHECK) {
    int32_t st = 0, detail = 0;
    rc = plstm_read_status(ws, stream, &st, &detail);
    if (rc != PLSTM_OK) return rc;
    if (st != PLSTM_OK) {
      set_error("device status " + std::to_string(st) + ": a bounded inter-CTA wait gave up");
      return st;
    }
  }
  return PLSTM_OK;
}
