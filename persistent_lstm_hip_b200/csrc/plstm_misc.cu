// plstm_misc.cu — small entry points: repeat_first_row and the tcgen05
// data-path layout self-check the test suite runs before trusting the
// wavefront kernel's register mapping.
#include <algorithm>
#include <string>

#include "plstm_common.cuh"
#include "sm100_ptx.cuh"

namespace plstm {
namespace {

__global__ void repeat_first_row_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                        int64_t row_bytes, int64_t total_bytes) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total_bytes;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = in[i % row_bytes];
}

// One CTA, 4 warps.  Each thread writes (lane << 8 | column) into TMEM
// columns 0..15 of its own lane with tcgen05.st 32x32b, then every warp reads
// its quadrant back with tcgen05.ld 16x256b.x2 at lane offsets 0 and 16 and
// with 32x32b.x8; the raw registers go to out[warp][lane][24].
__global__ void tmem_layout_kernel(uint32_t* out) {
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    ptx::tmem_alloc(ptx::smem_u32(&slot), 32);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = slot;
  const uint32_t row = (uint32_t)(32 * warp + lane);
  uint32_t v[8];
  for (int half = 0; half < 2; ++half) {
    for (int c = 0; c < 8; ++c) v[c] = (row << 8) | (uint32_t)(8 * half + c);
    ptx::tmem_st_32x32b_x8(tmem + ((uint32_t)(32 * warp) << 16) + 8 * half, v);
  }
  ptx::tmem_wait_st();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  uint32_t a[8], b[8], c[8];
  ptx::tmem_ld_16x256b_x2(tmem + ((uint32_t)(32 * warp) << 16), a);
  ptx::tmem_ld_16x256b_x2(tmem + ((uint32_t)(32 * warp + 16) << 16), b);
  ptx::tmem_ld_32x32b_x8(tmem + ((uint32_t)(32 * warp) << 16) + 8, c);
  ptx::tmem_wait_ld();
  uint32_t* o = out + (size_t)row * 24;
  for (int i = 0; i < 8; ++i) {
    o[i] = a[i];
    o[8 + i] = b[i];
    o[16 + i] = c[i];
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 32);
  }
}

}  // namespace
}  // namespace plstm

using namespace plstm;

extern "C" {

int32_t plstm_repeat_first_row(const void* input, int32_t cols, int32_t out_rows, int32_t dtype,
                               void* output, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(cols >= 0 && out_rows >= 0, "cols / out_rows must be >= 0");
  PLSTM_CHECK_ARG(dtype == PLSTM_F32 || dtype == PLSTM_F16 || dtype == PLSTM_BF16, "bad dtype");
  const int64_t row_bytes = (int64_t)cols * (int64_t)dtype_size(dtype);
  const int64_t total = row_bytes * out_rows;
  if (total == 0) return PLSTM_OK;
  PLSTM_CHECK_ARG(input != nullptr && output != nullptr, "NULL pointer");
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  repeat_first_row_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(input), static_cast<uint8_t*>(output), row_bytes, total);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

int32_t plstm_diag_tmem_layout(uint32_t* out, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(out != nullptr, "out is NULL");
  tmem_layout_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(out);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

// ---- hidden update -----------------------------------------------------------------------
static int32_t hu_problem(int32_t batch, int32_t seq_len, int32_t hidden, int32_t dtype, int32_t flags,
                          int32_t w_layout, int32_t device, HuProblem* p) {
  PLSTM_CHECK_ARG(batch >= 0 && seq_len >= 0, "plstm_hidden_update: batch and seq_len must be >= 0");
  PLSTM_CHECK_ARG(hidden >= 1, "plstm_hidden_update: hidden must be >= 1");
  PLSTM_CHECK_ARG(dtype == PLSTM_F32 || dtype == PLSTM_F16 || dtype == PLSTM_BF16, "plstm_hidden_update: bad dtype");
  PLSTM_CHECK_ARG((flags & ~(PLSTM_HU_SEQ_MAJOR | PLSTM_HU_WRITE_SEQUENCE)) == 0, "plstm_hidden_update: unknown flags");
  PLSTM_CHECK_ARG(w_layout == PLSTM_W_NATIVE || w_layout == PLSTM_W_TRANSPOSED || w_layout == PLSTM_W_MMAC,
                  "plstm_hidden_update: w_layout must be PLSTM_W_NATIVE, _TRANSPOSED or _MMAC");
  PLSTM_CHECK_ARG(w_layout != PLSTM_W_MMAC || hidden % 16 == 0, "plstm_hidden_update: PLSTM_W_MMAC needs H % 16 == 0");
  p->B = batch;
  p->T = seq_len;
  p->H = hidden;
  p->dtype = dtype;
  p->flags = flags;
  p->w_layout = w_layout;
  p->device = device;
  return PLSTM_OK;
}

int32_t plstm_hidden_update_workspace_size(int32_t batch, int32_t seq_len, int32_t hidden, int32_t dtype,
                                           int32_t flags, int32_t device, size_t* bytes) {
  clear_error();
  PLSTM_CHECK_ARG(bytes != nullptr, "bytes is NULL");
  HuProblem p;
  const int32_t rc = hu_problem(batch, seq_len, hidden, dtype, flags, PLSTM_W_NATIVE, device, &p);
  if (rc != PLSTM_OK) return rc;
  *bytes = std::max(tcl_hu_supported(p) ? tcl_hu_workspace_size(p) : (size_t)0, simt_hu_workspace_size(p));
  return PLSTM_OK;
}

int32_t plstm_hidden_update(const void* gate_proj, int32_t batch, int32_t seq_len, int32_t hidden, const void* w_hh,
                            int32_t w_layout, const void* bias, int32_t dtype, int32_t flags, void* h_state,
                            float* c_state, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int dev = 0;
  PLSTM_TRY_CUDA(cudaGetDevice(&dev));
  HuProblem p;
  int32_t rc = hu_problem(batch, seq_len, hidden, dtype, flags, w_layout, dev, &p);
  if (rc != PLSTM_OK) return rc;
  PLSTM_CHECK_ARG(w_hh != nullptr && h_state != nullptr && c_state != nullptr && out != nullptr,
                  "plstm_hidden_update: w_hh, h_state, c_state and out must not be NULL");
  PLSTM_CHECK_ARG(seq_len == 0 || batch == 0 || gate_proj != nullptr, "plstm_hidden_update: gate_proj is NULL");
  PLSTM_CHECK_ARG(aligned16(workspace), "plstm_hidden_update: workspace must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t es = dtype_size(dtype);
  if (batch == 0) return PLSTM_OK;
  if (seq_len == 0) {  // no step: the state stays zero
    PLSTM_TRY_CUDA(cudaMemsetAsync(h_state, 0, (size_t)batch * hidden * es, s));
    PLSTM_TRY_CUDA(cudaMemsetAsync(c_state, 0, (size_t)batch * hidden * 4, s));
    if (!(flags & PLSTM_HU_WRITE_SEQUENCE)) PLSTM_TRY_CUDA(cudaMemsetAsync(out, 0, (size_t)batch * hidden * es, s));
    return PLSTM_OK;
  }
  const bool tc = tcl_hu_supported(p);
  const size_t need = tc ? tcl_hu_workspace_size(p) : simt_hu_workspace_size(p);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("plstm_hidden_update: workspace of " + std::to_string(need) + " bytes required");
    return PLSTM_EWORKSPACE;
  }
  PLSTM_TRY_CUDA(cudaMemsetAsync(workspace, 0, kStatusBytes, s));
  rc = tc ? tcl_hidden_update(p, gate_proj, w_hh, bias, h_state, c_state, out, workspace, s)
          : simt_hidden_update(p, gate_proj, w_hh, bias, h_state, c_state, out, workspace, s);
  return rc;
}

}  // extern "C"
