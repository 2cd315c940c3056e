// plstm_misc.cu — small entry points: repeat_first_row and the tcgen05
// data-path layout self-check the test suite runs before trusting the
// wavefront kernel's register mapping.
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

}  // extern "C"
