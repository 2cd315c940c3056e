// plstm_gemm.cu — input-projection GEMM on tcgen05 tensor cores.
//
// gate[M][N] = x[M][K] . w_t[K][N] (no bias), f16 or bf16 in and out, f32
// accumulation: the reference's adaptive_lstm_input_gemm_forward_workspace
// (miopen_adaptive_lstm_hip/csrc/adaptive_lstm_hip.cu:389-433, :2355-2385),
// which calls hipblasGemmEx per layer.  For the LSTM's layer 0 (K = I = 5,
// N = 4H) it is a pure streaming kernel: ~10 bytes in, 4H * 2 bytes out per row.
//
// Design: persistent CTAs, each owning one 128-column slice of N (its
// W^T slice [128 x Kp] stays resident in shared memory, transposed to K-major)
// and walking 128-row tiles of M.  Warp roles:
//   warps 0-3  producers: thread = row; the x row is loaded, zero-padded to Kp
//              and written K-major (no swizzle for Kp = 16, 128-byte swizzle
//              for Kp = 64 .. 256) into one of two A stages;
//   warp 4     issues tcgen05.mma M=128 N=128 into one of two TMEM accumulators;
//   warps 5-12 epilogue: two warps per TMEM lane quadrant, 64 accumulator
//              columns each: tcgen05.ld, convert to 16-bit in pairs, stage the
//              tile in one of two shared-memory buffers as two 128 x 64 boxes in
//              the 128-byte swizzle, then two TMA tensor stores
//              (cp.async.bulk.tensor.2d) write it out and drain to HBM while the
//              next tile is loaded.  Without a tensor map (driver entry point
//              unavailable) the tile goes out as one bulk copy per 256-byte row.
// All waits are bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "plstm_common.cuh"
#include "sm100_ptx.cuh"

namespace plstm {
namespace gemm {

constexpr int kBM = 128, kBN = 128;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (4 + 1 + kEpiWarps) * 32;
constexpr int kStageRowPad = kBN * 2 + 16;  // staging row stride of the row-copy path (bank-conflict padding)
constexpr int kStageBytes = kBM * kStageRowPad;  // one stage buffer (>= the TMA path's two 16 KB boxes)

__host__ __device__ constexpr int kpad_of(int K) { return K <= 16 ? 16 : ((K + 63) / 64) * 64; }

constexpr int kMaxSmem = 232448;  // opt-in dynamic shared memory per CTA on sm_100

struct Layout {
  int kp;
  int stages;   // A stages (2 unless that would not fit)
  int a_stage;  // bytes of one A stage
  int b_off, a_off, stage_off, bar_off, total;
};

__host__ __device__ inline Layout layout_for(int K) {
  Layout lo;
  lo.kp = kpad_of(K);
  lo.a_stage = kBM * lo.kp * 2;
  lo.b_off = 0;
  lo.a_off = kBN * lo.kp * 2;  // B tile [128 x Kp]
  for (lo.stages = 2; lo.stages >= 1; --lo.stages) {
    lo.stage_off = (lo.a_off + lo.stages * lo.a_stage + 1023) / 1024 * 1024;  // swizzle atoms: 1 KB aligned
    lo.bar_off = lo.stage_off + 2 * kStageBytes;
    lo.total = lo.bar_off + 128 + 1024;
    if (lo.total <= kMaxSmem) break;
  }
  return lo;
}

__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}
__device__ __forceinline__ uint32_t none16_off(int row, int k) {
  return (uint32_t)((row >> 3) * 256 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}
// Offset of (row, k) in a K-major operand of 128 rows and Kp columns.
__device__ __forceinline__ uint32_t kmajor_off(int row, int k, int kp) {
  if (kp == 16) return none16_off(row, k);
  return (uint32_t)((k >> 6) * (128 * 128)) + sw128_off(row, k & 63);
}

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(bar, parity))
    if (ptx::globaltimer() - t0 > 2000000000ull) return false;
  return true;
}

__device__ __forceinline__ void bulk_s2g(void* gdst, uint32_t ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Two values rounded to 16 bits in one conversion (lo -> bits [0, 16)): the paired
// cvt.rn.{f16x2,bf16x2}.f32 runs at ALU rate, the single-value one at the MUFU rate.
template <bool BF16>
__device__ __forceinline__ uint32_t bits16x2(float lo, float hi) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// TMA store of one box of the tensor map at element coordinates (x = column, y = row) from
// this CTA's shared memory, tracked by the issuing thread's bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t ssrc, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
               "r"(y), "r"(ssrc)
               : "memory");
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    input_gemm_kernel(const uint16_t* __restrict__ x, int M, int K, const uint16_t* __restrict__ w_t, int N,
                      uint16_t* __restrict__ gate, int n_tiles_n, int m_tiles, const __grid_constant__ CUtensorMap gmap,
                      int use_tma) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const Layout lo = layout_for(K);
  const int kp = lo.kp;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Tiles of this CTA: fixed N slice, M tiles strided over the CTAs sharing it.
  const int nt = blockIdx.x % n_tiles_n;
  const int n0 = nt * kBN;
  const int ctas_per_n = (gridDim.x + n_tiles_n - 1 - nt) / n_tiles_n;
  const int first_m = blockIdx.x / n_tiles_n;
  const int my_tiles = first_m < m_tiles ? (m_tiles - first_m + ctas_per_n - 1) / ctas_per_n : 0;

  const uint32_t bar = sbase + lo.bar_off;
  const uint32_t a_full = bar, a_empty = bar + 16, d_full = bar + 32, d_empty = bar + 48;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + lo.bar_off + 64);
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(a_full + 8 * s, 4);   // one arrive per producer warp
      ptx::mbar_init(a_empty + 8 * s, 1);  // MMA commit
      ptx::mbar_init(d_full + 8 * s, 1);   // MMA commit
      ptx::mbar_init(d_empty + 8 * s, kEpiWarps);  // one arrive per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), 2 * kBN);
    ptx::tmem_relinquish();
  }
  // Resident B: B[n][k] = w_t[k][n0 + n], K-major, zero past K / N.
  for (int i = tid; i < kBN * kp; i += kThreads) {
    const int n = i / kp, k = i % kp;
    uint16_t v = 0;
    if (k < K && n0 + n < N) v = w_t[(size_t)k * N + n0 + n];
    *reinterpret_cast<uint16_t*>(sm + lo.b_off + kmajor_off(n, k, kp)) = v;
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp < 4 && kp == 16) {
    // ---------------- producers, K <= 16 ----------------
    // Thread = row.  A row is at most 16 values, so its loads stay raw in registers and the
    // loads of tile it + 1 are issued before tile it is written (and rows 4 tiles ahead are
    // prefetched into L2): the producers never wait a whole memory latency per tile.
    const int m_local = tid;
    const int ns = lo.stages;
    auto row_of = [&](int it) { return (first_m + it * ctas_per_n) * kBM + m_local; };
    auto load = [&](int it, uint32_t (&raw)[16]) {
      const int m = row_of(it);
      const bool valid = it < my_tiles && m < M;
      const uint16_t* src = x + (size_t)(valid ? m : 0) * K;
#pragma unroll
      for (int k = 0; k < 16; ++k) raw[k] = (valid && k < K) ? (uint32_t)__ldg(src + k) : 0u;
    };
    uint32_t cur[16], nxt[16];
    load(0, cur);
    for (int it = 0; it < my_tiles; ++it) {
      const int s = it % ns;
      if (it + 4 < my_tiles && row_of(it + 4) < M) ptx::prefetch_l2(x + (size_t)row_of(it + 4) * K);
      load(it + 1, nxt);
      if (it >= ns && !wait_bounded(a_empty + 8 * s, ((it / ns) - 1) & 1)) break;
      uint8_t* a = sm + lo.a_off + s * lo.a_stage;
      *reinterpret_cast<uint4*>(a + none16_off(m_local, 0)) =
          make_uint4(cur[0] | cur[1] << 16, cur[2] | cur[3] << 16, cur[4] | cur[5] << 16, cur[6] | cur[7] << 16);
      *reinterpret_cast<uint4*>(a + none16_off(m_local, 8)) = make_uint4(
          cur[8] | cur[9] << 16, cur[10] | cur[11] << 16, cur[12] | cur[13] << 16, cur[14] | cur[15] << 16);
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(a_full + 8 * s);
#pragma unroll
      for (int k = 0; k < 16; ++k) cur[k] = nxt[k];
    }
  } else if (warp < 4) {
    // ---------------- producers ----------------
    const int m_local = tid;  // 0..127
    const int ns = lo.stages;
    for (int it = 0; it < my_tiles; ++it) {
      const int s = it % ns;
      if (it >= ns && !wait_bounded(a_empty + 8 * s, ((it / ns) - 1) & 1)) break;
      const int m = (first_m + it * ctas_per_n) * kBM + m_local;
      uint8_t* a = sm + lo.a_off + s * lo.a_stage;
      const uint16_t* src = x + (size_t)m * K;
      const bool valid = m < M;
      if (valid && (K % 8) == 0 && ((reinterpret_cast<uintptr_t>(x) & 15) == 0)) {
        for (int k = 0; k < kp; k += 8) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (k < K) v = *reinterpret_cast<const uint4*>(src + k);
          *reinterpret_cast<uint4*>(a + kmajor_off(m_local, k, kp)) = v;
        }
      } else {
        for (int k = 0; k < kp; ++k) {
          const uint16_t v = (valid && k < K) ? src[k] : (uint16_t)0;
          *reinterpret_cast<uint16_t*>(a + kmajor_off(m_local, k, kp)) = v;
        }
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(a_full + 8 * s);
    }
  } else if (warp == 4) {
    // ---------------- MMA issue ----------------
    const uint32_t idesc = ptx::idesc_f16(kBM, kBN, BF16);
    const int ns = lo.stages;
    for (int it = 0; it < my_tiles; ++it) {
      const int s = it % ns, db = it & 1;
      bool ok = true;
      if (lane == 0) {
        ok = wait_bounded(a_full + 8 * s, (it / ns) & 1);
        if (ok && it >= 2) ok = wait_bounded(d_empty + 8 * db, ((it - 2) >> 1) & 1);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(db * kBN);
        const uint32_t a0 = sbase + lo.a_off + s * lo.a_stage;
        const uint32_t b0 = sbase + lo.b_off;
        if (kp == 16) {
          ptx::mma_f16_ss(d, ptx::desc_k_none(a0, 128, 256), ptx::desc_k_none(b0, 128, 256), idesc, 0u);
        } else {
          for (int kb = 0; kb < kp / 64; ++kb)
            for (int kk = 0; kk < 4; ++kk)
              ptx::mma_f16_ss(d, ptx::desc_k_sw128(a0 + kb * 128 * 128 + kk * 32),
                              ptx::desc_k_sw128(b0 + kb * 128 * 128 + kk * 32), idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        ptx::mma_commit(d_full + 8 * db);
        ptx::mma_commit(a_empty + 8 * s);
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - 5;                 // 0 .. 7
    const int q = warp & 3, hc = ew >> 2;    // TMEM lane quadrant, column half
    const int m_local = 32 * q + lane;
    const int etid = ew * 32 + lane;         // 0 .. 255
    const int ncols = min(kBN, N - n0);
    for (int it = 0; it < my_tiles; ++it) {
      const int db = it & 1;
      if (!wait_bounded(d_full + 8 * db, (it >> 1) & 1)) break;
      ptx::tc_fence_after();
      uint32_t r[64];
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(db * kBN + hc * 64);
      ptx::tmem_ld_32x32b_x16(taddr + 0, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
      ptx::tmem_ld_32x32b_x16(taddr + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
      ptx::tmem_ld_32x32b_x16(taddr + 32, *reinterpret_cast<uint32_t(*)[16]>(&r[32]));
      ptx::tmem_ld_32x32b_x16(taddr + 48, *reinterpret_cast<uint32_t(*)[16]>(&r[48]));
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(d_empty + 8 * db);
      uint8_t* stage = sm + lo.stage_off + db * kStageBytes;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          pk[i] = bits16x2<BF16>(__uint_as_float(r[8 * c + 2 * i]), __uint_as_float(r[8 * c + 2 * i + 1]));
        // TMA: box hc (columns 64 hc ..), 128-byte rows with 16-byte chunks swizzled by row % 8;
        // row copies: padded rows of kStageRowPad bytes.
        uint8_t* dst = use_tma ? stage + hc * (kBM * 128) + m_local * 128 + ((c ^ (m_local & 7)) << 4)
                               : stage + m_local * kStageRowPad + hc * 128 + 16 * c;
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      ptx::fence_proxy_async_smem();  // the staged tile is read by the async copies below
      // The previous tile's copies (other stage buffer) have read their data: the buffer this
      // tile's successor writes is free once everyone is past the barrier.
      if (etid < kBM) bulk_wait_read0();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
      // The tile drains to HBM asynchronously while the next tile is loaded from tensor memory.
      const int m0 = (first_m + it * ctas_per_n) * kBM;
      if (use_tma) {
        if (etid == 0) {  // rows past M and columns past N are clipped by the tensor map
          tma_store_2d(&gmap, ptx::smem_u32(stage), n0, m0);
          if (ncols > 64) tma_store_2d(&gmap, ptx::smem_u32(stage + kBM * 128), n0 + 64, m0);
          bulk_commit();
        }
      } else if (etid < kBM && m0 + etid < M) {
        bulk_s2g(gate + (size_t)(m0 + etid) * N + n0, ptx::smem_u32(stage + etid * kStageRowPad),
                 (uint32_t)(ncols * 2));
        bulk_commit();
      }
    }
    if (etid < kBM) bulk_wait0();  // every copy has written global memory before the CTA ends
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 2 * kBN);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// Tensor map of gate[M][N] (16-bit) with 128-row x 64-column boxes in the 128-byte swizzle;
// false if it cannot be made (the kernel then stores rows with plain bulk copies).
bool make_gate_map(void* gate, int M, int N, CUtensorMap* map) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)N * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kBM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, gate, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gemm
}  // namespace plstm

using namespace plstm;

extern "C" int32_t plstm_input_gemm(const void* x, int32_t m, int32_t k, const void* w_t, int32_t n,
                                    int32_t dtype, void* gate, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(dtype == PLSTM_F16 || dtype == PLSTM_BF16, "plstm_input_gemm: dtype must be f16 or bf16");
  PLSTM_CHECK_ARG(m >= 0 && k >= 1 && n >= 1, "plstm_input_gemm: m >= 0, k >= 1, n >= 1 required");
  PLSTM_CHECK_ARG(n % 8 == 0, "plstm_input_gemm: n must be a multiple of 8 (16-byte output rows)");
  if (k > 256) {
    set_error("plstm_input_gemm: k > 256 is not supported by this kernel");
    return PLSTM_ENOTSUP;
  }
  if (m == 0) return PLSTM_OK;
  PLSTM_CHECK_ARG(x != nullptr && w_t != nullptr && gate != nullptr, "plstm_input_gemm: NULL pointer");
  PLSTM_CHECK_ARG((reinterpret_cast<uintptr_t>(gate) & 15) == 0, "plstm_input_gemm: gate must be 16-byte aligned");
  int dev = 0, sms = 148;
  PLSTM_TRY_CUDA(cudaGetDevice(&dev));
  PLSTM_TRY_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const gemm::Layout lo = gemm::layout_for(k);
  const int n_tiles_n = (n + gemm::kBN - 1) / gemm::kBN;
  const int m_tiles = (m + gemm::kBM - 1) / gemm::kBM;
  const int grid = std::max(n_tiles_n, std::min(m_tiles * n_tiles_n, (sms / n_tiles_n) * n_tiles_n));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap gmap;
  std::memset(&gmap, 0, sizeof(gmap));
  const int use_tma = gemm::make_gate_map(gate, m, n, &gmap) ? 1 : 0;
  auto kern = dtype == PLSTM_BF16 ? gemm::input_gemm_kernel<true> : gemm::input_gemm_kernel<false>;
  PLSTM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lo.total));
  kern<<<grid, gemm::kThreads, lo.total, s>>>(static_cast<const uint16_t*>(x), m, k, static_cast<const uint16_t*>(w_t),
                                              n, static_cast<uint16_t*>(gate), n_tiles_n, m_tiles, gmap, use_tma);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}
