// plstm_tcl.cu — tcgen05 layer-sequential backend for hidden sizes other than the H = 128
// wavefront kernel's (multiples of 64 up to 512; configs 3 and 4 are H = 256 / 512).
//
// What it replaces.  The reference runs these sizes through its adaptive path:
// per layer an input-projection GEMM (adaptive_lstm_input_gemm_forward_workspace,
// miopen_adaptive_lstm_hip/csrc/adaptive_lstm_hip.cu:389-433) and then either a
// packed-MMAC persistent recurrence (adaptive_lstm_mmac_packed_kernel, :3461-3667)
// or, per timestep, a library GEMM [B,H]x[H,4H] plus a pointwise launch
// (:2388-2678); the generic path does the same with ATen matmuls
// (persistent_lstm_hip.cu:2923-3181).
//
// Design (B200-first), per layer l:
//   1. proj_kernel: gates_l = in_l . W_ih_l^T + b_ih_l + b_hh_l on tcgen05 (M = 128
//      batch rows of one timestep, N = 128 gate rows, f32 accumulation in TMEM).
//      in_0 is x (K = I padded to 16); in_l (l >= 1) is layer l-1's h sequence.
//      The W_ih slice of the CTA's 128 gate rows stays resident in shared memory;
//      the epilogue writes one 128-row x 64-column block per (step, batch tile,
//      recurrent CTA), already in the order the recurrence reads it.
//   2. rec_kernel: one cluster of C = H / 32 CTAs per batch tile (32-80 rows); CTA r owns
//      hidden units [32 r, 32 r + 32), i.e. 128 gate rows = one M = 128 MMA tile.
//      Its W_hh slice [128 x H] stays resident in tensor memory (H / 2 columns) for
//      the whole sequence.  Per step: D[128 x NT] = W_hh . h_{t-1}^T as H / 16
//      tcgen05.mma (A from TMEM, B = h_{t-1} from shared memory), the MMAs over the
//      CTA's own 32 units issued as soon as it has written them, the rest once the
//      other C - 1 pieces have landed, split between the control warp and a helper
//      warp that accumulates into a second TMEM accumulator (one thread issues an MMA
//      only every ~45-100 cycles); with 64- / 80-row tiles layer 0's input projection
//      runs here too (W_ih slice in TMEM, x tiles streamed in); the compute warps add the projected gate
//      block (prefetched three steps ahead by bulk copy), apply the gate math in
//      registers (c in f32), write their h piece (and store it to the layer's h
//      sequence in global memory, the next layer's projection input); the last
//      one to finish pushes the piece to the C - 1 peers with shared -> distributed
//      shared bulk copies that complete on the peers' barriers, then prefetches the
//      gate block of step t + 3.
//   3. the Linear head (or the h sequence output) from the last layer's h.
// Layers run one after the other; every wait in the kernels is bounded.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "plstm_common.cuh"
#include "sm100_ptx.cuh"

namespace plstm {
namespace tcl {

constexpr int kU = 32;      // hidden units per recurrent CTA (4 x 32 = 128 gate rows)
constexpr int kRows = 128;  // gate rows per CTA
constexpr int kXK = 16;     // layer-0 input width step (one MMA K step)
constexpr int kMaxXK = 128; // widest padded layer-0 input
// Layer-0 input width rounded up to one MMA K step.
__host__ __device__ inline int kx_of(int I) { return (I + kXK - 1) / kXK * kXK; }
// Batch rows per cluster tile (N of the recurrent MMAs): 64; 32 or 48 for H <= 256 when
// the batch then still runs in one wave of clusters (more, shorter steps in flight); 80
// for H >= 384 where 64-row tiles would need a second wave.  The kernels are templated on it (NT) and
// declare these quantities locally (PLSTM_TCL_TILE_CONSTANTS).
// Gate block rows are NT + 8 elements (+16 bytes against bank conflicts); one CTA's h piece
// is 32 units x NT rows.
__host__ __device__ constexpr int gblock_of(int nt) { return kRows * (nt + 8) * 2; }
__host__ __device__ constexpr int piece_of(int nt) { return nt * kU * 2; }
#define PLSTM_TCL_TILE_CONSTANTS(NT)                                                             \
  constexpr int kNT = NT, kGRow = NT + 8, kGBlock = kRows * (NT + 8) * 2, kPiece = NT * kU * 2, \
                kKG = (NT / 8) * 128;                                                             \
  (void)kGRow;                                                                                    \
  (void)kGBlock;                                                                                  \
  (void)kPiece;                                                                                   \
  (void)kKG
constexpr int kMaxL = 16;

__host__ __device__ inline int ctas_of(int H) { return H / kU; }

// Packed image: [W_hh images L x 4H x H][W_ih images per layer 4H x Kin (layer 0: Kin = kx, the
// input width rounded up to 16, in a region sized for 128)][bias f32 L x 4H][W_lin 16-bit O x H]
// [b_lin f32 O]; gate rows in the recurrent CTA order below.
__host__ __device__ inline size_t off_whh(int l, int H) { return (size_t)l * 4 * H * H * 2; }
__host__ __device__ inline size_t off_wih(int l, int H, int L) {
  return off_whh(L, H) + (l == 0 ? 0 : (size_t)4 * H * kMaxXK * 2 + (size_t)(l - 1) * 4 * H * H * 2);
}
__host__ __device__ inline size_t off_bias(int H, int L) { return off_wih(L, H, L); }
__host__ __device__ inline size_t off_wlin(int H, int L) { return off_bias(H, L) + (size_t)L * 4 * H * 4; }
__host__ __device__ inline size_t off_blin(int H, int L, int O) {
  return off_wlin(H, L) + (((size_t)O * H * 2 + 15) / 16) * 16;
}
__host__ __device__ inline size_t packed_total(int H, int L, int O) { return off_blin(H, L, O) + (size_t)O * 4 + 16; }

// Permuted gate row rho of CTA r: quadrant q = rho / 32 holds units 32 r + 8 q + [0, 8)
// as [i x 8 | f x 8 | g x 8 | o x 8]; returns the nn.LSTM row (gate * H + unit).
__host__ __device__ inline int src_row(int H, int r, int rho) {
  const int q = rho >> 5, gate = (rho >> 3) & 3, j = rho & 7;
  return gate * H + kU * r + 8 * q + j;
}
// Gate rows i, f, o are stored pre-scaled by 1/2: sigmoid(z) = (1 + tanh(z / 2)) / 2.
__host__ __device__ inline float row_scale(int rho) { return ((rho >> 3) & 3) == 2 ? 1.0f : 0.5f; }

template <bool BF16>
__device__ __forceinline__ uint16_t to_bits(float v) {
  if (BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
  }
  __half h = __float2half_rn(v);
  return *reinterpret_cast<uint16_t*>(&h);
}
template <bool BF16>
__device__ __forceinline__ float from_bits(uint16_t b) {
  if (BF16) return __bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&b));
  return __half2float(*reinterpret_cast<__half*>(&b));
}
template <bool BF16>
__device__ __forceinline__ float2 from_bits2(uint32_t b) {
  if (BF16) return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&b));
  return __half22float2(*reinterpret_cast<__half2*>(&b));
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack2_bits(float lo, float hi) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}
__device__ __forceinline__ uint32_t none16_off(int row, int k) {
  return (uint32_t)((row >> 3) * 256 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}
// Byte offset of (unit k, tile row n) in an h tile of H units: pieces of 32 units,
// each [4 K groups][8 row groups][8 rows][8 units] (K-major, no swizzle: the K
// groups of the whole tile are kKG bytes apart, row groups 128 bytes apart).
template <int NT>
__device__ __forceinline__ uint32_t hoff(int k, int n) {
  return (uint32_t)((k >> 3) * ((NT / 8) * 128) + (n >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2);
}

// Bounded mbarrier wait; false = gave up (timeout or abort).
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         unsigned long long timeout_ns) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (ptx::globaltimer() - t0 > timeout_ns) return false;
  }
}

// Warp-uniform version: lane 0 waits, the result is broadcast.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long timeout_ns) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_bar(bar, parity, abort_flag, timeout_ns) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}


// ---- packing ------------------------------------------------------------------------
struct PackArgs {
  const void* w_ih[kMaxL];
  const void* w_hh[kMaxL];
  const void* b_ih[kMaxL];
  const void* b_hh[kMaxL];
  const void* w_lin;
  const void* b_lin;
  int ih_layout, hh_layout, dtype, L, I, H, O;
  int hid;  // the model's hidden size (<= H; units >= hid are zero padding)
  int kx;   // layer-0 input width rounded up to 16 (<= 128)
};

__global__ void pack_kernel(const PackArgs a, uint8_t* packed) {
  const int H = a.H, L = a.L, G = 4 * H, GR = 4 * a.hid;
  // nn.LSTM row of permuted row rho of CTA r in a model of hidden size hid; -1 = padding unit.
  auto real_row = [&](int r, int rho) -> int {
    const int q = rho >> 5, gate = (rho >> 3) & 3, j = rho & 7;
    const int unit = kU * r + 8 * q + j;
    return unit < a.hid ? gate * a.hid + unit : -1;
  };
  const int64_t n_hh = (int64_t)L * G * H;
  const int64_t n_ih = (int64_t)G * a.kx + (int64_t)(L - 1) * G * H;
  const int64_t n_b = (int64_t)L * G;
  const int64_t n_wl = (int64_t)a.O * H;
  const int64_t total = n_hh + n_ih + n_b + n_wl + a.O;
  const bool bf16 = a.dtype == PLSTM_BF16;
  auto put16 = [&](size_t off_bytes, int64_t idx, float v) {
    __half hv = __float2half_rn(v);
    __nv_bfloat16 bv = __float2bfloat16_rn(v);
    reinterpret_cast<uint16_t*>(packed + off_bytes)[idx] =
        bf16 ? *reinterpret_cast<uint16_t*>(&bv) : *reinterpret_cast<uint16_t*>(&hv);
  };
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n_hh) {
      const int l = (int)(i / ((int64_t)G * H));
      const int64_t rem = i % ((int64_t)G * H);
      const int rp = (int)(rem / H), k = (int)(rem % H);
      const int r = rp / kRows, rho = rp % kRows;
      const int sr = real_row(r, rho);
      float v = 0.0f;
      if (sr >= 0 && k < a.hid) v = load_any(a.w_hh[l], a.dtype, weight_src_index(a.hh_layout, GR, a.hid, sr, k));
      put16(off_whh(l, H), rem, v * row_scale(rho));
    } else if (i < n_hh + n_ih) {
      int64_t j = i - n_hh;
      int l = 0, kin = a.kx;
      if (j >= (int64_t)G * a.kx) {
        j -= (int64_t)G * a.kx;
        l = 1 + (int)(j / ((int64_t)G * H));
        j %= (int64_t)G * H;
        kin = H;
      }
      const int rp = (int)(j / kin), k = (int)(j % kin);
      const int r = rp / kRows, rho = rp % kRows;
      const int kreal = l == 0 ? a.I : a.hid;
      const int sr = real_row(r, rho);
      float v = 0.0f;
      if (sr >= 0 && k < kreal) v = load_any(a.w_ih[l], a.dtype, weight_src_index(a.ih_layout, GR, kreal, sr, k));
      put16(off_wih(l, H, L), j, v * row_scale(rho));
    } else if (i < n_hh + n_ih + n_b) {
      const int64_t j = i - n_hh - n_ih;
      const int l = (int)(j / G), rp = (int)(j % G);
      const int r = rp / kRows, rho = rp % kRows;
      const int sr = real_row(r, rho);
      float v = 0.0f;
      if (sr >= 0 && a.b_ih[l] != nullptr) v += load_any(a.b_ih[l], a.dtype, sr);
      if (sr >= 0 && a.b_hh[l] != nullptr) v += load_any(a.b_hh[l], a.dtype, sr);
      reinterpret_cast<float*>(packed + off_bias(H, L))[j] = v * row_scale(rho);
    } else if (i < n_hh + n_ih + n_b + n_wl) {
      const int64_t j = i - n_hh - n_ih - n_b;
      const int o = (int)(j / H), k = (int)(j % H);
      float v = 0.0f;
      if (a.w_lin != nullptr && k < a.hid)
        v = load_any(a.w_lin, a.dtype, weight_src_index(PLSTM_W_NATIVE, a.O, a.hid, o, k));
      put16(off_wlin(H, L), j, v);
    } else {
      const int o = (int)(i - n_hh - n_ih - n_b - n_wl);
      float v = 0.0f;
      if (a.b_lin != nullptr) v = load_any(a.b_lin, a.dtype, o);
      reinterpret_cast<float*>(packed + off_blin(H, L, a.O))[o] = v;
    }
  }
}

// ---- projection GEMM ----------------------------------------------------------------
// One job = (step t, batch tile, recurrent CTA r): D[128 gate rows x 64 batch rows] =
// W_ih[r's rows] . in(t, tile)^T.  W_ih's slice stays resident in tensor memory (A
// operand); the input tile (all K of one step and batch tile: layer l-1's h pieces,
// or the packed x tile for layer 0) arrives with one bulk copy into a 3-stage ring;
// two TMEM accumulators let the epilogue of one job overlap the MMAs of the next.
// The epilogue (lane = gate row) adds the bias and writes the gate block row of the
// recurrence directly: 64 contiguous 16-bit values.  The CTAs sharing a step / tile
// (one per r) run together, so each input tile is read from HBM once and from L2
// C times.
constexpr int kGemmThreads = 6 * 32;  // warp 0 loads, warp 1 issues MMAs, warps 2-5 epilogue
constexpr int kBStages = 3;

// XIN: the input is the packed x tile of layer 0 (KP = kx columns, no swizzle, 8-row groups
// KP * 16 bytes apart); otherwise layer l-1's h pieces (KP = H).
template <int KP, bool XIN, int NT>
struct GemmSmem {
  static constexpr int kStage = KP * NT * 2;  // one step's input tile
  static constexpr int kOut = gblock_of(NT);  // one staged gate block (bulk-stored by the epilogue)
  // Input ring kBStages deep and two staged output blocks; a 2-deep ring where that does
  // not fit (K = 512 with 64- or 80-row tiles).
  static constexpr int kStages = kBStages * kStage + 2 * kOut + 4096 <= 232448 ? kBStages : 2;
  static constexpr int kB = 0;
  static constexpr int kO = kB + kStages * kStage;
  static constexpr int kBias = kO + 2 * kOut;
  static constexpr int kBar = kBias + kRows * 4;
  static constexpr int kTmemSlot = kBar + 96;
  static constexpr int kEnd = kBar + 128;
  static constexpr int kDyn = kEnd + 1024;
  static constexpr int kACols = KP / 2;  // W_ih slice: 128 lanes x KP 16-bit values
  static constexpr int kTmemCols = kACols + 2 * NT <= 256 ? 256 : 512;
  static_assert(kDyn <= 232448, "shared memory");
};

struct GemmArgs {
  const uint8_t* xp;    // layer 0: [tiles][T] packed x tiles (64 rows x 16, core matrices)
  const uint8_t* hseq;  // layers >= 1: [T][tiles][C] h pieces of layer l-1
  const uint16_t* wih;  // [4H][KP] this layer's permuted, pre-scaled W_ih
  const float* bias;    // [4H] this layer's permuted, pre-scaled bias
  uint16_t* gates;      // [T][tiles][C][128][kGRow]
  int* status;
  int T, H, tiles;
};

template <int KP, bool BF16, bool XIN, int NT>
__global__ void __launch_bounds__(kGemmThreads, 1) proj_kernel(const GemmArgs a) {
  using S = GemmSmem<KP, XIN, NT>;
  PLSTM_TCL_TILE_CONSTANTS(NT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = ctas_of(a.H);
  const long long jobs = (long long)a.T * a.tiles * C;
  const int r = blockIdx.x % C;  // gridDim.x is a multiple of C: every job of this CTA has the same r
  const int my = blockIdx.x < jobs ? (int)((jobs - blockIdx.x + gridDim.x - 1) / gridDim.x) : 0;
  const unsigned long long kTimeout = 2000000000ull;
  const uint32_t bar = sbase + S::kBar;
  const uint32_t b_full = bar, b_empty = bar + 24, d_full = bar + 48, d_empty = bar + 64;
  float* bias_s = reinterpret_cast<float*>(sm + S::kBias);
  if (tid == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      ptx::mbar_init(b_full + 8 * s, 1);
      ptx::mbar_init(b_empty + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(d_full + 8 * s, 1);
      ptx::mbar_init(d_empty + 8 * s, 4);
    }
    ptx::fence_mbar_init_cluster();
  }
  if (warp == 1) {
    ptx::tmem_alloc(sbase + S::kTmemSlot, S::kTmemCols);
    ptx::tmem_relinquish();
  }
  for (int i = tid; i < kRows; i += kGemmThreads) bias_s[i] = a.bias[r * kRows + i];
  __syncthreads();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + S::kTmemSlot);
  // W_ih slice -> TMEM columns [0, KP / 2): epilogue warp (quadrant q) stores rows 32 q + lane.
  if (warp >= 2) {
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.wih + ((size_t)r * kRows + row) * KP);
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    if (S::kACols % 32 != 0) {  // 8 columns at a time (layer-0 widths that are not a multiple of 64)
#pragma unroll 1
      for (int c = 0; c < S::kACols; c += 8) {
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = src[c + i];
        ptx::tmem_st_32x32b_x8(tmem + lane_off + (uint32_t)c, v);
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < S::kACols; c += 32) {
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 u = reinterpret_cast<const uint4*>(src + c)[i];
          v[4 * i + 0] = u.x;
          v[4 * i + 1] = u.y;
          v[4 * i + 2] = u.z;
          v[4 * i + 3] = u.w;
        }
        ptx::tmem_st_32x32b_x32(tmem + lane_off + (uint32_t)c, v);
      }
    }
    ptx::tmem_wait_st();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  auto job_src = [&](int k, int* t_out, int* tile_out) -> const uint8_t* {
    const long long j = blockIdx.x + (long long)k * gridDim.x;
    const long long ts = j / C;
    const int t = (int)(ts / a.tiles), tile = (int)(ts % a.tiles);
    *t_out = t;
    *tile_out = tile;
    if (XIN) return a.xp + ((size_t)tile * a.T + t) * (size_t)(kNT * KP * 2);
    return a.hseq + ((size_t)t * a.tiles + tile) * (size_t)C * kPiece;
  };

  if (warp == 0) {
    // ---------------- loads ----------------
    if (lane == 0) {
      for (int k = 0; k < my; ++k) {
        const int s = k % S::kStages;
        if (k >= S::kStages && !wait_bar(b_empty + 8 * s, ((k / S::kStages) - 1) & 1, nullptr, kTimeout)) {
          report_status(a.status, PLSTM_ETIMEOUT, 0x7ffe0000);
          break;
        }
        int t, tile;
        const uint8_t* src = job_src(k, &t, &tile);
        ptx::mbar_arrive_expect_tx(b_full + 8 * s, S::kStage);
        ptx::bulk_g2s(sbase + S::kB + s * S::kStage, src, S::kStage, b_full + 8 * s);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    constexpr uint32_t idesc = ptx::idesc_f16(128, kNT, BF16);
    for (int k = 0; k < my; ++k) {
      const int s = k % S::kStages, db = k & 1;
      int w = 1;
      if (lane == 0) {
        if (k >= 2) w = wait_bar(d_empty + 8 * db, ((k - 2) >> 1) & 1, nullptr, kTimeout) ? 1 : 0;
        if (w) w = wait_bar(b_full + 8 * s, (k / S::kStages) & 1, nullptr, kTimeout) ? 1 : 0;
      }
      if (!__shfl_sync(0xffffffffu, w, 0)) break;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(S::kACols + db * kNT);
        const uint32_t b0 = sbase + S::kB + s * S::kStage;
        if (XIN) {
#pragma unroll
          for (int i = 0; i < KP / 16; ++i)
            ptx::mma_f16_ts(d, tmem + (uint32_t)(8 * i), ptx::desc_k_none(b0 + (uint32_t)(256 * i), 128, KP * 16), idesc,
                            i != 0 ? 1u : 0u);
        } else {
#pragma unroll 4
          for (int i = 0; i < KP / 16; ++i)
            ptx::mma_f16_ts(d, tmem + (uint32_t)(8 * i), ptx::desc_k_none(b0 + (uint32_t)(2 * i * kKG), kKG, 128),
                            idesc, i != 0 ? 1u : 0u);
        }
        ptx::mma_commit(b_empty + 8 * s);
        ptx::mma_commit(d_full + 8 * db);
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue: lane = gate row, columns = the tile's batch rows ----------------
    // Each job's gate block (128 rows x kGRow, contiguous in global memory) is staged in
    // shared memory and written with one bulk copy (two staging buffers).
    const int q = warp & 3;
    const int row = 32 * q + lane;
    // Every epilogue warp runs all `my` iterations and both named barriers of each (after a
    // timed-out wait it only skips the work), so no warp is left waiting on the others.
    const bool issuer = warp == 2 && lane == 0;
    const float bv = bias_s[row];
    bool ok = true;
    for (int k = 0; k < my; ++k) {
      const int db = k & 1;
      uint8_t* ob = sm + S::kO + db * S::kOut;
      if (k >= 2) {  // staging buffer db was last bulk-stored two jobs ago
        if (issuer) ptx::bulk_wait_group_read<1>();
        ptx::named_bar_sync(1, 128);
      }
      if (ok && !wait_bar(d_full + 8 * db, (k >> 1) & 1, nullptr, kTimeout)) {
        ok = false;
        if (lane == 0) report_status(a.status, PLSTM_ETIMEOUT, 0x7ffd0000);
      }
      if (!ok) {
        ptx::named_bar_sync(1, 128);
        continue;
      }
      ptx::tc_fence_after();
      uint32_t v[kNT];
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(S::kACols + db * kNT);
#pragma unroll
      for (int c = 0; c < kNT; c += 16) ptx::tmem_ld_32x32b_x16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(&v[c]));
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(d_empty + 8 * db);
      int t, tile;
      job_src(k, &t, &tile);
      uint4* dst = reinterpret_cast<uint4*>(ob + (size_t)row * kGRow * 2);
#pragma unroll
      for (int c = 0; c < kNT / 8; ++c) {
        uint4 o;
        o.x = pack2_bits<BF16>(__uint_as_float(v[8 * c + 0]) + bv, __uint_as_float(v[8 * c + 1]) + bv);
        o.y = pack2_bits<BF16>(__uint_as_float(v[8 * c + 2]) + bv, __uint_as_float(v[8 * c + 3]) + bv);
        o.z = pack2_bits<BF16>(__uint_as_float(v[8 * c + 4]) + bv, __uint_as_float(v[8 * c + 5]) + bv);
        o.w = pack2_bits<BF16>(__uint_as_float(v[8 * c + 6]) + bv, __uint_as_float(v[8 * c + 7]) + bv);
        dst[c] = o;
      }
      ptx::fence_proxy_async_smem();
      ptx::named_bar_sync(1, 128);
      if (issuer && ok) {
        ptx::bulk_s2g(a.gates + (((size_t)t * a.tiles + tile) * C + r) * kRows * kGRow, ptx::smem_u32(ob),
                      (uint32_t)S::kOut);
        ptx::bulk_commit_group();
      }
    }
    if (issuer) ptx::bulk_wait_group_all();  // stores complete before the CTA's shared memory goes away
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ---- recurrence -----------------------------------------------------------------------
template <int H, int NCW, int NT>
struct RecSmem {
  static constexpr int C = H / kU;
  static constexpr int kTile = H * NT * 2;   // one h tile (all units x NT rows)
  static constexpr int kB = 0;               // h tiles, double-buffered by step parity
  static constexpr int kG = kB + 2 * kTile;  // gate blocks: a ring of kGS (3, or 2 if 3 do not fit)
  static constexpr int kGS = 2 * kTile + 3 * gblock_of(NT) + 2048 <= 232448 ? 3 : 2;
  static constexpr int kBar = kG + kGS * gblock_of(NT);
  // barriers: full_rec[2] @0, mma[2] @16, hready[2] @32, gfull[3] @48
  static constexpr int kTmemSlot = kBar + 80, kAbort = kBar + 84, kDone = kBar + 88;
  static constexpr int kPerm = kBar + 128, kLens = kPerm + 4 * NT;
  static constexpr int kEnd = kLens + 4 * NT;
  static constexpr int kDyn = kEnd + 1024;
  static constexpr int kComputeWarps = NCW;  // NCW / 4 per TMEM lane quadrant, 256 / NCW columns each
  // + the control warp (own-piece MMAs and the first half of the peer-piece MMAs) + the helper
  // warp (the second half, into its own accumulator).
  static constexpr int kThreads = (kComputeWarps + 2) * 32;
  static constexpr int kACols = H / 2;  // W_hh slice: 128 lanes x H 16-bit values
  static constexpr int kD = kACols;     // gate accumulator [128 x NT] (single buffer)
  static constexpr int kD1 = kD + NT;   // the helper warp's partial accumulator [128 x NT]
  static constexpr int kX = kD1 + NT;   // layer 0's W_ih slice (fused input projection, kx / 2 <= 64 columns)
  static constexpr int kTmemCols = kX + kMaxXK / 2 <= 256 ? 256 : 512;
  static_assert(kX + kMaxXK / 2 <= 512, "tensor memory");
  static_assert(kDyn <= 232448, "shared memory");
};

struct RecArgs {
  const uint8_t* whh;      // this layer's W_hh images [C][128][H]
  const uint16_t* gates;   // [T][tiles][C][128][kGRow] (unless xp is set)
  // Layer 0 with its input projection fused in (no gate blocks): packed x tiles [tiles][T]
  // (NT rows x kx, core matrices), the layer's W_ih image [4H][kx] and f32 bias [4H]; else null.
  const uint8_t* xp;
  const uint16_t* wih0;
  const float* bias0;
  int kx;
  const int32_t* perm;     // [tiles * kNT]
  const int32_t* lengths;  // [B] or null
  const int32_t* tile_len; // [tiles]
  const void* h0;          // [L][B][H] or null
  const void* c0;
  uint8_t* hseq;           // [T][tiles][C] pieces, or null
  void* h_n;               // [L][B][H] or null
  void* c_n;
  uint16_t* hlast;         // [B][H] (last layer, Linear input) or null
  int* status;
  int B, T, layer, flags;
  int hid;                 // the model's hidden size (<= H): h0 / c0 / h_n / c_n rows are hid wide
  unsigned long long timeout_ns;
  unsigned long long* trace;  // PLSTM_FLAG_TRACE: [C][64][8] clock64 stamps of cluster 0, or null
  int trace_t0;
};

// Trace events (steps trace_t0 .. +63 of cluster 0): control warp 0 peer pieces of
// h_{t-1} landed, 1 peer MMAs + commit issued, 2 compute warps done with step t,
// 3 own-piece MMAs of step t+1 issued; compute warp 0: 4 accumulator ready,
// 5 loaded, 6 h written; 7 the step's pusher issued its copies.
constexpr int kTraceSteps = 64, kTraceEvents = 8;
__device__ __forceinline__ void trace_mark(const RecArgs& a, int tile, int r, int t, int ev) {
  if (a.trace != nullptr && tile == 0 && t >= a.trace_t0 && t < a.trace_t0 + kTraceSteps)
    a.trace[((size_t)r * kTraceSteps + (t - a.trace_t0)) * kTraceEvents + ev] = clock64();
}

__device__ __forceinline__ void rec_abort(const RecArgs& a, uint8_t* sm_abort, int ncta, int step) {
  const uint32_t local = ptx::smem_u32(sm_abort);
  for (int r = 0; r < ncta; ++r) ptx::st_cluster_u32(ptx::mapa(local, (uint32_t)r), 1u);
  report_status(a.status, PLSTM_ETIMEOUT, (int)((blockIdx.x & 0x7fff) << 16) | (step & 0xffff));
}

template <int H, int NCW, bool BF16, bool VARLEN, int NT>
__global__ void __launch_bounds__(RecSmem<H, NCW, NT>::kThreads, NT <= 32 ? 2 : 1) rec_kernel(const RecArgs a) {
  using S = RecSmem<H, NCW, NT>;
  PLSTM_TCL_TILE_CONSTANTS(NT);
  constexpr int C = S::C;
  constexpr int GS = S::kGS;
  constexpr int CPW = kNT * 4 / (NCW * 8);  // 8-column chunks per compute warp
  static_assert(CPW * NCW * 8 == kNT * 4, "tile rows must split evenly over the compute warps");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = (int)ptx::cluster_ctarank();
  const int tile = blockIdx.x / C;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kAbort);
  int32_t* perm_s = reinterpret_cast<int32_t*>(sm + S::kPerm);
  int32_t* lens_s = reinterpret_cast<int32_t*>(sm + S::kLens);
  const uint32_t bar_rec = sbase + S::kBar, bar_mma = bar_rec + 16, bar_hready = bar_rec + 32,
                 bar_g = bar_rec + 48;
  auto bbuf = [&](int b) -> uint32_t { return sbase + (uint32_t)(S::kB + b * S::kTile); };
  auto gslot = [&](int s) -> uint32_t { return sbase + (uint32_t)(S::kG + s * kGBlock); };
  const int l = a.layer;

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar_rec + 8 * b, 1);
      ptx::mbar_init(bar_mma + 8 * b, 2);  // the control and the helper warp's commits
      ptx::mbar_init(bar_hready + 8 * b, S::kComputeWarps);
    }
    for (int s = 0; s < GS; ++s) ptx::mbar_init(bar_g + 8 * s, 1);
    *abort_flag = 0;
    *reinterpret_cast<uint32_t*>(sm + S::kDone) = 0;
    ptx::fence_mbar_init_cluster();
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + S::kTmemSlot, S::kTmemCols);
    ptx::tmem_relinquish();
  }
  for (int i = tid; i < kNT; i += S::kThreads) {
    const int b = a.perm[tile * kNT + i];
    perm_s[i] = b;
    int len = 0;
    if (b >= 0) len = VARLEN ? min(max(a.lengths[b], 0), a.T) : a.T;
    lens_s[i] = len;
  }
  __syncthreads();
  // h_{-1} = h0 (all units of the tile's rows) -> h tile buffer 0.
  for (int i = tid; i < kNT * H; i += S::kThreads) {
    const int n = i / H, k = i % H;
    uint16_t v = 0;
    const int b = perm_s[n];
    if (a.h0 != nullptr && b >= 0 && k < a.hid) v = static_cast<const uint16_t*>(a.h0)[((size_t)l * a.B + b) * a.hid + k];
    *reinterpret_cast<uint16_t*>(sm + S::kB + hoff<NT>(k, n)) = v;
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + S::kTmemSlot);
  // W_hh slice -> TMEM columns [0, H / 2): warp q < 4 stores its quadrant's 32 rows.
  if (warp < 4) {
    const int row = 32 * warp + lane;
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const uint4* src = reinterpret_cast<const uint4*>(a.whh + ((size_t)r * kRows + row) * H * 2);
#pragma unroll 1
    for (int c = 0; c < H / 2; c += 32) {
      uint32_t v[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 u = src[c / 4 + i];
        v[4 * i + 0] = u.x;
        v[4 * i + 1] = u.y;
        v[4 * i + 2] = u.z;
        v[4 * i + 3] = u.w;
      }
      ptx::tmem_st_32x32b_x32(tmem + lane_off + (uint32_t)c, v);
    }
    if (a.xp != nullptr) {  // layer 0's W_ih slice [128 x kx] -> columns [kX, kX + kx / 2)
      const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(a.wih0 + ((size_t)r * kRows + row) * a.kx);
#pragma unroll 1
      for (int c = 0; c < a.kx / 2; c += 8) {
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = wsrc[c + i];
        ptx::tmem_st_32x32b_x8(tmem + lane_off + (uint32_t)(S::kX + c), v);
      }
    }
    ptx::tmem_wait_st();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::cluster_sync();  // every CTA's barriers are initialised before any remote copy

  const int Tt = a.tile_len[tile];
  const uint32_t dcol = tmem + (uint32_t)S::kD, dcol1 = tmem + (uint32_t)S::kD1;
  // The peer-piece MMAs of a step, K steps j in [0, H / 16) but this CTA's own two (units [32 r,
  // 32 r + 32)), are issued by two warps in parallel (one thread issues an MMA every ~45-100
  // cycles): index i < kHalfO by the control warp into D, the rest by the helper warp into D1,
  // which the compute warps add.  Each accumulator sums its K steps in a fixed order.
  constexpr int kOthers = H / 16 - 2, kHalfO = kOthers / 2;
  auto kstep = [&](int i) { return i < 2 * r ? i : i + 2; };
  // Each step's input block, prefetched GS steps ahead into the gate ring: the projected gate block,
  // or with the fused layer-0 projection the step's x tile (the input MMAs' B operand).
  const bool fused_x = a.xp != nullptr;
  const uint32_t blk_bytes = fused_x ? (uint32_t)(kNT * a.kx * 2) : (uint32_t)kGBlock;
  auto gates_src = [&](int t) -> const uint8_t* {
    if (fused_x) return a.xp + ((size_t)tile * a.T + t) * (size_t)blk_bytes;
    return reinterpret_cast<const uint8_t*>(a.gates) + (((size_t)t * gridDim.x / C + tile) * C + r) * (size_t)kGBlock;
  };

  if (warp == S::kComputeWarps) {
    // ============================ control warp ============================
    constexpr uint32_t idesc = ptx::idesc_f16(128, kNT, BF16);
    const uint32_t rec_bytes = (uint32_t)(C - 1) * kPiece;
    // One MMA covers K = 16 units = two 8-unit K groups (kKG bytes apart).
    auto issue = [&](int t, int j0, int j1, bool init) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        for (int j = j0; j < j1; ++j) {
          const uint64_t dB = ptx::desc_k_none(bbuf(b) + (uint32_t)(2 * j * kKG), kKG, 128);
          ptx::mma_f16_ts(dcol, tmem + (uint32_t)(8 * j), dB, idesc, (init && j == j0) ? 0u : 1u);
        }
      }
      __syncwarp();
    };
    auto issue_others = [&](int t) {  // the control warp's half of the peer-piece K steps, into D
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        for (int i = 0; i < kHalfO; ++i) {
          const int j = kstep(i);
          const uint64_t dB = ptx::desc_k_none(bbuf(b) + (uint32_t)(2 * j * kKG), kKG, 128);
          ptx::mma_f16_ts(dcol, tmem + (uint32_t)(8 * j), dB, idesc, 1u);
        }
      }
      __syncwarp();
    };
    auto commit = [&](int t) {
      if (ptx::elect_one()) ptx::mma_commit(bar_mma + 8 * (t & 1));
      __syncwarp();
    };
    auto load_gates = [&](int t) {
      if (ptx::elect_one()) {
        const int s = t % GS;
        ptx::mbar_arrive_expect_tx(bar_g + 8 * s, blk_bytes);
        ptx::bulk_g2s(gslot(s), gates_src(t), blk_bytes, bar_g + 8 * s);
      }
      __syncwarp();
    };
    // Fused layer 0: D = W_ih . x_t (kx / 16 MMAs, initialising D) once the x tile has landed; the
    // own-piece MMAs then accumulate.
    auto issue_x = [&](int t) -> bool {
      if (!fused_x) return true;
      const int s = t % GS;
      if (!warp_wait(bar_g + 8 * s, (t / GS) & 1, abort_flag, a.timeout_ns)) return false;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        for (int i = 0; i < a.kx / 16; ++i)
          ptx::mma_f16_ts(dcol, tmem + (uint32_t)(S::kX + 8 * i),
                          ptx::desc_k_none(gslot(s) + (uint32_t)(256 * i), 128, (uint32_t)(a.kx * 16)), idesc,
                          i != 0 ? 1u : 0u);
      }
      __syncwarp();
      return true;
    };
    bool ok = true;
    auto fail = [&](int t) {
      if (ptx::elect_one()) rec_abort(a, sm + S::kAbort, C, t);
      __syncwarp();
      ok = false;
    };
    if (Tt > 0) {
      for (int t = 0; t < GS && t < Tt; ++t) load_gates(t);
      if (ptx::elect_one())
        for (int t = 1; t <= 2 && t < Tt; ++t) ptx::mbar_arrive_expect_tx(bar_rec + 8 * (t & 1), rec_bytes);
      __syncwarp();
      // Step 0 runs on h0, already complete in buffer 0.
      if (!issue_x(0)) fail(0);
      issue(0, 2 * r, 2 * r + 2, !fused_x);
      issue_others(0);
      commit(0);
    }
    for (int t = 0; ok && t < Tt; ++t) {
      const int b = t & 1;
      if (t >= 1) {
        if (!warp_wait(bar_rec + 8 * b, ((t - 1) >> 1) & 1, abort_flag, a.timeout_ns)) {
          fail(t);
          break;
        }
        if (lane == 0) trace_mark(a, tile, r, t, 0);
        if (t + 2 < Tt && ptx::elect_one()) ptx::mbar_arrive_expect_tx(bar_rec + 8 * b, rec_bytes);
        __syncwarp();
        issue_others(t);
        commit(t);
        if (lane == 0) trace_mark(a, tile, r, t, 1);
      }
      // Compute warps done with step t: its gate block slot and accumulator are free,
      // h(t)'s own piece is written (buffer b ^ 1).
      if (!warp_wait(bar_hready + 8 * b, (t >> 1) & 1, abort_flag, a.timeout_ns)) {
        fail(t);
        break;
      }
      if (lane == 0) trace_mark(a, tile, r, t, 2);
      if (t + 1 < Tt) {
        if (!issue_x(t + 1)) {
          fail(t + 1);
          break;
        }
        issue(t + 1, 2 * r, 2 * r + 2, !fused_x);
        if (lane == 0) trace_mark(a, tile, r, t, 3);
      }
    }
  } else if (warp == S::kComputeWarps + 1) {
    // ============================ helper warp ==============================
    // The second half of each step's peer-piece MMAs into D1: once the peers' pieces have landed
    // and the compute warps have loaded D1 of the previous step.
    constexpr uint32_t idesc = ptx::idesc_f16(128, kNT, BF16);
    for (int t = 0; t < Tt; ++t) {
      const int b = t & 1;
      if (t >= 1 && (!warp_wait(bar_rec + 8 * b, ((t - 1) >> 1) & 1, abort_flag, a.timeout_ns) ||
                     !warp_wait(bar_hready + 8 * ((t - 1) & 1), ((t - 1) >> 1) & 1, abort_flag, a.timeout_ns))) {
        if (ptx::elect_one()) rec_abort(a, sm + S::kAbort, C, t);
        __syncwarp();
        break;
      }
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        for (int i = kHalfO; i < kOthers; ++i) {
          const int j = kstep(i);
          const uint64_t dB = ptx::desc_k_none(bbuf(b) + (uint32_t)(2 * j * kKG), kKG, 128);
          ptx::mma_f16_ts(dcol1, tmem + (uint32_t)(8 * j), dB, idesc, i > kHalfO ? 1u : 0u);
        }
        ptx::mma_commit(bar_mma + 8 * b);
      }
      __syncwarp();
    }
  } else {
    // ============================ compute warps ============================
    const int q = warp & 3, cg = warp >> 2;  // TMEM lane quadrant, column group
    const int j8 = lane >> 2, cpair = (lane & 3) * 2;
    const int n0 = 8 * CPW * cg;
    const int ul = 8 * q + j8;  // unit within this CTA's 32
    const int u = kU * r + ul;  // unit within the layer
    float bias_x[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // fused layer 0: f32 bias of this thread's four gate rows
    if (fused_x) {
#pragma unroll
      for (int g = 0; g < 4; ++g) bias_x[g] = a.bias0[r * kRows + 32 * q + 8 * g + j8];
    }
    float c_st[CPW][2];
    uint16_t h_st[CPW][2];
    int len_c[CPW][2], bidx[CPW][2];
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = n0 + 8 * jc + cpair + e;
        const int bb = perm_s[n];
        bidx[jc][e] = bb;
        len_c[jc][e] = lens_s[n];
        uint16_t hv = 0;
        float cv = 0.0f;
        if (bb >= 0 && a.h0 != nullptr && u < a.hid) {
          hv = static_cast<const uint16_t*>(a.h0)[((size_t)l * a.B + bb) * a.hid + u];
          cv = from_bits<BF16>(static_cast<const uint16_t*>(a.c0)[((size_t)l * a.B + bb) * a.hid + u]);
        }
        h_st[jc][e] = hv;
        c_st[jc][e] = cv;
      }
    for (int t = 0; t < Tt; ++t) {
      const int b = t & 1, gs = t % GS;
      if (*abort_flag) break;
      if ((!fused_x && !wait_bar(bar_g + 8 * gs, (t / GS) & 1, abort_flag, a.timeout_ns)) ||
          !wait_bar(bar_mma + 8 * b, (t >> 1) & 1, abort_flag, a.timeout_ns)) {
        if (lane == 0) rec_abort(a, sm + S::kAbort, C, t);
        break;
      }
      ptx::tc_fence_after();
      if (warp == 0 && lane == 0) trace_mark(a, tile, r, t, 4);
      uint32_t rif[4 * CPW], rgo[4 * CPW];
      const uint32_t lo = (uint32_t)(32 * q) << 16, hi = (uint32_t)(32 * q + 16) << 16;
#pragma unroll
      for (int i = 0; i < CPW / 4; ++i) {
        ptx::tmem_ld_16x256b_x4(dcol + lo + (uint32_t)(n0 + 32 * i), *reinterpret_cast<uint32_t(*)[16]>(&rif[16 * i]));
        ptx::tmem_ld_16x256b_x4(dcol + hi + (uint32_t)(n0 + 32 * i), *reinterpret_cast<uint32_t(*)[16]>(&rgo[16 * i]));
      }
      if (CPW % 4 != 0) {  // 80-row tiles: 5 chunks per warp
        constexpr int c0 = CPW / 4 * 4;
#pragma unroll
        for (int c = c0; c < CPW; ++c) {
          ptx::tmem_ld_16x256b_x1(dcol + lo + (uint32_t)(n0 + 8 * c), *reinterpret_cast<uint32_t(*)[4]>(&rif[4 * c]));
          ptx::tmem_ld_16x256b_x1(dcol + hi + (uint32_t)(n0 + 8 * c), *reinterpret_cast<uint32_t(*)[4]>(&rgo[4 * c]));
        }
      }
      ptx::tmem_wait_ld();
      {  // + the helper warp's partial accumulator
        uint32_t p1[4 * CPW], p2[4 * CPW];
#pragma unroll
        for (int i = 0; i < CPW / 4; ++i) {
          ptx::tmem_ld_16x256b_x4(dcol1 + lo + (uint32_t)(n0 + 32 * i), *reinterpret_cast<uint32_t(*)[16]>(&p1[16 * i]));
          ptx::tmem_ld_16x256b_x4(dcol1 + hi + (uint32_t)(n0 + 32 * i), *reinterpret_cast<uint32_t(*)[16]>(&p2[16 * i]));
        }
        if (CPW % 4 != 0) {
          constexpr int c0 = CPW / 4 * 4;
#pragma unroll
          for (int c = c0; c < CPW; ++c) {
            ptx::tmem_ld_16x256b_x1(dcol1 + lo + (uint32_t)(n0 + 8 * c), *reinterpret_cast<uint32_t(*)[4]>(&p1[4 * c]));
            ptx::tmem_ld_16x256b_x1(dcol1 + hi + (uint32_t)(n0 + 8 * c), *reinterpret_cast<uint32_t(*)[4]>(&p2[4 * c]));
          }
        }
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4 * CPW; ++i) {
          rif[i] = __float_as_uint(__uint_as_float(rif[i]) + __uint_as_float(p1[i]));
          rgo[i] = __float_as_uint(__uint_as_float(rgo[i]) + __uint_as_float(p2[i]));
        }
      }
      ptx::tc_fence_before();
      if (warp == 0 && lane == 0) trace_mark(a, tile, r, t, 5);
      // Projected input + bias of the four gates of this thread's cells (with the fused layer-0
      // projection the accumulator holds the input part, and the f32 bias is added here).
      const uint8_t* gsl = sm + S::kG + gs * kGBlock;
      float pre[4][CPW][2];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const uint8_t* grow = gsl + (size_t)(32 * q + 8 * g + j8) * kGRow * 2;
#pragma unroll
        for (int jc = 0; jc < CPW; ++jc) {
          const float2 gv = fused_x ? make_float2(bias_x[g], bias_x[g])
                                    : from_bits2<BF16>(*reinterpret_cast<const uint32_t*>(grow + (n0 + 8 * jc + cpair) * 2));
          const uint32_t* acc = g < 2 ? rif : rgo;
          const int base = 4 * jc + (g & 1) * 2;
          pre[g][jc][0] = __uint_as_float(acc[base]) + gv.x;
          pre[g][jc][1] = __uint_as_float(acc[base + 1]) + gv.y;
        }
      }
      uint8_t* dst = sm + S::kB + (b ^ 1) * S::kTile;
      // The layer's h sequence (the next layer's projection input, or the output).
      uint8_t* gdst = a.hseq != nullptr ? a.hseq + ((size_t)t * (gridDim.x / C) + tile) * (size_t)C * kPiece : nullptr;
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc) {
        float h[2], cn[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float ti = ptx::tanh_approx(pre[0][jc][e]), tf = ptx::tanh_approx(pre[1][jc][e]);
          const float tg = ptx::tanh_approx(pre[2][jc][e]), to = ptx::tanh_approx(pre[3][jc][e]);
          cn[e] = fmaf(fmaf(0.5f, tf, 0.5f), c_st[jc][e], fmaf(0.5f, ti, 0.5f) * tg);
          h[e] = fmaf(0.5f, to, 0.5f) * ptx::tanh_approx(cn[e]);
        }
        const uint32_t bits = pack2_bits<BF16>(h[0], h[1]);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (!VARLEN || t < len_c[jc][e]) {
            c_st[jc][e] = cn[e];
            h_st[jc][e] = (uint16_t)(e == 0 ? bits & 0xffffu : bits >> 16);
          }
          *reinterpret_cast<uint16_t*>(dst + hoff<NT>(u, n0 + 8 * jc + cpair + e)) = h_st[jc][e];
        }
      }
      ptx::fence_proxy_async_smem();
      if (warp == 0 && lane == 0) trace_mark(a, tile, r, t, 6);
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(bar_hready + 8 * b);
        // The last warp to finish pushes the piece to the peers (acquire-release
        // counter: the other warps' writes, fenced for the async proxy, come first).
        // It then prefetches the gate block of step t + GS into this step's slot
        // (after the pushes: they are on the critical path).
        if (t + 1 < Tt && ptx::atom_add_acq_rel_smem(sbase + S::kDone, 1u) % (uint32_t)S::kComputeWarps ==
                              (uint32_t)S::kComputeWarps - 1u) {
          const uint32_t piece = bbuf(b ^ 1) + (uint32_t)(r * kPiece);
          for (int pr = 0; pr < C; ++pr) {
            if (pr == r) continue;
            ptx::bulk_s2c(ptx::mapa(piece, (uint32_t)pr), piece, kPiece,
                          ptx::mapa(bar_rec + 8 * (b ^ 1), (uint32_t)pr));
          }
          if (t + GS < Tt) {
            ptx::mbar_arrive_expect_tx(bar_g + 8 * gs, blk_bytes);
            ptx::bulk_g2s(gslot(gs), gates_src(t + GS), blk_bytes, bar_g + 8 * gs);
          }
          trace_mark(a, tile, r, t, 7);
        }
      }
      // The layer's h sequence, after the step's arrivals: a release arrive (and the pusher's
      // acquire-release counter) would first wait for these global stores to complete.
      if (gdst != nullptr) {
#pragma unroll
        for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            *reinterpret_cast<uint16_t*>(gdst + hoff<NT>(u, n0 + 8 * jc + cpair + e)) = h_st[jc][e];
      }
    }
    // Final state of this CTA's units.
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int bb = bidx[jc][e];
        if (bb < 0) continue;
        if (a.hlast != nullptr) a.hlast[(size_t)bb * H + u] = h_st[jc][e];
        if (u >= a.hid) continue;
        const size_t idx = ((size_t)l * a.B + bb) * a.hid + u;
        if (a.h_n != nullptr) static_cast<uint16_t*>(a.h_n)[idx] = h_st[jc][e];
        if (a.c_n != nullptr) {
          if (a.flags & PLSTM_FLAG_CN_F32)
            static_cast<float*>(a.c_n)[idx] = c_st[jc][e];
          else
            static_cast<uint16_t*>(a.c_n)[idx] = to_bits<BF16>(c_st[jc][e]);
        }
      }
  }

  if (*abort_flag) {
    const unsigned long long t0 = ptx::globaltimer();
    while (ptx::globaltimer() - t0 < 50000ull) {
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, S::kTmemCols);
  }
  ptx::cluster_sync();
}

// ---- outputs -------------------------------------------------------------------------
// out[b][o] = b_lin[o] + W_lin[o] . h_last[b]
template <bool BF16>
__global__ void linear_last_kernel(const uint16_t* __restrict__ hlast, const uint16_t* __restrict__ wlin,
                                   const float* __restrict__ blin, uint16_t* __restrict__ out, int B, int H, int O) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * O; i += gridDim.x * blockDim.x) {
    const int b = i / O, o = i % O;
    float acc = 0.0f;
    for (int k = 0; k < H; k += 2) {
      const float2 hv = from_bits2<BF16>(*reinterpret_cast<const uint32_t*>(hlast + (size_t)b * H + k));
      const float2 wv = from_bits2<BF16>(*reinterpret_cast<const uint32_t*>(wlin + (size_t)o * H + k));
      acc = fmaf(hv.x, wv.x, acc);
      acc = fmaf(hv.y, wv.y, acc);
    }
    out[i] = to_bits<BF16>(acc + blin[o]);
  }
}

// One block per (step, tile): the tile's h from its C pieces, then either the Linear
// head (out[b][t][o]) or the h sequence itself (out[b][t][u]); zero past each length.
template <bool BF16, bool LINEAR, int NT>
__global__ void seq_out_kernel(const uint8_t* __restrict__ hseq, const int32_t* __restrict__ perm,
                               const int32_t* __restrict__ lengths, const uint16_t* __restrict__ wlin,
                               const float* __restrict__ blin, uint16_t* __restrict__ out, int B, int T, int H,
                               int O, int tiles, int out_seq_major, int hid) {
  PLSTM_TCL_TILE_CONSTANTS(NT);
  extern __shared__ uint8_t smem_o[];
  float* hs = reinterpret_cast<float*>(smem_o);  // [kNT][H + 1]
  const int C = ctas_of(H);
  const int t = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const uint8_t* base = hseq + ((size_t)t * tiles + tile) * (size_t)C * kPiece;
  for (int i = threadIdx.x; i < kNT * H; i += blockDim.x) {
    const int n = i / H, k = i % H;
    hs[n * (H + 1) + k] = from_bits<BF16>(*reinterpret_cast<const uint16_t*>(
        base + (size_t)(k >> 3) * kKG + (n >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2));
  }
  __syncthreads();
  const int W = LINEAR ? O : hid;  // h-sequence output rows are the model's hid units
  for (int i = threadIdx.x; i < kNT * W; i += blockDim.x) {
    const int n = i / W, w = i % W;
    const int b = perm[tile * kNT + n];
    if (b < 0) continue;
    const int len = lengths != nullptr ? min(max(lengths[b], 0), T) : T;
    float v = 0.0f;
    if (t < len) {
      if (LINEAR) {
        float acc = blin[w];
        for (int k = 0; k < H; ++k) acc = fmaf(hs[n * (H + 1) + k], from_bits<BF16>(wlin[(size_t)w * H + k]), acc);
        v = acc;
      } else {
        v = hs[n * (H + 1) + w];
      }
    }
    const size_t row = out_seq_major ? (size_t)t * B + b : (size_t)b * T + t;
    out[row * W + w] = to_bits<BF16>(v);
  }
}

// ---- hidden update (plstm_hidden_update) ------------------------------------------------
// W_hh [4H][H] in any PLSTM_W_* layout -> the recurrence's TMEM images [C][128][H]
// (rows permuted per CTA, i / f / o pre-scaled by 1/2).
__global__ void hu_pack_whh_kernel(const void* w_hh, int dtype, int layout, int H, uint16_t* img) {
  const int G = 4 * H;
  const bool bf16 = dtype == PLSTM_BF16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)G * H;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int rp = (int)(i / H), k = (int)(i % H);
    const int r = rp / kRows, rho = rp % kRows;
    const float v = load_any(w_hh, dtype, weight_src_index(layout, G, H, src_row(H, r, rho), k)) * row_scale(rho);
    __half hv = __float2half_rn(v);
    __nv_bfloat16 bv = __float2bfloat16_rn(v);
    img[i] = bf16 ? *reinterpret_cast<uint16_t*>(&bv) : *reinterpret_cast<uint16_t*>(&hv);
  }
}

// gate_proj [B][T][4H] (or [T][B][4H]) + bias -> gate blocks [T][tiles][C][128][kGRow]
// (rows permuted per CTA and pre-scaled like the weights; padding rows zero).  One
// block per (step, tile, CTA): reads 64 rows x 4 runs of 32 gate values, writes the
// 128 x 64 block row by row.
template <bool BF16, int NT>
__global__ void hu_gates_kernel(const uint16_t* __restrict__ gp, const uint16_t* __restrict__ bias, int B, int T,
                                int H, int tiles, int seq_major, uint16_t* __restrict__ gates) {
  PLSTM_TCL_TILE_CONSTANTS(NT);
  __shared__ float blk[kRows][NT + 1];
  const int C = ctas_of(H);
  const int r = blockIdx.x % C;
  const int ts = blockIdx.x / C;
  const int t = ts / tiles, tile = ts % tiles;
  for (int i = threadIdx.x; i < kNT * kRows; i += blockDim.x) {
    const int n = i / kRows, rho = i % kRows;  // rho fastest: 32-value runs are contiguous in gate_proj
    const int b = tile * kNT + n;
    const int sr = src_row(H, r, rho);
    float v = 0.0f;
    if (b < B) {
      const size_t row = seq_major ? (size_t)t * B + b : (size_t)b * T + t;
      v = from_bits<BF16>(gp[row * 4 * H + sr]);
      if (bias != nullptr) v += from_bits<BF16>(bias[sr]);
      v *= row_scale(rho);
    }
    blk[rho][n] = v;
  }
  __syncthreads();
  uint16_t* dst = gates + (((size_t)ts * C + r) * kRows) * kGRow;
  for (int i = threadIdx.x; i < kRows * kNT / 2; i += blockDim.x) {
    const int rho = i / (kNT / 2), n = (i % (kNT / 2)) * 2;
    *reinterpret_cast<uint32_t*>(dst + (size_t)rho * kGRow + n) = pack2_bits<BF16>(blk[rho][n], blk[rho][n + 1]);
  }
}

struct HuWs {
  size_t perm, tile_len, whh, gates, hseq, total;
};
HuWs hu_ws(const HuProblem& p, int nt) {
  HuWs w;
  const int tiles = (p.B + nt - 1) / nt;
  const int C = ctas_of(p.H);
  size_t off = kStatusBytes;
  w.perm = off;
  off = align_up(off + (size_t)tiles * nt * 4, 256);
  w.tile_len = off;
  off = align_up(off + (size_t)tiles * 4, 256);
  w.whh = off;
  off = align_up(off + (size_t)4 * p.H * p.H * 2, 256);
  w.gates = off;
  off = align_up(off + (size_t)p.T * tiles * C * gblock_of(nt), 256);
  w.hseq = off;
  if (p.write_seq()) off = align_up(off + (size_t)p.T * tiles * C * piece_of(nt), 256);
  w.total = off;
  return w;
}

// ---- host side -------------------------------------------------------------------------
struct Ws {
  size_t perm, tile_len, hist, sorted, xp, gates, hseq, hlast, trace, total;
};

// nt: batch rows per tile (64 or 80).
Ws ws_layout(const Problem& p, int nt) {
  Ws w;
  const int tiles = (p.B + nt - 1) / nt;
  const int C = ctas_of(p.H);
  size_t off = kStatusBytes;
  w.perm = off;
  off = align_up(off + (size_t)tiles * nt * 4, 256);
  w.tile_len = off;
  off = align_up(off + (size_t)tiles * 4, 256);
  w.hist = off;
  off = align_up(off + (size_t)(p.T + 1) * 4, 256);
  w.sorted = off;
  off = align_up(off + (size_t)std::max(p.B, 1) * 4, 256);
  w.xp = off;
  off = align_up(off + (size_t)tiles * p.T * nt * kx_of(p.I) * 2, 256);
  w.gates = off;
  off = align_up(off + (size_t)p.T * tiles * C * gblock_of(nt), 256);
  w.hseq = off;
  off = align_up(off + (size_t)p.T * tiles * C * piece_of(nt), 256);
  w.hlast = off;
  off = align_up(off + (size_t)std::max(p.B, 1) * p.H * 2, 256);
  w.trace = off;
  if (p.flags & PLSTM_FLAG_TRACE) off += (size_t)C * kTraceSteps * kTraceEvents * 8;
  w.total = off;
  return w;
}

// Compute warps of the recurrence: 8 (two per TMEM lane quadrant, 8 cells per
// thread; measured faster) unless PLSTM_TCL_WARPS=4 (one per quadrant, 16 cells).
int rec_warps() {
  static const int w = [] {
    const char* e = std::getenv("PLSTM_TCL_WARPS");
    return (e != nullptr && std::atoi(e) == 4) ? 4 : 8;
  }();
  return w;
}
template <int H, int NCW, int NT>
void* rec_ptr(bool bf16, bool varlen) {
  if (bf16) return varlen ? reinterpret_cast<void*>(&rec_kernel<H, NCW, true, true, NT>)
                          : reinterpret_cast<void*>(&rec_kernel<H, NCW, true, false, NT>);
  return varlen ? reinterpret_cast<void*>(&rec_kernel<H, NCW, false, true, NT>)
                : reinterpret_cast<void*>(&rec_kernel<H, NCW, false, false, NT>);
}
// Hidden sizes of the recurrence: multiples of 64 up to 512 (C = H / 32 CTAs per cluster,
// 2..16).  The 4-warp variant (PLSTM_TCL_WARPS=4) exists for 128 / 256 / 512 with 64-row
// tiles only; 80-row tiles exist for H >= 384 (C >= 12: the sizes whose clusters run out),
// 32- and 48-row tiles for H <= 256 (C <= 8).
bool rec_nt80(int H) { return H >= 384 && H <= 512 && H % 64 == 0; }
bool rec_nt32(int H) { return H >= 64 && H <= 256 && H % 64 == 0; }
void* pick_rec(int H, bool bf16, bool varlen, int nt) {
  if (nt == 32 || nt == 48) {
    switch (H * 100 + nt) {
      case 6432: return rec_ptr<64, 8, 32>(bf16, varlen);
      case 12832: return rec_ptr<128, 8, 32>(bf16, varlen);
      case 19232: return rec_ptr<192, 8, 32>(bf16, varlen);
      case 25632: return rec_ptr<256, 8, 32>(bf16, varlen);
      case 6448: return rec_ptr<64, 8, 48>(bf16, varlen);
      case 12848: return rec_ptr<128, 8, 48>(bf16, varlen);
      case 19248: return rec_ptr<192, 8, 48>(bf16, varlen);
      case 25648: return rec_ptr<256, 8, 48>(bf16, varlen);
      default: return nullptr;
    }
  }
  if (nt == 80) {
    switch (H) {
      case 384: return rec_ptr<384, 8, 80>(bf16, varlen);
      case 448: return rec_ptr<448, 8, 80>(bf16, varlen);
      case 512: return rec_ptr<512, 8, 80>(bf16, varlen);
      default: return nullptr;
    }
  }
  if (rec_warps() == 4 && (H == 128 || H == 256 || H == 512))
    return H == 128 ? rec_ptr<128, 4, 64>(bf16, varlen) : H == 256 ? rec_ptr<256, 4, 64>(bf16, varlen)
                                                            : rec_ptr<512, 4, 64>(bf16, varlen);
  switch (H) {
    case 64: return rec_ptr<64, 8, 64>(bf16, varlen);
    case 128: return rec_ptr<128, 8, 64>(bf16, varlen);
    case 192: return rec_ptr<192, 8, 64>(bf16, varlen);
    case 256: return rec_ptr<256, 8, 64>(bf16, varlen);
    case 320: return rec_ptr<320, 8, 64>(bf16, varlen);
    case 384: return rec_ptr<384, 8, 64>(bf16, varlen);
    case 448: return rec_ptr<448, 8, 64>(bf16, varlen);
    case 512: return rec_ptr<512, 8, 64>(bf16, varlen);
    default: return nullptr;
  }
}
int rec_smem(int H, int nt) {
  if (nt == 32)
    return H == 64 ? RecSmem<64, 8, 32>::kDyn : H == 128 ? RecSmem<128, 8, 32>::kDyn
                   : H == 192 ? RecSmem<192, 8, 32>::kDyn : RecSmem<256, 8, 32>::kDyn;
  if (nt == 48)
    return H == 64 ? RecSmem<64, 8, 48>::kDyn : H == 128 ? RecSmem<128, 8, 48>::kDyn
                   : H == 192 ? RecSmem<192, 8, 48>::kDyn : RecSmem<256, 8, 48>::kDyn;
  if (nt == 80) return H == 384 ? RecSmem<384, 8, 80>::kDyn : H == 448 ? RecSmem<448, 8, 80>::kDyn
                                                                       : RecSmem<512, 8, 80>::kDyn;
  switch (H) {
    case 64: return RecSmem<64, 8, 64>::kDyn;
    case 128: return RecSmem<128, 8, 64>::kDyn;
    case 192: return RecSmem<192, 8, 64>::kDyn;
    case 256: return RecSmem<256, 8, 64>::kDyn;
    case 320: return RecSmem<320, 8, 64>::kDyn;
    case 384: return RecSmem<384, 8, 64>::kDyn;
    case 448: return RecSmem<448, 8, 64>::kDyn;
    default: return RecSmem<512, 8, 64>::kDyn;
  }
}
bool rec_hidden_ok(int H) { return H >= 64 && H <= 512 && H % 64 == 0; }
int rec_threads(int H, int nt) { return ((nt != 64 ? 8 : rec_warps()) + 2) * 32; }

cudaError_t config_rec(void* k, int H, int nt) {
  if (k == nullptr) return cudaErrorInvalidDeviceFunction;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, rec_smem(H, nt));
  if (e == cudaSuccess && ctas_of(H) > 8) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

// Clusters of C CTAs of the recurrence that fit on `device` at once (0 = none); cached.
int rec_max_clusters(int device, int H, int nt) {
  static std::mutex mu;
  static int cache[64][8][4];
  static bool init = false;
  std::lock_guard<std::mutex> g(mu);
  if (!init) {
    for (auto& a : cache)
      for (auto& c : a) c[0] = c[1] = c[2] = c[3] = -1;
    init = true;
  }
  if (device < 0 || device >= 64 || !rec_hidden_ok(H) || (nt == 80 && !rec_nt80(H)) ||
      ((nt == 32 || nt == 48) && !rec_nt32(H)))
    return 0;
  int& slot = cache[device][H / 64 - 1][nt == 80 ? 1 : nt == 32 ? 2 : nt == 48 ? 3 : 0];
  if (slot >= 0) return slot;
  void* k = pick_rec(H, false, false, nt);
  int n = 0;
  if (config_rec(k, H, nt) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(ctas_of(H) * 16), 1, 1);
    cfg.blockDim = dim3((unsigned)rec_threads(H, nt), 1, 1);
    cfg.dynamicSmemBytes = rec_smem(H, nt);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = ctas_of(H);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  slot = n;
  return n;
}

// Recurrence CTAs (of both length variants of `dtype`) that one SM holds at once, at most two, by
// whole-SM registers, shared memory and tensor memory (H / 2 + 2 NT columns, 256 or 512 allocated);
// cached.  The cluster occupancy query counts one CTA per SM (15 clusters of 8 on a B200), but
// measured: 32 clusters of 8 CTAs of 32-row H = 256 tiles (f16 and bf16) ran in one wave, two CTAs
// on most SMs, 2.82 ms per layer at B = 1024 against 2.65 ms at B = 512.
int rec_ctas_per_sm(int device, int H, int nt, int dtype) {
  static std::mutex mu;
  static int cache[64][8][4][2];
  static bool init = false;
  std::lock_guard<std::mutex> g(mu);
  if (!init) {
    for (auto& a : cache)
      for (auto& b : a)
        for (auto& c : b) c[0] = c[1] = -1;
    init = true;
  }
  if (device < 0 || device >= 64 || !rec_hidden_ok(H)) return 0;
  const bool bf16 = dtype == PLSTM_BF16;
  int& slot = cache[device][H / 64 - 1][nt == 80 ? 1 : nt == 32 ? 2 : nt == 48 ? 3 : 0][bf16 ? 1 : 0];
  if (slot >= 0) return slot;
  int smem_sm = 0;
  int n = (H / 2 + 2 * nt + kMaxXK / 2 <= 256) ? 2 : 1;
  if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device) != cudaSuccess) n = 1;
  else n = std::min(n, smem_sm / (rec_smem(H, nt) + 1024));
  for (bool varlen : {false, true}) {
    cudaFuncAttributes fa = {};
    if (cudaFuncGetAttributes(&fa, pick_rec(H, bf16, varlen, nt)) != cudaSuccess) {
      n = 1;
      continue;
    }
    const int regs = (fa.numRegs + 7) / 8 * 8;
    n = std::min(n, 65536 / std::max(1, regs * rec_threads(H, nt)));
  }
  cudaGetLastError();
  slot = std::max(n, 1);
  return slot;
}

// Clusters of the recurrence that run at once: the occupancy query's count where one CTA fits an
// SM; with two, 7/8 of the SMs' CTA slots in whole clusters (a cluster must fit one GPC; 32
// clusters of 8 ran in one wave on 148 SMs), at least twice the query's count.
int rec_resident_clusters(int device, int H, int nt, int dtype) {
  const int m = rec_max_clusters(device, H, nt);
  const int k = rec_ctas_per_sm(device, H, nt, dtype);
  if (m < 1 || k < 2) return m;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    cudaGetLastError();
    return m;
  }
  return std::max(k * m, sms * k * 7 / (8 * ctas_of(H)));
}

// Tile rows of a forward: 32 or 48 for H <= 256 when those tiles still fit in one wave of
// clusters (32 first: at B = 512, H = 256 its 16 clusters run at once, 2.65 ms per layer
// against 2.86 ms with 11 clusters of 48 rows); 80 when 64-row tiles need more clusters than fit
// at once and 80-row tiles need fewer waves (B = 512 at H = 384..512: 8 tiles of 64 but 7
// clusters); else 64.
// PLSTM_TCL_NT=32|48|64|80 forces a tile height the hidden size has (tests, diagnostics).
int choose_nt(const Problem& q) {
  if (const char* e = std::getenv("PLSTM_TCL_NT")) {
    const int v = std::atoi(e);
    const bool has = v == 64 || (v == 80 && rec_nt80(q.H)) || ((v == 32 || v == 48) && rec_nt32(q.H));
    if (has && rec_max_clusters(q.device, q.H, v) >= 1) return v;
  }
  if (rec_nt32(q.H)) {
    for (int nt : {32, 48}) {
      const int m = rec_resident_clusters(q.device, q.H, nt, q.dtype);
      if (m >= 1 && (q.B + nt - 1) / nt <= m) return nt;
    }
    return 64;
  }
  if (!rec_nt80(q.H)) return 64;
  const int m64 = rec_max_clusters(q.device, q.H, 64), m80 = rec_max_clusters(q.device, q.H, 80);
  const int t64 = (q.B + 63) / 64, t80 = (q.B + 79) / 80;
  if (m64 >= 1 && m80 >= 1 && t64 > m64 && (t80 + m80 - 1) / m80 < (t64 + m64 - 1) / m64) return 80;
  return 64;
}

template <int KP, bool BF16, bool XIN, int NT>
int32_t launch_proj(const GemmArgs& ga, int sms, cudaStream_t s);
// Projection of layer 0 (K = kx, the packed x tile).
template <int NT>
int32_t launch_proj_x(const GemmArgs& ga, int kx, bool bf16, int sms, cudaStream_t s) {
#define PLSTM_TCL_PROJX(KX) \
  case KX: return bf16 ? launch_proj<KX, true, true, NT>(ga, sms, s) : launch_proj<KX, false, true, NT>(ga, sms, s);
  switch (kx) {
    PLSTM_TCL_PROJX(16) PLSTM_TCL_PROJX(32) PLSTM_TCL_PROJX(48) PLSTM_TCL_PROJX(64)
    PLSTM_TCL_PROJX(80) PLSTM_TCL_PROJX(96) PLSTM_TCL_PROJX(112) PLSTM_TCL_PROJX(128)
    default: break;
  }
#undef PLSTM_TCL_PROJX
  set_error("no projection kernel for this input width");
  return PLSTM_ENOTSUP;
}
// Projection of a layer >= 1 (K = H).
int32_t launch_proj_h64(const GemmArgs& ga, bool bf16, int sms, cudaStream_t s) {
#define PLSTM_TCL_PROJ(HH) \
  case HH: return bf16 ? launch_proj<HH, true, false, 64>(ga, sms, s) : launch_proj<HH, false, false, 64>(ga, sms, s);
  switch (ga.H) {
    PLSTM_TCL_PROJ(64) PLSTM_TCL_PROJ(128) PLSTM_TCL_PROJ(192) PLSTM_TCL_PROJ(256)
    PLSTM_TCL_PROJ(320) PLSTM_TCL_PROJ(384) PLSTM_TCL_PROJ(448) PLSTM_TCL_PROJ(512)
    default: break;
  }
#undef PLSTM_TCL_PROJ
  set_error("no projection kernel for this hidden size");
  return PLSTM_ENOTSUP;
}
template <int NT>
int32_t launch_proj_hs(const GemmArgs& ga, bool bf16, int sms, cudaStream_t s) {
#define PLSTM_TCL_PROJ(HH) \
  case HH: return bf16 ? launch_proj<HH, true, false, NT>(ga, sms, s) : launch_proj<HH, false, false, NT>(ga, sms, s);
  switch (ga.H) {
    PLSTM_TCL_PROJ(64) PLSTM_TCL_PROJ(128) PLSTM_TCL_PROJ(192) PLSTM_TCL_PROJ(256)
    default: break;
  }
#undef PLSTM_TCL_PROJ
  set_error("no projection kernel for this hidden size");
  return PLSTM_ENOTSUP;
}
int32_t launch_proj_h80(const GemmArgs& ga, bool bf16, int sms, cudaStream_t s) {
#define PLSTM_TCL_PROJ(HH) \
  case HH: return bf16 ? launch_proj<HH, true, false, 80>(ga, sms, s) : launch_proj<HH, false, false, 80>(ga, sms, s);
  switch (ga.H) {
    PLSTM_TCL_PROJ(384) PLSTM_TCL_PROJ(448) PLSTM_TCL_PROJ(512)
    default: break;
  }
#undef PLSTM_TCL_PROJ
  set_error("no projection kernel for this hidden size");
  return PLSTM_ENOTSUP;
}

template <int KP, bool BF16, bool XIN, int NT>
int32_t launch_proj(const GemmArgs& ga, int sms, cudaStream_t s) {
  using G = GemmSmem<KP, XIN, NT>;
  auto k = proj_kernel<KP, BF16, XIN, NT>;
  // Two CTAs per SM where tensor memory holds both (small jobs: their per-job latency chains
  // overlap); the shared-memory request then keeps a third off the SM (its allocation of tensor
  // memory would wait for one of the two to finish).
  const int per_sm = (G::kTmemCols <= 256 && getenv("PLSTM_TCL_PROJ1") == nullptr) ? 2 : 1;
  const int smem = per_sm == 2 ? std::max(G::kDyn, 80 * 1024) : G::kDyn;
  PLSTM_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int C = ctas_of(ga.H);
  const long long jobs = (long long)ga.T * ga.tiles * C;
  const int grid = (int)std::max<long long>(C, std::min<long long>((per_sm * sms / C) * C, jobs));
  k<<<grid, kGemmThreads, smem, s>>>(ga);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

}  // namespace tcl

using namespace tcl;

// The padded hidden size the kernels run (a multiple of 64); units >= p.H are zero.
int tcl_hp(int H) { return (H + 63) / 64 * 64; }
Problem padded(const Problem& p) {
  Problem q = p;
  q.H = tcl_hp(p.H);
  return q;
}

bool tcl_supported(const Problem& p, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (p.dtype != PLSTM_F16 && p.dtype != PLSTM_BF16) return no("activation type must be f16 or bf16");
  if (p.H < 1 || !rec_hidden_ok(tcl_hp(p.H))) return no("hidden_size must be <= 512");
  if (p.L < 1 || p.L > kMaxL) return no("num_layers must be 1..16");
  if (p.I > kMaxXK) return no("input_size must be <= 128");
  if (p.T < 1 || p.T > 65535) return no("seq_len must be 1..65535");
  int dev = p.device, major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    cudaGetLastError();
    return no("no CUDA device");
  }
  if (major != 10 || minor != 0) return no("device is not sm_100 (B200)");
  if (rec_max_clusters(dev, tcl_hp(p.H), 64) < 1) return no("the recurrence's CTA cluster does not fit on this device");
  return true;
}

size_t tcl_packed_size(const Problem& p) { return packed_total(tcl_hp(p.H), p.L, p.has_linear() ? p.O : 0); }

size_t tcl_workspace_size(const Problem& p) {
  const Problem q = padded(p);
  return ws_layout(q, choose_nt(q)).total;
}

int32_t tcl_pack(const Problem& p, int ih_layout, int hh_layout, const void* const* w_ih, const void* const* w_hh,
                 const void* const* b_ih, const void* const* b_hh, const void* w_lin, const void* b_lin,
                 void* packed, cudaStream_t s) {
  PackArgs a = {};
  for (int l = 0; l < p.L; ++l) {
    a.w_ih[l] = w_ih[l];
    a.w_hh[l] = w_hh[l];
    a.b_ih[l] = b_ih ? b_ih[l] : nullptr;
    a.b_hh[l] = b_hh ? b_hh[l] : nullptr;
  }
  a.w_lin = p.has_linear() ? w_lin : nullptr;
  a.b_lin = p.has_linear() ? b_lin : nullptr;
  a.ih_layout = ih_layout;
  a.hh_layout = hh_layout;
  a.dtype = p.dtype;
  a.L = p.L;
  a.I = p.I;
  a.H = tcl_hp(p.H);
  a.hid = p.H;
  a.kx = kx_of(p.I);
  a.O = p.has_linear() ? p.O : 0;
  pack_kernel<<<148 * 4, 256, 0, s>>>(a, static_cast<uint8_t*>(packed));
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

bool tcl_hu_supported(const HuProblem& p) {
  if (p.dtype != PLSTM_F16 && p.dtype != PLSTM_BF16) return false;
  if (p.H != 128 && p.H != 256 && p.H != 512) return false;
  if (p.T < 1 || p.T > 65535 || p.B < 1) return false;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, p.device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, p.device) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return major == 10 && minor == 0 && rec_max_clusters(p.device, p.H, 64) >= 1;
}

// Tile rows of a hidden update: the forward's choice for the same batch and hidden size.
int hu_nt(const HuProblem& p) {
  Problem q = {};
  q.B = p.B;
  q.T = p.T;
  q.H = p.H;
  q.L = 1;
  q.dtype = p.dtype;
  q.device = p.device;
  return choose_nt(q);
}

size_t tcl_hu_workspace_size(const HuProblem& p) { return hu_ws(p, hu_nt(p)).total; }

int32_t tcl_hidden_update(const HuProblem& p, const void* gate_proj, const void* w_hh, const void* bias, void* h_state,
                          float* c_state, void* out, void* ws, cudaStream_t s) {
  const int H = p.H, C = ctas_of(H);
  const int nt = hu_nt(p);
  const int tiles = (p.B + nt - 1) / nt;
  const HuWs w = hu_ws(p, nt);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  const bool bf16 = p.dtype == PLSTM_BF16;
  int32_t* perm = reinterpret_cast<int32_t*>(wsb + w.perm);
  int32_t* tile_len = reinterpret_cast<int32_t*>(wsb + w.tile_len);
  Problem pp = {};
  pp.B = p.B;
  pp.T = p.T;
  pp.H = H;
  pp.L = 1;
  pp.dtype = p.dtype;
  pp.device = p.device;
  {
    const int32_t rc = tc_make_perm(pp, nt, tiles, nullptr, perm, tile_len, nullptr, nullptr, s);
    if (rc != PLSTM_OK) return rc;
  }
  uint16_t* img = reinterpret_cast<uint16_t*>(wsb + w.whh);
  hu_pack_whh_kernel<<<148 * 4, 256, 0, s>>>(w_hh, p.dtype, p.w_layout, H, img);
  const int gblocks = p.T * tiles * C;
  const uint16_t* gp = static_cast<const uint16_t*>(gate_proj);
  const uint16_t* bp = static_cast<const uint16_t*>(bias);
  uint16_t* gates = reinterpret_cast<uint16_t*>(wsb + w.gates);
  auto gk = nt == 80   ? (bf16 ? hu_gates_kernel<true, 80> : hu_gates_kernel<false, 80>)
            : nt == 48 ? (bf16 ? hu_gates_kernel<true, 48> : hu_gates_kernel<false, 48>)
            : nt == 32 ? (bf16 ? hu_gates_kernel<true, 32> : hu_gates_kernel<false, 32>)
                       : (bf16 ? hu_gates_kernel<true, 64> : hu_gates_kernel<false, 64>);
  gk<<<gblocks, 256, 0, s>>>(gp, bp, p.B, p.T, H, tiles, p.seq_major() ? 1 : 0, gates);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(2);

  void* rk = pick_rec(H, bf16, false, nt);
  PLSTM_TRY_CUDA(config_rec(rk, H, nt));
  RecArgs ra = {};
  ra.whh = reinterpret_cast<const uint8_t*>(img);
  ra.gates = gates;
  ra.perm = perm;
  ra.lengths = nullptr;
  ra.tile_len = tile_len;
  ra.h0 = nullptr;
  ra.c0 = nullptr;
  ra.hseq = p.write_seq() ? wsb + w.hseq : nullptr;
  ra.h_n = h_state;
  ra.c_n = c_state;
  ra.hlast = nullptr;
  ra.status = reinterpret_cast<int*>(wsb);
  ra.B = p.B;
  ra.T = p.T;
  ra.layer = 0;
  ra.hid = H;
  ra.flags = PLSTM_FLAG_CN_F32;
  ra.timeout_ns = 2000000000ull;
  ra.trace = nullptr;
  ra.trace_t0 = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * C), 1, 1);
  cfg.blockDim = dim3((unsigned)rec_threads(H, nt), 1, 1);
  cfg.dynamicSmemBytes = rec_smem(H, nt);
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = C;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  void* args[] = {&ra};
  profile_begin(s);
  PLSTM_TRY_CUDA(cudaLaunchKernelExC(&cfg, rk, args));
  profile_end(s);
  note_launches(1);
  if (p.write_seq()) {
    const int smem = nt * (H + 1) * 4;
    auto k = nt == 80   ? (bf16 ? seq_out_kernel<true, false, 80> : seq_out_kernel<false, false, 80>)
             : nt == 48 ? (bf16 ? seq_out_kernel<true, false, 48> : seq_out_kernel<false, false, 48>)
             : nt == 32 ? (bf16 ? seq_out_kernel<true, false, 32> : seq_out_kernel<false, false, 32>)
                        : (bf16 ? seq_out_kernel<true, false, 64> : seq_out_kernel<false, false, 64>);
    PLSTM_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    k<<<p.T * tiles, 256, smem, s>>>(wsb + w.hseq, perm, nullptr, nullptr, nullptr, static_cast<uint16_t*>(out), p.B,
                                     p.T, H, 0, tiles, p.seq_major() ? 1 : 0, H);
    PLSTM_TRY_CUDA(cudaGetLastError());
    note_launches(1);
  } else {
    PLSTM_TRY_CUDA(cudaMemcpyAsync(out, h_state, (size_t)p.B * H * 2, cudaMemcpyDeviceToDevice, s));
  }
  return PLSTM_OK;
}

int32_t tcl_forward(const Problem& p, const void* packed, const void* x, const int32_t* lengths, const void* h0,
                    const void* c0, void* out, void* h_n, void* c_n, void* ws, cudaStream_t s) {
  const int H = tcl_hp(p.H), L = p.L, C = ctas_of(H);
  const int nt = choose_nt(padded(p));
  const int tiles = (p.B + nt - 1) / nt;
  if (const char* dbg = std::getenv("PLSTM_TC_DEBUG"))
    if (std::atoi(dbg) != 0)
      std::fprintf(stderr, "plstm tcl: H %d, %d-row tiles, %d tiles; clusters of %d CTAs at once (32/48/64 rows): %d/%d/%d\n",
                   H, nt, tiles, C, rec_resident_clusters(p.device, H, 32, p.dtype),
                   rec_resident_clusters(p.device, H, 48, p.dtype), rec_resident_clusters(p.device, H, 64, p.dtype));
  const Ws w = ws_layout(padded(p), nt);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  int32_t* perm = reinterpret_cast<int32_t*>(wsb + w.perm);
  int32_t* tile_len = reinterpret_cast<int32_t*>(wsb + w.tile_len);
  const bool bf16 = p.dtype == PLSTM_BF16;
  const bool varlen = lengths != nullptr;
  const int O = p.has_linear() ? p.O : 0;
  {
    const int32_t rc = tc_make_perm(p, nt, tiles, lengths, perm, tile_len, reinterpret_cast<int32_t*>(wsb + w.hist),
                                    reinterpret_cast<int32_t*>(wsb + w.sorted), s);
    if (rc != PLSTM_OK) return rc;
  }
  {
    const int32_t rc = tc_xpack(p, nt, tiles, x, perm, wsb + w.xp, kx_of(p.I), s);
    if (rc != PLSTM_OK) return rc;
  }
  int sms = 148;
  PLSTM_TRY_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p.device));
  void* rk = pick_rec(H, bf16, varlen, nt);
  PLSTM_TRY_CUDA(config_rec(rk, H, nt));
  const bool seq_out = !p.has_linear() || p.out_seq();
  // Layer 0's input projection runs inside its recurrence for tile heights of 64 / 80 rows (one CTA per
  // SM; config 4: 23.8 -> 23.2 ms); with 32-row tiles, two CTAs sharing an SM, the separate projection
  // measured as fast (config 3: 10.12 against 10.16 ms).  PLSTM_TCL_PROJ0 forces the separate one.
  const bool fuse_x0 = nt >= 64 && std::getenv("PLSTM_TCL_PROJ0") == nullptr;
  for (int l = 0; l < L; ++l) {
    GemmArgs ga = {};
    ga.xp = wsb + w.xp;
    ga.hseq = wsb + w.hseq;
    ga.wih = reinterpret_cast<const uint16_t*>(pk + off_wih(l, H, L));
    ga.bias = reinterpret_cast<const float*>(pk + off_bias(H, L)) + (size_t)l * 4 * H;
    ga.gates = reinterpret_cast<uint16_t*>(wsb + w.gates);
    ga.status = reinterpret_cast<int*>(wsb);
    ga.T = p.T;
    ga.H = H;
    ga.tiles = tiles;
    int32_t rc = PLSTM_OK;
    if (l == 0 && !fuse_x0)
      rc = nt == 80   ? launch_proj_x<80>(ga, kx_of(p.I), bf16, sms, s)
           : nt == 32 ? launch_proj_x<32>(ga, kx_of(p.I), bf16, sms, s)
           : nt == 48 ? launch_proj_x<48>(ga, kx_of(p.I), bf16, sms, s)
                      : launch_proj_x<64>(ga, kx_of(p.I), bf16, sms, s);
    else if (l > 0)
      rc = nt == 80   ? launch_proj_h80(ga, bf16, sms, s)
           : nt == 32 ? launch_proj_hs<32>(ga, bf16, sms, s)
           : nt == 48 ? launch_proj_hs<48>(ga, bf16, sms, s)
                      : launch_proj_h64(ga, bf16, sms, s);
    if (rc != PLSTM_OK) return rc;

    RecArgs ra = {};
    ra.whh = pk + off_whh(l, H);
    ra.gates = reinterpret_cast<const uint16_t*>(wsb + w.gates);
    if (l == 0 && fuse_x0) {
      ra.xp = wsb + w.xp;
      ra.wih0 = reinterpret_cast<const uint16_t*>(pk + off_wih(0, H, L));
      ra.bias0 = reinterpret_cast<const float*>(pk + off_bias(H, L));
      ra.kx = kx_of(p.I);
    }
    ra.perm = perm;
    ra.lengths = lengths;
    ra.tile_len = tile_len;
    ra.h0 = h0;
    ra.c0 = c0;
    ra.hseq = (l + 1 < L || seq_out) ? wsb + w.hseq : nullptr;
    ra.h_n = h_n;
    ra.c_n = c_n;
    ra.hlast = l + 1 == L ? reinterpret_cast<uint16_t*>(wsb + w.hlast) : nullptr;
    ra.status = reinterpret_cast<int*>(wsb);
    ra.B = p.B;
    ra.T = p.T;
    ra.layer = l;
    ra.hid = p.H;
    ra.flags = p.flags;
    ra.timeout_ns = (unsigned long long)p.timeout_ms * 1000000ull;
    ra.trace = nullptr;
    ra.trace_t0 = p.T / 2;
    if ((p.flags & PLSTM_FLAG_TRACE) && l == 0) {  // the first layer's recurrence
      ra.trace = reinterpret_cast<unsigned long long*>(wsb + w.trace);
      PLSTM_TRY_CUDA(cudaMemsetAsync(ra.trace, 0, (size_t)C * kTraceSteps * kTraceEvents * 8, s));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles * C), 1, 1);
    cfg.blockDim = dim3((unsigned)rec_threads(H, nt), 1, 1);
    cfg.dynamicSmemBytes = rec_smem(H, nt);
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = C;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    void* args[] = {&ra};
    if (l == 0) profile_begin(s);
    PLSTM_TRY_CUDA(cudaLaunchKernelExC(&cfg, rk, args));
    if (l + 1 == L) profile_end(s);
    note_launches(1);
  }
  const uint16_t* wlin = reinterpret_cast<const uint16_t*>(pk + off_wlin(H, L));
  const float* blin = reinterpret_cast<const float*>(pk + off_blin(H, L, O));
  uint16_t* o16 = static_cast<uint16_t*>(out);
  if (p.has_linear() && !p.out_seq()) {
    const int n = p.B * O;
    if (bf16)
      linear_last_kernel<true><<<(n + 255) / 256, 256, 0, s>>>(reinterpret_cast<const uint16_t*>(wsb + w.hlast), wlin,
                                                               blin, o16, p.B, H, O);
    else
      linear_last_kernel<false><<<(n + 255) / 256, 256, 0, s>>>(reinterpret_cast<const uint16_t*>(wsb + w.hlast), wlin,
                                                                blin, o16, p.B, H, O);
  } else {
    const int smem = nt * (H + 1) * 4;
    const int grid = p.T * tiles;
    if (p.has_linear()) {
      auto k = nt == 80   ? (bf16 ? seq_out_kernel<true, true, 80> : seq_out_kernel<false, true, 80>)
               : nt == 32 ? (bf16 ? seq_out_kernel<true, true, 32> : seq_out_kernel<false, true, 32>)
               : nt == 48 ? (bf16 ? seq_out_kernel<true, true, 48> : seq_out_kernel<false, true, 48>)
                          : (bf16 ? seq_out_kernel<true, true, 64> : seq_out_kernel<false, true, 64>);
      PLSTM_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      k<<<grid, 256, smem, s>>>(wsb + w.hseq, perm, lengths, wlin, blin, o16, p.B, p.T, H, O, tiles, 0, p.H);
    } else {
      auto k = nt == 80   ? (bf16 ? seq_out_kernel<true, false, 80> : seq_out_kernel<false, false, 80>)
               : nt == 32 ? (bf16 ? seq_out_kernel<true, false, 32> : seq_out_kernel<false, false, 32>)
               : nt == 48 ? (bf16 ? seq_out_kernel<true, false, 48> : seq_out_kernel<false, false, 48>)
                          : (bf16 ? seq_out_kernel<true, false, 64> : seq_out_kernel<false, false, 64>);
      PLSTM_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      k<<<grid, 256, smem, s>>>(wsb + w.hseq, perm, lengths, wlin, blin, o16, p.B, p.T, H, 0, tiles, 0, p.H);
    }
  }
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

}  // namespace plstm
