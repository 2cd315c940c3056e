// plstm_tc.cu — tcgen05 cluster wavefront backend for H = 128 LSTM stacks.
//
// What it replaces.  The reference runs this path as a chain of persistent
// per-layer-pair kernels with weights re-read from global memory every step
// (persistent_lstm_pair01_interleaved_kernel / pair23_last_interleaved_kernel,
// persistent_lstm_hip.cu:457-662, host :2126-2254), a 4-layer "monolithic"
// variant (:664-806) and a separate linear_head_kernel (:1662-1682).
//
// Design (B200-first).
//   * One thread-block cluster of 2L CTAs per tile of N batch rows.  CTA rank
//     r = 2l + s owns layer l, hidden units [64 s, 64 s + 64): 256 gate rows.
//   * Its slice of [W_ih | W_hh] (256 rows x K, K = 256 for l >= 1,
//     16 + 128 for l = 0 with x zero-padded to 16 columns) stays resident in
//     tensor memory for the whole sequence as the A operand (256 of the SM's
//     512 TMEM columns), so each MMA streams only the small h operand from
//     shared memory.  The per-step contraction gates^T[256 x N] = W . [x_t | h_{t-1}]^T
//     runs as tcgen05.mma kind::f16 (f16/bf16 in, f32 accumulate in TMEM),
//     M = 128 per instruction, N = batch tile.
//   * The contraction is split in three: the input part W_ih . x_t is
//     issued as soon as x_t (layer 0) or h_{l-1}(t) (from layer l-1) lands, into
//     one of two TMEM accumulators, while the previous step's gates are still
//     being processed; the recurrent part over this CTA's own 64 units of
//     h_{t-1} is issued as soon as this CTA has written them; only the
//     recurrent part over the sibling CTA's 64 units (K = 64, 8 MMAs) waits for
//     the cross-CTA hand-off.
//   * Layers run as a wavefront: layer l works on step t while layer l+1 works
//     on step t-1.  The new h tile (64 units x N rows, 16-bit) is written once
//     into this CTA's next B buffer and pushed to the sibling CTA (recurrent
//     half) and to both CTAs of layer l+1 (input half) with shared::cta ->
//     shared::cluster bulk copies that complete as transaction bytes on the
//     destination's mbarrier.  Back-pressure from layer l+1 arrives through a
//     multicast tcgen05.commit on this CTA's "empty" barriers.  No grid-wide
//     barrier, no global-memory round trip for h.
//   * Gate rows are ordered inside each 32-lane TMEM quadrant as
//     [i x 8 units | f x 8 | g x 8 | o x 8], so one tcgen05.ld 16x256b per
//     half-quadrant hands every thread the i, f, g, o values of the same
//     (unit, batch) cells; bias, sigmoid / tanh and the c / h update run in
//     registers with c kept in f32 (the reference keeps c in f32 registers and
//     rounds h to 16 bits between steps, persistent_lstm_hip.cu:316-324).
//   * The Linear head is one more M = 128 MMA (rows >= O are zero) on the last
//     layer's recurrent half of the next step's B buffer, i.e. on h_{t-1}; it
//     is added to the step-t MMA batch, and a final "drain" step handles
//     h_{T-1}.  OUT_LAST only runs the drain.
//   * Variable lengths: rows are sorted by length (descending) into tiles, a
//     tile runs max(len) steps, finished rows freeze their state and write
//     zeros.
//   * Every wait is bounded (globaltimer deadline); a wait that gives up
//     records PLSTM_ETIMEOUT in the workspace status word, raises the abort
//     flag of every CTA of the cluster and the kernel unwinds without trapping.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "plstm_common.cuh"
#include "sm100_ptx.cuh"

namespace plstm {
namespace tc {

constexpr int kH = 128;  // hidden size of the kernels (64 units per CTA); smaller H runs zero-padded
constexpr int kXK = 16;       // layer-0 input width step (one MMA K step); the single-slot kernel's width
constexpr int kMaxXK = 128;   // widest padded layer-0 input: [W_ih | W_hh] fills the 256-wide A image
constexpr int kMaxLayers = 8; // one cluster of 2L <= 16 CTAs (16 needs the non-portable cluster size)
constexpr int kABytes = 128 * 1024;                 // A image slot per CTA: [tile 2][row 128][K 256] 16-bit
constexpr int kAK = 256;                            // K extent of an A image row
constexpr int kTmemACols = 256;                     // TMEM columns holding A: 2 tiles x 128
constexpr int kALinBytes = 32 * 1024;               // Linear head A image (2 K blocks)
constexpr int kATileKB = 128 * 128;                 // one (M tile, 64-wide K block): 16 KB
constexpr int kModeSeq = 0, kModeLast = 1, kModeHSeq = 2;

// Packed image layout (global): [2L slots of kABytes][A_lin][bias f32 [2L][256]][b_lin f32 [32]]
__host__ __device__ inline size_t packed_alin_off(int L) { return (size_t)2 * L * kABytes; }
__host__ __device__ inline size_t packed_bias_off(int L) { return packed_alin_off(L) + kALinBytes; }
__host__ __device__ inline size_t packed_blin_off(int L) { return packed_bias_off(L) + (size_t)2 * L * 256 * 4; }
__host__ __device__ inline size_t packed_total(int L) { return packed_blin_off(L) + 32 * 4; }

__host__ __device__ constexpr int tmem_cols_for(int need) {
  return need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
}

// Shared memory layout (offsets from a 1024-byte aligned base).
template <int N>
struct Smem {
  static constexpr int kBKB = N * 128;  // one 64-wide K block of the B operand
  static constexpr int kXBytes = N * 32;
  static constexpr int kB = 0;
  static constexpr int kBufBytes = 4 * kBKB;  // slots: [in0 | in1 | rec0 | rec1]
  static constexpr int kALin = kB + 2 * kBufBytes;
  static constexpr int kBar = kALin + kALinBytes;
  // mbarriers (8 bytes each, two per kind: one per step parity)
  static constexpr int kFullIn = kBar, kFullRec = kBar + 16, kEmpty = kBar + 32, kHReady = kBar + 48,
                       kMma = kBar + 64;
  static constexpr int kTmemSlot = kBar + 96, kAbort = kBar + 100, kDone = kBar + 104;
  static constexpr int kPerm = kBar + 128, kLens = kPerm + 4 * N;
  static constexpr int kEnd = kLens + 4 * N;
  static constexpr int kDynBytes = kEnd + 1024;  // + alignment slack
  // Linear head columns per CTA: split between the two last-layer CTAs when
  // N / 2 is a legal MMA width (multiple of 16), else CTA 0 takes all N.
  static constexpr bool kSplitLinear = (N / 2) % 16 == 0;
  // N / 16 compute warps per TMEM lane quadrant, two 256-bit column chunks each.
  static constexpr int kG = N / 16;
  static constexpr int kComputeWarps = 4 * kG;
  static constexpr int kThreads = (kComputeWarps + 1) * 32;  // + one control warp (MMA issue, h hand-off)
  static constexpr int kNL = kSplitLinear ? N / 2 : N;
  // TMEM: A (256 columns), gates D[buffer 0..1][tile 0..1] (N columns each), the Linear tile.
  static constexpr int kD = kTmemACols;
  static constexpr int kDLin = kD + 4 * N;
  static constexpr int kTmemCols = tmem_cols_for(kDLin + kNL);
  static_assert(kDLin + kNL <= 512, "tile too wide for tensor memory");
};

struct Params {
  const uint8_t* packed;
  const uint8_t* xp;        // [tiles][T][N * kx * 2 bytes], or null: the kernel reads x itself (x_raw)
  const uint16_t* x_raw;    // x[B][T][I] 16-bit, read by the layer-0 x warp of the multi-slot kernel when xp is null
  int I;                    // input columns of x_raw (<= 16, so that kx = 16)
  const int32_t* perm;      // [tiles * N], -1 = padding row
  const int32_t* lengths;   // [B] (varlen) or null
  const int32_t* tile_len;  // [tiles]
  const void* h0;
  const void* c0;
  void* out;
  void* h_n;
  void* c_n;
  int* status;
  int B, T, L, O, flags;
  int kx;                   // padded layer-0 input width (multiple of 16, <= 128; 16 for the single-slot kernel)
  int hid;                  // the model's hidden size H <= 128: units >= H are zero padding (zero weights,
                            // state and output), h0 / c0 / h_n / c_n / h-sequence rows are H wide
  unsigned long long timeout_ns;
  int drop_rank, drop_step;  // fault injection: rank that skips one sibling hand-off (-1 = off)
  unsigned long long* trace;  // PLSTM_FLAG_TRACE: [2L][64][8] clock64 stamps of cluster 0, or null
  int trace_t0;
  int trace_slot;  // two-slot kernel: the slot whose events are recorded
  const int* choice;  // two tile heights enqueued (variable lengths): run only if *choice == N, else null
};

// Trace events: control warp 0 sibling h landed, 1 recurrent MMAs + commit issued,
// 2 hready seen (copies follow), 3 own-half MMAs issued (loop top); compute warp 0:
// 4 accumulators ready, 5 loaded, 6 h written; 7 h written by the last compute warp.
constexpr int kTraceSteps = 64, kTraceEvents = 8;

__device__ __forceinline__ void trace_mark(const Params& p, int rank, int t, int ev) {
  if (p.trace != nullptr && blockIdx.x < (unsigned)(2 * p.L) && t >= p.trace_t0 && t < p.trace_t0 + kTraceSteps)
    p.trace[((size_t)rank * kTraceSteps + (t - p.trace_t0)) * kTraceEvents + ev] = clock64();
}

// 128-byte swizzled K-major offset of element (row, k) of a 64-wide K block.
__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

template <bool BF16>
__device__ __forceinline__ uint16_t to_bits(float v) {
  if (BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
  } else {
    __half h = __float2half_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
  }
}
// Two values rounded to 16 bits in one instruction: lo -> bits [0, 16), hi -> [16, 32).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2_bits(float lo, float hi) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}
template <bool BF16>
__device__ __forceinline__ float from_bits(uint16_t b) {
  if (BF16) {
    return __bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&b));
  } else {
    return __half2float(*reinterpret_cast<__half*>(&b));
  }
}

// Gate math of one step for this thread's cells [tau][jc][e] (its two units x CPW
// 8-column chunks x two columns).  rif / rgo hold the raw i, f / g, o accumulators
// (gate rows i, f, o pre-scaled by 1/2), bz the f32 bias per unit and gate.  Every
// activation is one hardware tanh: sigmoid(z) = (1 + tanh(z / 2)) / 2.  The four gate
// activations of all cells are issued back to back (independent MUFU operations),
// then the cell update, then tanh(c).  c stays f32; h is rounded to 16 bits in pairs.
// Rows past their length keep c and h; hw receives the h bits to write.
template <int CPW, bool BF16, bool VARLEN>
__device__ __forceinline__ void lstm_cells(const uint32_t (&rif)[2][4 * CPW], const uint32_t (&rgo)[2][4 * CPW],
                                           const float (&bz)[2][4], float (&c_st)[2][CPW][2],
                                           uint16_t (&h_st)[2][CPW][2], const int (&len_c)[CPW][2], int t,
                                           uint16_t (&hw)[2][CPW][2]) {
  float ti[2][CPW][2], tf[2][CPW][2], tg[2][CPW][2], to[2][CPW][2];
#pragma unroll
  for (int tau = 0; tau < 2; ++tau)
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        ti[tau][jc][e] = ptx::tanh_approx(__uint_as_float(rif[tau][4 * jc + e]) + bz[tau][0]);
        tf[tau][jc][e] = ptx::tanh_approx(__uint_as_float(rif[tau][4 * jc + 2 + e]) + bz[tau][1]);
        tg[tau][jc][e] = ptx::tanh_approx(__uint_as_float(rgo[tau][4 * jc + e]) + bz[tau][2]);
        to[tau][jc][e] = ptx::tanh_approx(__uint_as_float(rgo[tau][4 * jc + 2 + e]) + bz[tau][3]);
      }
  float c_new[2][CPW][2];
#pragma unroll
  for (int tau = 0; tau < 2; ++tau)
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
      for (int e = 0; e < 2; ++e)
        c_new[tau][jc][e] = fmaf(fmaf(0.5f, tf[tau][jc][e], 0.5f), c_st[tau][jc][e],
                                 fmaf(0.5f, ti[tau][jc][e], 0.5f) * tg[tau][jc][e]);
#pragma unroll
  for (int tau = 0; tau < 2; ++tau)
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc) {
      float h[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) h[e] = fmaf(0.5f, to[tau][jc][e], 0.5f) * ptx::tanh_approx(c_new[tau][jc][e]);
      const uint32_t bits = pack2_bits<BF16>(h[0], h[1]);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint16_t hb = (uint16_t)(e == 0 ? bits & 0xffffu : bits >> 16);
        if (!VARLEN || t < len_c[jc][e]) {
          c_st[tau][jc][e] = c_new[tau][jc][e];
          h_st[tau][jc][e] = hb;
        }
        hw[tau][jc][e] = h_st[tau][jc][e];
      }
    }
}

// Registers written by an asynchronous tcgen05.ld: the compiler sees them defined at the load,
// so an empty asm that rewrites them, placed after tcgen05.wait::ld, keeps every use behind the
// wait (volatile asm statements stay in order).
template <int N>
__device__ __forceinline__ void reg_after_wait(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// lstm_cells restricted to tile `tau` (the same arithmetic per cell), so that one tile's gate
// math can run while the other tile's accumulators are still being loaded.
template <int CPW, bool BF16, bool VARLEN>
__device__ __forceinline__ void lstm_cells_tile(int tau, const uint32_t (&rif)[2][4 * CPW],
                                                const uint32_t (&rgo)[2][4 * CPW], const float (&bz)[2][4],
                                                float (&c_st)[2][CPW][2], uint16_t (&h_st)[2][CPW][2],
                                                const int (&len_c)[CPW][2], int t, uint16_t (&hw)[2][CPW][2]) {
  float ti[CPW][2], tf[CPW][2], tg[CPW][2], to[CPW][2];
#pragma unroll
  for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      ti[jc][e] = ptx::tanh_approx(__uint_as_float(rif[tau][4 * jc + e]) + bz[tau][0]);
      tf[jc][e] = ptx::tanh_approx(__uint_as_float(rif[tau][4 * jc + 2 + e]) + bz[tau][1]);
      tg[jc][e] = ptx::tanh_approx(__uint_as_float(rgo[tau][4 * jc + e]) + bz[tau][2]);
      to[jc][e] = ptx::tanh_approx(__uint_as_float(rgo[tau][4 * jc + 2 + e]) + bz[tau][3]);
    }
#pragma unroll
  for (int jc = 0; jc < CPW; ++jc) {
    float h[2], c_new[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      c_new[e] = fmaf(fmaf(0.5f, tf[jc][e], 0.5f), c_st[tau][jc][e], fmaf(0.5f, ti[jc][e], 0.5f) * tg[jc][e]);
      h[e] = fmaf(0.5f, to[jc][e], 0.5f) * ptx::tanh_approx(c_new[e]);
    }
    const uint32_t bits = pack2_bits<BF16>(h[0], h[1]);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint16_t hb = (uint16_t)(e == 0 ? bits & 0xffffu : bits >> 16);
      if (!VARLEN || t < len_c[jc][e]) {
        c_st[tau][jc][e] = c_new[e];
        h_st[tau][jc][e] = hb;
      }
      hw[tau][jc][e] = h_st[tau][jc][e];
    }
  }
}

// Bounded wait on an mbarrier phase; false = gave up (timeout or cluster abort).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                           unsigned long long timeout_ns) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer() - t0 > timeout_ns) return false;
  }
}

// Warp-uniform versions: lane 0 polls, the result is broadcast.
__device__ __forceinline__ bool warp_wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                unsigned long long timeout_ns) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_phase(bar, parity, abort_flag, timeout_ns) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
// Non-blocking: a warp that polls two barriers in turn must not sleep on one of them.
__device__ __forceinline__ bool warp_test_wait(uint32_t bar, uint32_t parity) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = ptx::mbar_test_wait(bar, parity) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Pushes this CTA's half of h(t) (`bytes` at shared address `src`) to the sibling
// CTA (recurrent half of its next step: same local offset, barrier `sib_bar`) and to
// both CTAs of layer l+1 (input slot `in_dst`, barrier `in_bar`).  Issued by the last
// compute warp to finish the step, right after its writes.
__device__ __forceinline__ void push_h(uint32_t src, uint32_t bytes, int rank, bool to_sibling, uint32_t sib_bar,
                                       bool downstream, int next_layer_rank0, uint32_t in_dst, uint32_t in_bar) {
  if (to_sibling) {
    const uint32_t peer = (uint32_t)(rank ^ 1);
    ptx::bulk_s2c(ptx::mapa(src, peer), src, bytes, ptx::mapa(sib_bar, peer));
  }
  if (downstream) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t peer = (uint32_t)(next_layer_rank0 + j);
      ptx::bulk_s2c(ptx::mapa(in_dst, peer), src, bytes, ptx::mapa(in_bar, peer));
    }
  }
}

// Raises the abort flag in every CTA of the cluster and records the failure.
__device__ __forceinline__ void raise_abort(const Params& p, uint8_t* sm_abort, int ncta, int step) {
  const uint32_t local = ptx::smem_u32(sm_abort);
  for (int r = 0; r < ncta; ++r) ptx::st_cluster_u32(ptx::mapa(local, (uint32_t)r), 1u);
  report_status(p.status, PLSTM_ETIMEOUT, (int)((blockIdx.x & 0x7fff) << 16) | (step & 0xffff));
}

// Loads CPW 256-bit column chunks of 16 lanes starting at `taddr` into r[0 .. 4*CPW).
template <int CPW>
__device__ __forceinline__ void tmem_ld_chunks(uint32_t taddr, uint32_t (&r)[4 * CPW]) {
  if constexpr (CPW == 1) {
    ptx::tmem_ld_16x256b_x1(taddr, *reinterpret_cast<uint32_t(*)[4]>(&r[0]));
  } else if constexpr (CPW == 2) {
    ptx::tmem_ld_16x256b_x2(taddr, *reinterpret_cast<uint32_t(*)[8]>(&r[0]));
  } else if constexpr (CPW == 3) {
    ptx::tmem_ld_16x256b_x2(taddr, *reinterpret_cast<uint32_t(*)[8]>(&r[0]));
    ptx::tmem_ld_16x256b_x1(taddr + 16, *reinterpret_cast<uint32_t(*)[4]>(&r[8]));
  } else {
    static_assert(CPW == 4, "CPW must be 1..4");
    ptx::tmem_ld_16x256b_x4(taddr, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
  }
}

template <int N, bool BF16, bool VARLEN, int MODE>
__global__ void __launch_bounds__(Smem<N>::kThreads, 1) wavefront_kernel(const Params p) {
  using S = Smem<N>;
  constexpr int G = S::kG;
  constexpr int kThreads = S::kThreads;
  constexpr int kComputeWarps = S::kComputeWarps;
  constexpr int CPW = 2;  // 256-bit column chunks per compute warp
  constexpr int NL = S::kNL;
  constexpr bool kHasLinear = MODE != kModeHSeq;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ncta = 2 * p.L;
  const int rank = (int)ptx::cluster_ctarank();
  const int l = rank >> 1, s = rank & 1;
  const int tile = blockIdx.x / ncta;
  const bool last_layer = l == p.L - 1;
  const bool drain = kHasLinear && last_layer;
  const bool does_linear = drain && (S::kSplitLinear || s == 0);
  const bool sibling_linear = drain && (S::kSplitLinear || s == 1);
  const int Tt = p.tile_len[tile];
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kAbort);
  int32_t* perm_s = reinterpret_cast<int32_t*>(sm + S::kPerm);
  int32_t* lens_s = reinterpret_cast<int32_t*>(sm + S::kLens);

  const uint32_t bar_in = sbase + S::kFullIn, bar_rec = sbase + S::kFullRec, bar_empty = sbase + S::kEmpty;
  const uint32_t bar_hready = sbase + S::kHReady, bar_mma = sbase + S::kMma;
  auto bbuf = [&](int b) -> uint32_t { return sbase + S::kB + b * S::kBufBytes; };

  // ---- set-up ------------------------------------------------------------------
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar_in + 8 * b, 1);
      ptx::mbar_init(bar_rec + 8 * b, 1);
      ptx::mbar_init(bar_empty + 8 * b, 2);
      ptx::mbar_init(bar_hready + 8 * b, kComputeWarps);
      ptx::mbar_init(bar_mma + 8 * b, 1);
    }
    *abort_flag = 0;
    *reinterpret_cast<uint32_t*>(sm + S::kDone) = 0;
    ptx::fence_mbar_init_cluster();
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + S::kTmemSlot, S::kTmemCols);
    ptx::tmem_relinquish();
  }
  for (int i = tid; i < N; i += kThreads) {
    const int b = p.perm[tile * N + i];
    perm_s[i] = b;
    int len = 0;
    if (b >= 0) len = VARLEN ? min(max(p.lengths[b], 0), p.T) : p.T;
    lens_s[i] = len;
  }
  {
    if (does_linear) {
      const uint4* srcl = reinterpret_cast<const uint4*>(p.packed + packed_alin_off(p.L));
      uint4* dstl = reinterpret_cast<uint4*>(sm + S::kALin);
      for (int i = tid; i < kALinBytes / 16; i += kThreads) dstl[i] = srcl[i];
    }
  }
  __syncthreads();  // perm_s / lens_s / tmem slot visible
  // Initial recurrent state h0 -> both recurrent K blocks of B buffer 0.
  {
    uint8_t* b0 = sm + S::kB;
    for (int i = tid; i < N * kH; i += kThreads) {
      const int n = i / kH, k = i % kH;
      float v = 0.0f;
      const int b = perm_s[n];
      if (p.h0 != nullptr && b >= 0 && k < p.hid) {
        const uint16_t* h0 = static_cast<const uint16_t*>(p.h0);
        v = from_bits<BF16>(h0[((size_t)l * p.B + b) * p.hid + k]);
      }
      *reinterpret_cast<uint16_t*>(b0 + (2 + (k >> 6)) * S::kBKB + sw128_off(n, k & 63)) = to_bits<BF16>(v);
    }
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + S::kTmemSlot);
  // This CTA's weight slice -> TMEM columns [0, 256), one A row per lane, K
  // packed two 16-bit values per column.
  if (warp < kComputeWarps) {
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    for (int tau = warp >> 2; tau < 2; tau += G) {
      const uint4* src = reinterpret_cast<const uint4*>(p.packed + (size_t)rank * kABytes +
                                                        ((size_t)tau * 128 + row) * kAK * 2);
#pragma unroll 1
      for (int c = 0; c < kAK / 2; c += 32) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 v = src[c / 4 + i];
          r[4 * i + 0] = v.x;
          r[4 * i + 1] = v.y;
          r[4 * i + 2] = v.z;
          r[4 * i + 3] = v.w;
        }
        ptx::tmem_st_32x32b_x32(tmem + lane_off + (uint32_t)(tau * 128 + c), r);
      }
    }
    ptx::tmem_wait_st();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::cluster_sync();  // every CTA's barriers are initialised before any remote operation

  auto dcol = [&](int buf, int tau) -> uint32_t { return tmem + (uint32_t)(S::kD + (2 * buf + tau) * N); };

  if (warp == kComputeWarps) {
    // ============================ control warp ==========================
    const uint32_t xbytes = S::kXBytes, bkb = S::kBKB;
    const uint32_t in_bytes = (l == 0) ? xbytes : 2 * bkb;
    constexpr uint32_t idesc_g = ptx::idesc_f16(128, N, BF16);
    constexpr uint32_t idesc_l = ptx::idesc_f16(128, NL, BF16);
    const uint16_t up_mask = l > 0 ? (uint16_t)(3u << (2 * (l - 1))) : 0;
    // Descriptors advance by (byte offset >> 4) in the start-address field; A
    // K-steps advance by 8 TMEM columns.  A columns: layer 0: x at [0, 8),
    // W_hh at [8, 72); layers >= 1: W_ih at [0, 64), W_hh at [64, 128) (+128 per tile).
    const uint32_t a_rec0 = l == 0 ? 8u : 64u;
    const uint64_t dAl = ptx::desc_k_sw128(sbase + S::kALin);
    const uint64_t dB0 = ptx::desc_k_sw128(bbuf(0));
    const uint64_t dBx0 = ptx::desc_k_none(bbuf(0), 128, 256);
    constexpr uint64_t kBufStep = (uint64_t)(S::kBufBytes >> 4);
    const uint32_t lin_row_off = S::kSplitLinear ? (uint32_t)(s * NL) * 128u : 0u;
    const int steps = Tt + (does_linear ? 1 : 0);
    int last_commit = -1;

    auto x_src = [&](int t) { return p.xp + ((size_t)tile * p.T + t) * xbytes; };  // layer 0 only
    // Input part of step t (W_ih . x_t) into D[t & 1]; it initialises the accumulator.
    auto issue_in = [&](int t) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = dB0 + kBufStep * b;
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const uint32_t a = tmem + (uint32_t)(tau * 128);
          if (l == 0) {
            ptx::mma_f16_ts(dcol(b, tau), a, dBx0 + kBufStep * b, idesc_g, 0u);
          } else {
#pragma unroll
            for (int kb = 0; kb < 2; ++kb)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                ptx::mma_f16_ts(dcol(b, tau), a + (uint32_t)(32 * kb + 8 * kk),
                                dB + (uint64_t)((kb * S::kBKB + kk * 32) >> 4), idesc_g, (kb | kk) != 0 ? 1u : 0u);
          }
        }
        // Layer l-1 may overwrite this input slot once these MMAs are done.
        if (l > 0 && t + 2 < Tt) ptx::mma_commit_mc(bar_empty + 8 * b, up_mask);
      }
      __syncwarp();
    };
    auto issue_rec_half = [&](int t, int kb) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = dB0 + kBufStep * b;
#pragma unroll
        for (int tau = 0; tau < 2; ++tau)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            ptx::mma_f16_ts(dcol(b, tau), tmem + (uint32_t)(tau * 128) + a_rec0 + (uint32_t)(32 * kb + 8 * kk),
                            dB + (uint64_t)(((2 + kb) * S::kBKB + kk * 32) >> 4), idesc_g, 1u);
      }
      __syncwarp();
    };
    auto issue_lin_commit = [&](int t, bool lin) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = dB0 + kBufStep * b;
        if (lin) {
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              ptx::mma_f16_ss(tmem + (uint32_t)S::kDLin, dAl + (uint64_t)((kb * kATileKB + kk * 32) >> 4),
                              dB + (uint64_t)(((2 + kb) * S::kBKB + lin_row_off + kk * 32) >> 4), idesc_l,
                              (kb | kk) != 0 ? 1u : 0u);
        }
        ptx::mma_commit(bar_mma + 8 * b);
      }
      __syncwarp();
    };
    bool ok = true;
    auto fail = [&](int t) {
      if (ptx::elect_one()) raise_abort(p, sm + S::kAbort, ncta, t);
      __syncwarp();
      ok = false;
    };

    // Prologue: expected bytes of steps 0 / 1 (inputs) and 1 / 2 (sibling h), x of steps 0 / 1.
    if (ptx::elect_one()) {
      for (int t = 0; t < 2 && t < Tt; ++t) {
        ptx::mbar_arrive_expect_tx(bar_in + 8 * t, in_bytes);
        if (l == 0) ptx::bulk_g2s(bbuf(t), x_src(t), xbytes, bar_in + 8 * t);
      }
      for (int t = 1; t <= 2; ++t)
        if (t < Tt || (does_linear && t == Tt))
          ptx::mbar_arrive_expect_tx(bar_rec + 8 * (t & 1), bkb);
    }
    __syncwarp();
    if (Tt > 0) {
      if (!warp_wait_phase(bar_in, 0, abort_flag, p.timeout_ns)) {
        fail(0);
      } else {
        issue_in(0);
        if (2 < Tt && ptx::elect_one()) ptx::mbar_arrive_expect_tx(bar_in, in_bytes);
        __syncwarp();
      }
    }
    // Layer 0: streams x of step t+2 into the input slot step t has finished with
    // (h(t) itself is pushed by the last compute warp to finish the step).
    auto hand_off = [&](int t) {
      const int b = t & 1;
      if (l == 0 && t + 2 < Tt && ptx::elect_one()) ptx::bulk_g2s(bbuf(b), x_src(t + 2), xbytes, bar_in + 8 * b);
      __syncwarp();
    };
    for (int t = 0; ok && t < steps; ++t) {
      const int b = t & 1;
      const bool gates = t < Tt;
      const bool lin = does_linear && (t == Tt || (MODE == kModeSeq && t >= 1));
      if (gates) issue_rec_half(t, s);  // own half of h_{t-1}: written before the previous step ended
      if (lane == 0) trace_mark(p, rank, t, 3);
      if (t >= 1) {
        if (!warp_wait_phase(bar_rec + 8 * b, ((t - 1) >> 1) & 1, abort_flag, p.timeout_ns)) {
          fail(t);
          break;
        }
        if ((t + 2 < Tt || (does_linear && t + 2 == Tt)) && ptx::elect_one())
          ptx::mbar_arrive_expect_tx(bar_rec + 8 * b, bkb);
        __syncwarp();
      }
      if (lane == 0) trace_mark(p, rank, t, 0);
      if (gates) issue_rec_half(t, 1 - s);
      issue_lin_commit(t, lin);
      last_commit = t;
      if (lane == 0) trace_mark(p, rank, t, 1);
      if (!gates) break;  // drain step issued
      // This step's h hand-off and the next step's input MMAs, whichever is ready first
      // (the hand-off first when both are).
      bool in_pending = t + 1 < Tt, copy_pending = true;
      const unsigned long long t0 = ptx::globaltimer();
      unsigned spins = 0;
      while (in_pending || copy_pending) {
        if (copy_pending && warp_test_wait(bar_hready + 8 * b, (t >> 1) & 1)) {
          if (lane == 0) trace_mark(p, rank, t, 2);
          hand_off(t);
          copy_pending = false;
          continue;
        }
        if (in_pending && warp_test_wait(bar_in + 8 * (b ^ 1), ((t + 1) >> 1) & 1)) {
          issue_in(t + 1);
          if (t + 3 < Tt && ptx::elect_one()) ptx::mbar_arrive_expect_tx(bar_in + 8 * (b ^ 1), in_bytes);
          __syncwarp();
          in_pending = false;
          continue;
        }
        if ((++spins & 31) == 0) {  // abort / timeout checks are slow: every 32 polls
          int bad = 0;
          if (lane == 0) bad = (*abort_flag != 0) || (ptx::globaltimer() - t0 > p.timeout_ns);
          if (__shfl_sync(0xffffffffu, bad, 0)) {
            fail(t);
            break;
          }
        }
      }
    }
    // All MMAs must have completed before TMEM is released.
    if (last_commit >= 0 && lane == 0)
      wait_phase(bar_mma + 8 * (last_commit & 1), (last_commit >> 1) & 1, abort_flag, p.timeout_ns);
    __syncwarp();
  } else {
    // =========================== compute warps ===========================
    const int q = warp & 3, grp = warp >> 2;
    const int j8 = lane >> 2;          // unit within the quadrant's group of 8
    const int cpair = (lane & 3) * 2;  // first of the two batch columns in a chunk
    // cells: [tau][chunk j][e]
    float c_st[2][CPW][2];
    uint16_t h_st[2][CPW][2];  // h bits (the frozen value of finished rows)
    int ncol[CPW][2], len_c[CPW][2], bidx[CPW][2];
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = 8 * (grp * CPW + jc) + cpair + e;
        ncol[jc][e] = n;
        len_c[jc][e] = lens_s[n];
        bidx[jc][e] = perm_s[n];
      }
#pragma unroll
    for (int tau = 0; tau < 2; ++tau) {
      const int u = 64 * s + 8 * (4 * tau + q) + j8;
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int b = bidx[jc][e];
          uint16_t hv = 0;
          float cv = 0.0f;
          if (b >= 0 && p.h0 != nullptr && u < p.hid) {
            hv = static_cast<const uint16_t*>(p.h0)[((size_t)l * p.B + b) * p.hid + u];
            cv = from_bits<BF16>(static_cast<const uint16_t*>(p.c0)[((size_t)l * p.B + b) * p.hid + u]);
          }
          h_st[tau][jc][e] = hv;
          c_st[tau][jc][e] = cv;
        }
    }
    // f32 gate bias of this thread's two units (i, f, o rows pre-scaled by 1/2 like the
    // weights), added to the accumulators in registers (the pointwise stage has spare issue slots).
    float bz[2][4];
    {
      const float* bias_img = reinterpret_cast<const float*>(p.packed + packed_bias_off(p.L)) + rank * 256;
#pragma unroll
      for (int tau = 0; tau < 2; ++tau)
#pragma unroll
        for (int g = 0; g < 4; ++g) bz[tau][g] = bias_img[tau * 128 + 32 * q + 8 * g + j8];
    }
    const float* blin = reinterpret_cast<const float*>(p.packed + packed_blin_off(p.L));
    const bool lin_warp = does_linear && q == 0;
    const int o = lane;  // Linear output row handled by this lane (lin_warp only)
    const float blin_o = (lin_warp && o < p.O) ? blin[o] : 0.0f;
    uint16_t* out16 = static_cast<uint16_t*>(p.out);
    const int lin_n0 = (S::kSplitLinear ? s * NL : 0) + grp * (NL / G);  // first batch column of this warp

    // This warp's columns of the Linear accumulator (lanes = output rows).
    constexpr int kLinChunks = NL / G / 8;
    auto load_linear = [&](uint32_t (&r)[kLinChunks][8]) {
#pragma unroll
      for (int c = 0; c < kLinChunks; ++c)
        ptx::tmem_ld_32x32b_x8(tmem + (uint32_t)(S::kDLin + grp * (NL / G) + 8 * c), r[c]);
      ptx::tmem_wait_ld();
    };
    // Stores the Linear outputs of step `ts` (or, last_mode, the [B][O] result).  In the
    // step loop this runs after the step's barrier arrivals: an arrive has release
    // semantics and would wait for global stores issued before it to complete.
    auto write_linear = [&](int ts, const uint32_t (&r)[kLinChunks][8], bool last_mode) {
      if (o >= p.O) return;
      // Two columns rounded to 16 bits per instruction (the single-value conversion issues on
      // the pipe the gate math's tanh runs on).
#pragma unroll
      for (int c = 0; c < kLinChunks; ++c)
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const int n = lin_n0 + 8 * c + i;
          float v[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            v[e] = __uint_as_float(r[c][i + e]) + blin_o;
            if (!last_mode && ts >= lens_s[n + e]) v[e] = 0.0f;
          }
          const uint32_t bits = pack2_bits<BF16>(v[0], v[1]);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int b = perm_s[n + e];
            if (b < 0) continue;
            const uint16_t hb = (uint16_t)(e == 0 ? bits & 0xffffu : bits >> 16);
            if (last_mode)
              out16[(size_t)b * p.O + o] = hb;
            else
              out16[((size_t)b * p.T + ts) * p.O + o] = hb;
          }
        }
    };
    auto store_linear = [&](int ts, bool last_mode) {
      uint32_t r[kLinChunks][8];
      load_linear(r);
      write_linear(ts, r, last_mode);
    };

    uint32_t lin_r[kLinChunks][8];  // Linear accumulator of step t-1, stored at the end of step t
    for (int t = 0; t < Tt; ++t) {
      const int b = t & 1;
      if (*abort_flag) break;
      if (!wait_phase(bar_mma + 8 * b, (t >> 1) & 1, abort_flag, p.timeout_ns)) {
        if (lane == 0) raise_abort(p, sm + S::kAbort, ncta, t);
        break;
      }
      ptx::tc_fence_after();
      if (tid == 0) trace_mark(p, rank, t, 4);
      uint32_t rif[2][4 * CPW], rgo[2][4 * CPW];
#pragma unroll
      for (int tau = 0; tau < 2; ++tau) {
        const uint32_t col = dcol(b, tau) + (uint32_t)(grp * CPW * 8);
        tmem_ld_chunks<CPW>(col + ((uint32_t)(32 * q) << 16), rif[tau]);
        tmem_ld_chunks<CPW>(col + ((uint32_t)(32 * q + 16) << 16), rgo[tau]);
      }
      ptx::tmem_wait_ld();
      if (tid == 0) trace_mark(p, rank, t, 5);
      if (MODE == kModeSeq && lin_warp && t >= 1) load_linear(lin_r);
      ptx::tc_fence_before();

      // Layer l+1 must have consumed h_{t-2} (same buffer and copy source) before it is overwritten.
      if (l + 1 < p.L && t >= 2) {
        if (!wait_phase(bar_empty + 8 * b, ((t - 2) >> 1) & 1, abort_flag, p.timeout_ns)) {
          if (lane == 0) raise_abort(p, sm + S::kAbort, ncta, t);
          break;
        }
      }
      uint16_t hw[2][CPW][2];
      lstm_cells<CPW, BF16, VARLEN>(rif, rgo, bz, c_st, h_st, len_c, t, hw);
      uint8_t* dst = sm + S::kB + (b ^ 1) * S::kBufBytes + (2 + s) * S::kBKB;
#pragma unroll
      for (int tau = 0; tau < 2; ++tau) {
        const int ul = 8 * (4 * tau + q) + j8;  // unit within this CTA's 64
#pragma unroll
        for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
          for (int e = 0; e < 2; ++e) *reinterpret_cast<uint16_t*>(dst + sw128_off(ncol[jc][e], ul)) = hw[tau][jc][e];
      }
      ptx::fence_proxy_async_smem();
      if (tid == 0) trace_mark(p, rank, t, 6);
      if (tid == 32 * (kComputeWarps - 1)) trace_mark(p, rank, t, 7);
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(bar_hready + 8 * b);  // the control warp: own half of the next step's MMAs
        // The last warp to finish pushes the tile (acquire-release counter: the other
        // warps' writes, fenced for the async proxy, are ordered before its copies).
        if (ptx::atom_add_acq_rel_smem(sbase + S::kDone, 1u) % (uint32_t)kComputeWarps == kComputeWarps - 1u) {
          const bool to_sibling = ((t + 1 < Tt) || (sibling_linear && t + 1 == Tt)) &&
                                  !(rank == p.drop_rank && t == p.drop_step);
          push_h(sbase + (uint32_t)(S::kB + (b ^ 1) * S::kBufBytes + (2 + s) * S::kBKB), S::kBKB, rank, to_sibling,
                 bar_rec + 8 * (b ^ 1), l + 1 < p.L, 2 * (l + 1),
                 sbase + (uint32_t)(S::kB + b * S::kBufBytes + s * S::kBKB), bar_in + 8 * b);
        }
      }
      // Global outputs of the step, after its arrivals (see write_linear).
      if (MODE == kModeSeq && lin_warp && t >= 1) write_linear(t - 1, lin_r, false);
      if (MODE == kModeHSeq && last_layer) {
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const int ul = 8 * (4 * tau + q) + j8;
#pragma unroll
          for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
            for (int e = 0; e < 2; ++e)
              if (bidx[jc][e] >= 0 && 64 * s + ul < p.hid)
                out16[((size_t)bidx[jc][e] * p.T + t) * p.hid + 64 * s + ul] =
                    (!VARLEN || t < len_c[jc][e]) ? hw[tau][jc][e] : (uint16_t)0;
        }
      }
    }
    // Drain: Linear of the last step's h.
    if (lin_warp && !*abort_flag) {
      if (wait_phase(bar_mma + 8 * (Tt & 1), (Tt >> 1) & 1, abort_flag, p.timeout_ns)) {
        ptx::tc_fence_after();
        if (MODE == kModeSeq) {
          if (Tt >= 1) store_linear(Tt - 1, false);
        } else {
          store_linear(0, true);
        }
        ptx::tc_fence_before();
      } else if (lane == 0) {
        raise_abort(p, sm + S::kAbort, ncta, Tt);
      }
    }
    // Outputs past the tile's last step are zero.
    if (MODE == kModeSeq && lin_warp && o < p.O) {
      for (int i = 0; i < NL / G; ++i) {
        const int n = lin_n0 + i;
        const int b = perm_s[n];
        if (b < 0) continue;
        for (int ts = Tt; ts < p.T; ++ts) out16[((size_t)b * p.T + ts) * p.O + o] = 0;
      }
    }
    if (MODE == kModeHSeq && last_layer) {
#pragma unroll
      for (int tau = 0; tau < 2; ++tau) {
        const int u = 64 * s + 8 * (4 * tau + q) + j8;
#pragma unroll
        for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int bb = bidx[jc][e];
            if (bb < 0 || u >= p.hid) continue;
            for (int ts = Tt; ts < p.T; ++ts) out16[((size_t)bb * p.T + ts) * p.hid + u] = 0;
          }
      }
    }
    // Final state.
#pragma unroll
    for (int tau = 0; tau < 2; ++tau) {
      const int u = 64 * s + 8 * (4 * tau + q) + j8;
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int bb = bidx[jc][e];
          if (bb < 0 || u >= p.hid) continue;
          const size_t idx = ((size_t)l * p.B + bb) * p.hid + u;
          if (p.h_n != nullptr) static_cast<uint16_t*>(p.h_n)[idx] = h_st[tau][jc][e];
          if (p.c_n != nullptr) {
            if (p.flags & PLSTM_FLAG_CN_F32)
              static_cast<float*>(p.c_n)[idx] = c_st[tau][jc][e];
            else
              static_cast<uint16_t*>(p.c_n)[idx] = to_bits<BF16>(c_st[tau][jc][e]);
          }
        }
    }
  }

  // ---- teardown -----------------------------------------------------------------
  if (*abort_flag) {
    // Let bulk copies already in flight toward peers land before any CTA leaves.
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

// ---- two-slot wavefront kernel -------------------------------------------------------
// Same cluster layout, weight residency and per-step protocol as wavefront_kernel, but
// each cluster tile of N = 2 NH batch rows runs as two independent slots of NH rows.
// The two recurrences have no data dependence on each other, so while one slot waits
// on its MMA pipeline, its TMEM loads or the DSMEM hand-off to the sibling CTA, the
// other slot's compute warps run their gate math: the latency of one slot's step is
// hidden behind the other's MUFU work.  Each slot has its own compute warps (one per
// TMEM lane quadrant), its own control warp, B buffers and barriers; the slots share
// the CTA's resident weights (TMEM columns [0, 256)) and the Linear head's A image.
// Each slot's gate accumulator is single-buffered (TMEM holds A + 2 slots x 2 tiles x
// NH columns + the Linear tiles): the next step's input MMAs wait until the compute
// warps have loaded the current accumulator ("dfree").  With [B][T][O] output the
// Linear head's MMAs have their own commit barrier and a double-buffered accumulator;
// each slot's head runs whole on the last-layer CTA of the slot's parity and is read by
// that CTA's output warp (the head's rows are replicated into every TMEM lane quadrant),
// so neither the gate math nor the global stores of the outputs sit on the recurrence's
// critical path.
template <int NH, int NSL = 2>
struct Smem2 {
  static constexpr int kBKB = NH * 128;             // one 64-wide K block of a slot's B operand
  static constexpr int kBufBytes = 4 * kBKB;        // [in0 | in1 | rec0 | rec1]
  static constexpr int kSlotBytes = 2 * kBufBytes;  // step-parity double buffer
  static constexpr int kB = 0;
  static constexpr int kALin = kB + NSL * kSlotBytes;
  static constexpr int kBar = kALin + kALinBytes;
  // Per slot: eight barrier kinds, one per buffer parity (8 bytes each).
  static constexpr int kFullIn = 0, kFullRec = 16, kEmpty = 32, kHReady = 48, kMma = 64, kDFree = 80, kLin = 96,
                       kLinFree = 112;
  static constexpr int kBarSlot = 128;
  static constexpr int kTmemSlot = kBar + NSL * kBarSlot, kAbort = kTmemSlot + 4, kDone = kTmemSlot + 8;
  static constexpr int kPerm = kTmemSlot + 64, kLens = kPerm + 4 * NSL * NH;
  // [B][T][O] mode: one step's Linear outputs of an output warp's slot, [row][o] 16-bit with a
  // 64-byte row pitch (O <= 32), staged for 16-byte global stores.
  static constexpr int kOutPitch = 64;
  static constexpr int kOutStage = kLens + 4 * NSL * NH;
  static constexpr int kEnd = kOutStage + ((NSL + 1) / 2) * NH * kOutPitch;
  static constexpr int kDynBytes = kEnd + 1024;  // + alignment slack
  static constexpr int CPW = NH / 8;               // 8-column chunks per compute warp (all NH columns)
  static constexpr int kSlotWarps = 4;             // compute warps per slot: one per TMEM lane quadrant
  static constexpr int kComputeWarps = NSL * kSlotWarps;
  static constexpr int kOutWarp0 = kComputeWarps + NSL;  // after one control warp per slot
  // + one more warp: in [B][T][O] mode a last-layer CTA's output warp (it stores the Linear outputs
  // of the slots s, s + 2, ... whose heads the CTA computes), in layer 0 the x warp, which reads
  // x[B][T][I] into the input tiles (a layer 0 that is also the last layer in [B][T][O] mode takes
  // the repacked x instead).
  static constexpr int xwarp(int) { return kOutWarp0; }
  static constexpr int threads(int mode) { return (kOutWarp0 + (mode == kModeSeq ? kOutWarps : 1)) * 32; }
  // The Linear head of a slot runs whole on the last-layer CTA of the slot's parity (kSplitLinear
  // false; splitting a 32-row slot's head over both CTAs gave each CTA's output warp two slots).
  static constexpr bool kSplitLinear = false;
  static constexpr int kNL = NH;
  // [B][T][O] mode: output warps per CTA, each storing the heads of kOutSlotsPerWarp of the
  // ceil(NSL / 2) slots the CTA owns the heads of.  One warp for all: a second one would take the
  // three-slot block past 16 warps and cap its registers at 96, which slows every layer's gate math
  // more than the output warp's work costs.
  static constexpr int kOutSlotsPerWarp = (NSL + 1) / 2;
  static constexpr int kOutWarps = (NSL + 1) / 2 / kOutSlotsPerWarp;
  static constexpr int kD = kTmemACols;            // D[slot][tau] at kD + (2 slot + tau) NH
  static constexpr int kDLin = kD + 2 * NSL * NH;  // D_lin[slot][buffer] at kDLin + (2 slot + buffer) NL
  static constexpr int kTmemCols = tmem_cols_for(kDLin + 2 * NSL * kNL);
  static_assert(kDLin + 2 * NSL * kNL <= 512, "tile too wide for tensor memory");
  static_assert(NH % 16 == 0 && CPW >= 2 && CPW <= 4, "slot width must be 16 or 32");
  static_assert(NSL >= 2 && NSL <= 3 && kDone + 4 * NSL <= kPerm, "two or three slots");
};

template <int NH, int NSL, bool BF16, bool VARLEN, int MODE>
__global__ void __launch_bounds__(Smem2<NH, NSL>::threads(MODE), 1) wavefront2_kernel(const Params p) {
  using S = Smem2<NH, NSL>;
  constexpr int N = NSL * NH;
  constexpr int kThreads = S::threads(MODE);
  constexpr int CPW = S::CPW;
  constexpr int NL = S::kNL;
  constexpr int kComputeWarps = S::kComputeWarps;
  constexpr bool kHasLinear = MODE != kModeHSeq;
  // The launch of the tile height not chosen ends here, before any barrier, TMEM or cluster traffic.
  if (p.choice != nullptr && *p.choice != N) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ncta = 2 * p.L;
  const int rank = (int)ptx::cluster_ctarank();
  const int l = rank >> 1, s = rank & 1;
  const int tile = blockIdx.x / ncta;
  const bool last_layer = l == p.L - 1;
  // Extents the bounds-check build tests indices against (bc_ok; compiled out otherwise).
  int* const st = p.status;
  const size_t n_tiles = gridDim.x / ncta;
  const size_t packed_bytes = packed_total(p.L);
  const size_t state_elems = (size_t)p.L * p.B * p.hid;
  const bool drain = kHasLinear && last_layer;
  // The Linear head of a slot: split over both last-layer CTAs when half the slot is a legal
  // MMA width, else computed by the CTA of the slot's parity (so the slots' heads are spread
  // over both CTAs).
  auto does_lin = [&](int sl) { return drain && (S::kSplitLinear || s == (sl & 1)); };
  auto sibling_lin = [&](int sl) { return drain && (S::kSplitLinear || s != (sl & 1)); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::kAbort);
  int32_t* perm_s = reinterpret_cast<int32_t*>(sm + S::kPerm);
  int32_t* lens_s = reinterpret_cast<int32_t*>(sm + S::kLens);
  auto bar = [&](int sl, int kind, int par) -> uint32_t {
    return sbase + (uint32_t)(S::kBar + sl * S::kBarSlot + kind + 8 * par);
  };
  auto bbuf = [&](int sl, int b) -> uint32_t {
    return sbase + (uint32_t)(S::kB + sl * S::kSlotBytes + b * S::kBufBytes);
  };

  // ---- set-up ------------------------------------------------------------------
  if (tid == 0) {
    for (int sl = 0; sl < NSL; ++sl)
      for (int b = 0; b < 2; ++b) {
        ptx::mbar_init(bar(sl, S::kFullIn, b), 1);
        ptx::mbar_init(bar(sl, S::kFullRec, b), 1);
        ptx::mbar_init(bar(sl, S::kEmpty, b), 2);
        ptx::mbar_init(bar(sl, S::kHReady, b), S::kSlotWarps);
        ptx::mbar_init(bar(sl, S::kMma, b), 1);
        ptx::mbar_init(bar(sl, S::kDFree, b), S::kSlotWarps);
        ptx::mbar_init(bar(sl, S::kLin, b), 1);
        ptx::mbar_init(bar(sl, S::kLinFree, b), 1);
      }
    *abort_flag = 0;
    for (int sl = 0; sl < NSL; ++sl) reinterpret_cast<uint32_t*>(sm + S::kDone)[sl] = 0;
    ptx::fence_mbar_init_cluster();
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + S::kTmemSlot, S::kTmemCols);
    ptx::tmem_relinquish();
  }
  for (int i = tid; i < N; i += kThreads) {
    const int b = bc_ok(st, (size_t)tile * N + i < n_tiles * N, 1) ? p.perm[tile * N + i] : -1;
    perm_s[i] = b;
    int len = 0;
    if (b >= 0 && bc_ok(st, b < p.B, 2)) len = VARLEN ? min(max(p.lengths[b], 0), p.T) : p.T;
    lens_s[i] = len;
  }
  if (drain) {
    // The head's rows (O <= 32, rows 0-31 of the packed image) are replicated into
    // every 32-row lane quadrant; 8-row swizzle groups keep their XOR pattern.
    const uint4* srcl = reinterpret_cast<const uint4*>(p.packed + packed_alin_off(p.L));
    uint4* dstl = reinterpret_cast<uint4*>(sm + S::kALin);
    for (int i = tid; i < kALinBytes / 16; i += kThreads) {
      const int kb = i / (kATileKB / 16), r = (i / 8) % 128, c = i % 8;
      const size_t si = (size_t)kb * (kATileKB / 16) + (r & 31) * 8 + c;
      if (bc_ok(st, packed_alin_off(p.L) + 16 * (si + 1) <= packed_bytes, 3)) dstl[i] = srcl[si];
    }
  }
  __syncthreads();  // perm_s / lens_s / tmem slot visible
  // Initial recurrent state h0 -> both recurrent K blocks of each slot's B buffer 0.
  for (int i = tid; i < N * kH; i += kThreads) {
    const int n = i / kH, k = i % kH;
    const int sl = n / NH, nn = n % NH;
    float v = 0.0f;
    const int b = perm_s[n];
    if (p.h0 != nullptr && b >= 0 && k < p.hid && bc_ok(st, ((size_t)l * p.B + b) * p.hid + k < state_elems, 4)) {
      const uint16_t* h0 = static_cast<const uint16_t*>(p.h0);
      v = from_bits<BF16>(h0[((size_t)l * p.B + b) * p.hid + k]);
    }
    const uint32_t off = S::kB + sl * S::kSlotBytes + (2 + (k >> 6)) * S::kBKB + sw128_off(nn, k & 63);
    if (bc_ok(st, off + 2 <= (uint32_t)S::kALin, 5)) *reinterpret_cast<uint16_t*>(sm + off) = to_bits<BF16>(v);
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + S::kTmemSlot);
  // This CTA's weight slice -> TMEM columns [0, 256): warps 0-3 store tile 0, warps
  // 4-7 tile 1, each its lane quadrant's 32 rows.
  if (warp < 8) {
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const int tau = warp >> 2;
    const uint4* src =
        reinterpret_cast<const uint4*>(p.packed + (size_t)rank * kABytes + ((size_t)tau * 128 + row) * kAK * 2);
#pragma unroll 1
    for (int c = 0; c < kAK / 2; c += 32) {
      uint32_t r[32];
      const bool a_in = bc_ok(st, (size_t)rank * kABytes + ((size_t)tau * 128 + row) * kAK * 2 + 16 * (c / 4 + 8) <=
                                      packed_alin_off(p.L), 6) &&
                        bc_ok(st, tau * 128 + c + 32 <= S::kTmemCols, 7);
      if (!a_in) continue;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = src[c / 4 + i];
        r[4 * i + 0] = v.x;
        r[4 * i + 1] = v.y;
        r[4 * i + 2] = v.z;
        r[4 * i + 3] = v.w;
      }
      ptx::tmem_st_32x32b_x32(tmem + lane_off + (uint32_t)(tau * 128 + c), r);
    }
    ptx::tmem_wait_st();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::cluster_sync();  // every CTA's barriers are initialised before any remote operation

  // Each slot runs as many steps as its longest row (rows are sorted by length for
  // variable lengths); a slot without rows does nothing.
  auto slot_len = [&](int sl, bool* any) -> int {
    int m = 0;
    bool a = false;
    for (int i = 0; i < NH; ++i) {
      a |= perm_s[sl * NH + i] >= 0;
      m = max(m, lens_s[sl * NH + i]);
    }
    *any = a;
    return m;
  };
  auto dcol = [&](int sl, int tau) -> uint32_t { return tmem + (uint32_t)(S::kD + (2 * sl + tau) * NH); };
  // The Linear MMAs issued at step t (on h_{t-1}; at t = T only in [B][O] mode) commit
  // to kLin[lin_buf(t)] and accumulate into D_lin[sl][lin_buf(t)]; lin_phase(t) is the
  // parity that commit completes.
  auto lin_buf = [&](int t) -> int { return MODE == kModeSeq ? (t - 1) & 1 : 0; };
  auto lin_phase = [&](int t) -> uint32_t { return MODE == kModeSeq ? (uint32_t)((t - 1) >> 1) & 1u : 0u; };
  auto dlin_at = [&](int sl, int t) -> uint32_t {
    return tmem + (uint32_t)(S::kDLin + (2 * sl + lin_buf(t)) * NL);
  };

  const bool x_warp = warp == S::xwarp(MODE) && l == 0 && p.xp == nullptr && !(MODE == kModeSeq && last_layer);
  if (x_warp) {
    // ============================== x warp ===============================
    // Layer 0 without a repacked x (xp null, I <= 16): lane n < NH holds row n of every slot
    // and writes x_t of it into the slot's input tile (kx = 16: K group 0 = columns 0-7 at
    // 8-row groups 256 bytes apart, K group 1 = columns 8-15 128 bytes further), two steps
    // ahead of the MMAs that read it (the tile of step t + 2 reuses step t's buffer once step
    // t's gate math has started, i.e. its MMAs are done: HReady).  The global loads of x_{t+3}
    // are issued right after x_{t+2} is written, so their latency hides under a whole step,
    // and every row is prefetched into L2 kXPrefetch steps ahead, so that those loads hit L2
    // even when x starts out in HBM (a step is shorter than an HBM miss).
    {
      const int I = p.I;
      int Tt[NSL];
      for (int sl = 0; sl < NSL; ++sl) {
        bool a = false;
        Tt[sl] = slot_len(sl, &a);
      }
      // Rows / columns never written stay zero: clear both parity tiles of every slot.
      for (int sl = 0; sl < NSL; ++sl)
        for (int b = 0; b < 2; ++b)
          for (int i = lane; i < NH * 16 * 2 / 16; i += 32)
            reinterpret_cast<uint4*>(sm + S::kB + sl * S::kSlotBytes + b * S::kBufBytes)[i] = make_uint4(0, 0, 0, 0);
      // Loads leave the 16-bit values raw in registers; they are packed only when the tile is
      // written (the next iteration), so the warp never waits for its own loads in between.
      auto load_row = [&](int sl, int t, uint32_t (&raw)[16]) {
        const int b = lane < NH ? perm_s[sl * NH + lane] : -1;
        const bool live = b >= 0 && t < Tt[sl] && bc_ok(st, b < p.B && t < p.T, 8);
        const uint16_t* src = p.x_raw + ((size_t)max(b, 0) * p.T + t) * I;
#pragma unroll
        for (int k = 0; k < 16; ++k) raw[k] = (live && k < I) ? (uint32_t)__ldg(src + k) : 0u;
      };
      constexpr int kXPrefetch = 24;
      auto prefetch_row = [&](int sl, int t) {
        const int b = lane < NH ? perm_s[sl * NH + lane] : -1;
        if (b >= 0 && t < Tt[sl]) ptx::prefetch_l2(p.x_raw + ((size_t)b * p.T + t) * I);
      };
      auto write_row = [&](int sl, int b, const uint32_t (&raw)[16]) {
        if (lane >= NH) return;
        if (!bc_ok(st, (lane >> 3) * 256 + (lane & 7) * 16 + (I > 8 ? 144 : 16) <= 2 * S::kBKB, 9)) return;
        uint8_t* dst = sm + S::kB + sl * S::kSlotBytes + b * S::kBufBytes + (lane >> 3) * 256 + (lane & 7) * 16;
        *reinterpret_cast<uint4*>(dst) = make_uint4(raw[0] | raw[1] << 16, raw[2] | raw[3] << 16,
                                                    raw[4] | raw[5] << 16, raw[6] | raw[7] << 16);
        if (I > 8)
          *reinterpret_cast<uint4*>(dst + 128) = make_uint4(raw[8] | raw[9] << 16, raw[10] | raw[11] << 16,
                                                            raw[12] | raw[13] << 16, raw[14] | raw[15] << 16);
      };
      uint32_t v[NSL][16];
      // The first kXPrefetch steps of every row into L2 (one prefetch per 64 bytes of a row).
      for (int sl = 0; sl < NSL; ++sl)
        for (int t = 0; t < kXPrefetch; t += max(1, 64 / (2 * I))) prefetch_row(sl, t);
      // Steps 0 and 1, then x_2 into registers.
      for (int t = 0; t < 2; ++t)
        for (int sl = 0; sl < NSL; ++sl) {
          if (t >= Tt[sl]) continue;
          load_row(sl, t, v[sl]);
          write_row(sl, t, v[sl]);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar(sl, S::kFullIn, t));
        }
      int Tmax = 0;
      for (int sl = 0; sl < NSL; ++sl) {
        load_row(sl, 2, v[sl]);
        Tmax = max(Tmax, Tt[sl]);
      }
      bool ok = true;
      for (int t = 0; ok && t + 2 < Tmax; ++t) {
        const int b = t & 1;
        for (int sl = 0; sl < NSL; ++sl) {
          if (t + 2 >= Tt[sl]) continue;
          if (!warp_wait_phase(bar(sl, S::kHReady, b), (t >> 1) & 1, abort_flag, p.timeout_ns)) {
            if (lane == 0 && !*abort_flag) raise_abort(p, sm + S::kAbort, ncta, t);
            ok = false;
            break;
          }
          write_row(sl, b, v[sl]);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar(sl, S::kFullIn, b));
          load_row(sl, t + 3, v[sl]);
          prefetch_row(sl, t + 3 + kXPrefetch);
        }
      }
    }
  } else if (warp >= S::kOutWarp0) {
    // ============================ output warps ===========================
    // [B][T][O] mode: the output warp of a last-layer CTA stores the Linear outputs of every step
    // of the slots whose heads this CTA computes, read from each slot's Linear accumulator in this
    // warp's lane quadrant (the head's rows are replicated into all four), off the critical path.
    if (MODE == kModeSeq) {
      const int o = lane;
      const float blin_o = o < p.O ? reinterpret_cast<const float*>(p.packed + packed_blin_off(p.L))[o] : 0.0f;
      uint16_t* out16 = static_cast<uint16_t*>(p.out);
      const uint32_t qlane = (uint32_t)(32 * (warp & 3)) << 16;
      // A step's outputs go out as few wide stores: each row's O values are staged in shared
      // memory and copied in chunks of cb bytes (16 when O % 8 == 0), one chunk per lane, with the
      // chunks' addresses worked out once.  (A 2-byte store per row and lane cost ~130 cycles a
      // row, longer than a step for 32 rows.)
      const uintptr_t oaddr = reinterpret_cast<uintptr_t>(p.out);
      const int cb = (p.O % 8 == 0 && oaddr % 16 == 0) ? 16
                     : (p.O % 4 == 0 && oaddr % 8 == 0) ? 8
                     : (p.O % 2 == 0 && oaddr % 4 == 0) ? 4 : 2;
      const int cpr = 2 * p.O / cb;  // chunks per row
      const int nchunks = NL * cpr;
      constexpr int kPer = S::kOutSlotsPerWarp;
      constexpr int kPlan = 4;  // chunks per lane with precomputed addresses (the rest: per step)
      const size_t row_bytes = (size_t)p.T * p.O * 2;
      auto copy_chunk = [&](uint32_t src, uint8_t* dst) {
        if (cb == 16)
          *reinterpret_cast<uint4*>(dst) = ptx::ld_shared_v4(src);
        else if (cb == 8)
          *reinterpret_cast<uint2*>(dst) = ptx::ld_shared_v2(src);
        else if (cb == 4)
          *reinterpret_cast<uint32_t*>(dst) = ptx::ld_shared_u32(src);
        else
          *reinterpret_cast<uint16_t*>(dst) = ptx::ld_shared_u16(src);
      };
      // The slots this warp stores: sl = s + 2 (w kPer + k) for output warp w; lane i holds the
      // batch row and length of head column i of each.
      // A slot whose rows all have length 0 has Tts 0 but still owns rows (written as zeros).
      int sls[kPer], Tts[kPer], my_b[kPer], my_len[kPer];
      bool owns[kPer];
      uint32_t stage[kPer], ch_src[kPer][kPlan];
      long long ch_dst[kPer][kPlan];  // byte offset of the chunk in out at t = 0, or -1
      int Tmax = 0;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        sls[k] = s + 2 * ((warp - S::kOutWarp0) * kPer + k);
        bool active = false;
        Tts[k] = (sls[k] < NSL && does_lin(sls[k])) ? slot_len(sls[k], &active) : 0;
        owns[k] = sls[k] < NSL && does_lin(sls[k]) && active;
        if (!owns[k]) Tts[k] = 0;
        Tmax = max(Tmax, Tts[k]);
        const int lin_n0 = min(sls[k], NSL - 1) * NH;
        my_b[k] = (owns[k] && lane < NL) ? perm_s[lin_n0 + lane] : -1;
        my_len[k] = (owns[k] && lane < NL) ? lens_s[lin_n0 + lane] : 0;
        stage[k] = sbase + (uint32_t)(S::kOutStage + ((warp - S::kOutWarp0) * kPer + k) * NH * S::kOutPitch);
#pragma unroll
        for (int it = 0; it < kPlan; ++it) {
          const int jj = 32 * it + lane;
          const int n = jj < nchunks ? jj / cpr : 0;
          const int b = __shfl_sync(0xffffffffu, my_b[k], n);
          const int kc = jj - n * cpr;
          ch_src[k][it] = stage[k] + (uint32_t)(n * S::kOutPitch + kc * cb);
          ch_dst[k][it] = (jj < nchunks && b >= 0 && bc_ok(st, b < p.B, 10)) ? (long long)b * row_bytes + kc * cb : -1;
        }
      }
      bool ok = true;
      for (int t = 1; ok && t <= Tmax; ++t) {
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          if (t > Tts[k]) continue;
          const int sl = sls[k];
          if (!wait_phase(bar(sl, S::kLin, lin_buf(t)), lin_phase(t), abort_flag, p.timeout_ns)) {
            if (lane == 0 && !*abort_flag) raise_abort(p, sm + S::kAbort, ncta, t);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          uint32_t r[NL / 8][8];
#pragma unroll
          for (int c = 0; c < NL / 8; ++c) ptx::tmem_ld_32x32b_x8(dlin_at(sl, t) + qlane + (uint32_t)(8 * c), r[c]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < NL / 8; ++c) reg_after_wait<8>(r[c]);
          ptx::tc_fence_before();
          __syncwarp();
          // Relaxed: a release arrive would first wait for the previous step's output stores.
          if (lane == 0) ptx::mbar_arrive_relaxed(bar(sl, S::kLinFree, lin_buf(t)));
          const uint32_t live = __ballot_sync(0xffffffffu, t - 1 < my_len[k]);  // bit n: row n not finished
          // Two rows rounded to 16 bits per instruction (the single-value conversion issues on
          // the pipe the gate math's tanh runs on, and this warp shares schedulers with it).
#pragma unroll
          for (int c = 0; c < NL / 8; ++c)
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              float v[2];
#pragma unroll
              for (int e = 0; e < 2; ++e)
                v[e] = (live >> (8 * c + i + e)) & 1u ? __uint_as_float(r[c][i + e]) + blin_o : 0.0f;
              const uint32_t bits = pack2_bits<BF16>(v[0], v[1]);
              if (o < p.O) {
                const uint32_t row = stage[k] + (uint32_t)((8 * c + i) * S::kOutPitch + 2 * o);
                ptx::st_shared_u16(row, (uint16_t)(bits & 0xffffu));
                ptx::st_shared_u16(row + S::kOutPitch, (uint16_t)(bits >> 16));
              }
            }
          __syncwarp();
          uint8_t* const out_t = reinterpret_cast<uint8_t*>(p.out) + (size_t)(t - 1) * p.O * 2;
#pragma unroll
          for (int it = 0; it < kPlan; ++it)
            if (ch_dst[k][it] >= 0) copy_chunk(ch_src[k][it], out_t + ch_dst[k][it]);
          for (int j0 = 32 * kPlan; j0 < nchunks; j0 += 32) {  // wide plans only (cb < 16)
            const int jj = j0 + lane;
            const int n = jj < nchunks ? jj / cpr : 0, kc = jj - n * cpr;
            const int b = __shfl_sync(0xffffffffu, my_b[k], n);
            if (jj < nchunks && b >= 0 && bc_ok(st, b < p.B, 10))
              copy_chunk(stage[k] + (uint32_t)(n * S::kOutPitch + kc * cb), out_t + (size_t)b * row_bytes + kc * cb);
          }
          __syncwarp();  // the stage is rewritten next step
        }
      }
      // Outputs past each slot's last step are zero.
      if (ok && !*abort_flag) {
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          if (!owns[k]) continue;
          for (int i = 0; i < NL; ++i) {
            const int b = __shfl_sync(0xffffffffu, my_b[k], i);
            if (o < p.O && b >= 0 && bc_ok(st, b < p.B, 10))
              for (int ts = Tts[k]; ts < p.T; ++ts) out16[((size_t)b * p.T + ts) * p.O + o] = 0;
          }
        }
      }
    }
  } else if (warp >= kComputeWarps) {
    // ============================ control warps ==========================
    const int sl = warp - kComputeWarps;
    const bool does_linear = does_lin(sl);
    bool active = false;
    const int Tt = slot_len(sl, &active);
    // A slot's layer-0 x tile: NH rows x kx, no swizzle (fits the slot's two input K blocks).
    const uint32_t xbytes = (uint32_t)(NH * p.kx * 2), bkb = S::kBKB;
    const uint32_t in_bytes = (l == 0) ? xbytes : 2 * bkb;
    // Layer 0 whose x tiles the x warp writes: FullIn completes on that warp's arrival
    // (no transaction bytes to expect, nothing to copy).
    const bool x_by_warp = l == 0 && p.xp == nullptr;
    constexpr uint32_t idesc_g = ptx::idesc_f16(128, NH, BF16);
    constexpr uint32_t idesc_l = ptx::idesc_f16(128, NL, BF16);
    const uint16_t up_mask = l > 0 ? (uint16_t)(3u << (2 * (l - 1))) : 0;
    const uint32_t a_rec0 = l == 0 ? (uint32_t)(p.kx / 2) : 64u;  // A columns of W_hh within a tile
    const uint64_t dAl = ptx::desc_k_sw128(sbase + S::kALin);
    const uint64_t dB0 = ptx::desc_k_sw128(bbuf(sl, 0));
    // x: K groups 128 bytes apart, 8-row groups kx * 16 bytes apart.
    const uint64_t dBx0 = ptx::desc_k_none(bbuf(sl, 0), 128, (uint32_t)(p.kx * 16));
    constexpr uint64_t kBufStep = (uint64_t)(S::kBufBytes >> 4);
    const uint32_t lin_row_off = S::kSplitLinear ? (uint32_t)(s * NL) * 128u : 0u;
    const int steps = Tt + (does_linear ? 1 : 0);
    int last_commit = -1, last_lin = -1;
    bool ok = true;
    const bool tracer = sl == p.trace_slot;

    auto x_src = [&](int t) { return p.xp + (((size_t)tile * p.T + t) * N + (size_t)sl * NH) * (size_t)(p.kx * 2); };
    // The repacked x ends at n_tiles * T * N * kx * 2 bytes.
    auto x_in = [&](int t) {
      return bc_ok(st, (((size_t)tile * p.T + t) * N + (size_t)sl * NH) * (size_t)(p.kx * 2) + xbytes <=
                           n_tiles * p.T * N * (size_t)(p.kx * 2) && xbytes <= 2 * bkb, 11);
    };
    auto issue_in = [&](int t) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = dB0 + kBufStep * b;
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const uint32_t a = tmem + (uint32_t)(tau * 128);
          if (l == 0) {
            ptx::mma_f16_ts(dcol(sl, tau), a, dBx0 + kBufStep * b, idesc_g, 0u);
            for (int kk = 1; kk < p.kx / 16; ++kk)  // inputs wider than 16
              ptx::mma_f16_ts(dcol(sl, tau), a + (uint32_t)(8 * kk), dBx0 + kBufStep * b + (uint64_t)((kk * 256) >> 4),
                              idesc_g, 1u);
          } else {
#pragma unroll
            for (int kb = 0; kb < 2; ++kb)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                ptx::mma_f16_ts(dcol(sl, tau), a + (uint32_t)(32 * kb + 8 * kk),
                                dB + (uint64_t)((kb * S::kBKB + kk * 32) >> 4), idesc_g, (kb | kk) != 0 ? 1u : 0u);
          }
        }
        // Layer l-1 may overwrite this input slot once these MMAs are done.
        if (l > 0 && t + 2 < Tt) ptx::mma_commit_mc(bar(sl, S::kEmpty, b), up_mask);
      }
      __syncwarp();
    };
    auto issue_rec_half = [&](int t, int kb) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = dB0 + kBufStep * b;
#pragma unroll
        for (int tau = 0; tau < 2; ++tau)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            ptx::mma_f16_ts(dcol(sl, tau), tmem + (uint32_t)(tau * 128) + a_rec0 + (uint32_t)(32 * kb + 8 * kk),
                            dB + (uint64_t)(((2 + kb) * S::kBKB + kk * 32) >> 4), idesc_g, 1u);
      }
      __syncwarp();
    };
    // Commits the step's gate MMAs.
    auto commit_gates = [&](int t) {
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        ptx::mma_commit(bar(sl, S::kMma, t & 1));
      }
      __syncwarp();
    };
    // Issues and commits the Linear MMAs on h_{t-1} (behind the gate MMAs in the tensor pipe,
    // tracked by their own barrier).
    auto issue_linear = [&](int t) {
      const int b = t & 1;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = dB0 + kBufStep * b;
        const uint32_t dlin = dlin_at(sl, t);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            ptx::mma_f16_ss(dlin, dAl + (uint64_t)((kb * kATileKB + kk * 32) >> 4),
                            dB + (uint64_t)(((2 + kb) * S::kBKB + lin_row_off + kk * 32) >> 4), idesc_l,
                            (kb | kk) != 0 ? 1u : 0u);
        ptx::mma_commit(bar(sl, S::kLin, lin_buf(t)));
      }
      __syncwarp();
    };
    auto fail = [&](int t) {
      if (ptx::elect_one()) raise_abort(p, sm + S::kAbort, ncta, t);
      __syncwarp();
      ok = false;
    };
    // Layer 0: streams x of step t+2 into the input slot step t has finished with
    // (h(t) itself is pushed by the slot's last compute warp to finish the step).
    auto hand_off = [&](int t) {
      const int b = t & 1;
      if (l == 0 && !x_by_warp && t + 2 < Tt && x_in(t + 2) && ptx::elect_one())
        ptx::bulk_g2s(bbuf(sl, b), x_src(t + 2), xbytes, bar(sl, S::kFullIn, b));
      __syncwarp();
    };

    if (active) {
      // Prologue: expected bytes of steps 0 / 1 (inputs) and 1 / 2 (sibling h), x of steps 0 / 1.
      if (ptx::elect_one()) {
        for (int t = 0; t < 2 && t < Tt && !x_by_warp; ++t) {
          ptx::mbar_arrive_expect_tx(bar(sl, S::kFullIn, t), in_bytes);
          if (l == 0 && x_in(t)) ptx::bulk_g2s(bbuf(sl, t), x_src(t), xbytes, bar(sl, S::kFullIn, t));
        }
        for (int t = 1; t <= 2; ++t)
          if (t < Tt || (does_linear && t == Tt)) ptx::mbar_arrive_expect_tx(bar(sl, S::kFullRec, t & 1), bkb);
      }
      __syncwarp();
      if (Tt > 0) {
        if (!warp_wait_phase(bar(sl, S::kFullIn, 0), 0, abort_flag, p.timeout_ns)) {
          fail(0);
        } else {
          issue_in(0);
          if (2 < Tt && !x_by_warp && ptx::elect_one()) ptx::mbar_arrive_expect_tx(bar(sl, S::kFullIn, 0), in_bytes);
          __syncwarp();
        }
      }
      for (int t = 0; ok && t < steps; ++t) {
        const int b = t & 1;
        const bool gates = t < Tt;
        const bool lin = does_linear && (MODE == kModeSeq ? t >= 1 : t == Tt);
        if (gates) issue_rec_half(t, s);  // own half of h_{t-1}: written before the previous step ended
        if (tracer && lane == 0) trace_mark(p, rank, t, 3);
        if (t >= 1) {
          if (!warp_wait_phase(bar(sl, S::kFullRec, b), ((t - 1) >> 1) & 1, abort_flag, p.timeout_ns)) {
            fail(t);
            break;
          }
          if ((t + 2 < Tt || (does_linear && t + 2 == Tt)) && ptx::elect_one())
            ptx::mbar_arrive_expect_tx(bar(sl, S::kFullRec, b), bkb);
          __syncwarp();
        }
        if (tracer && lane == 0) trace_mark(p, rank, t, 0);
        if (gates) issue_rec_half(t, 1 - s);
        commit_gates(t);
        last_commit = t;
        // The output warp must have read the Linear accumulator buffer this step reuses (the gate
        // MMAs are committed first, so that the compute warps never wait for the output warp).
        if (MODE == kModeSeq && lin && t >= 3 &&
            !warp_wait_phase(bar(sl, S::kLinFree, lin_buf(t)), (uint32_t)((t - 3) >> 1) & 1u, abort_flag,
                             p.timeout_ns)) {
          fail(t);
          break;
        }
        if (lin) issue_linear(t);
        if (lin) last_lin = t;
        if (tracer && lane == 0) trace_mark(p, rank, t, 1);
        if (!gates) break;  // drain step issued
        // This step's h hand-off, and the next step's input MMAs once the compute
        // warps have loaded this step's accumulator and the input has landed (the
        // hand-off first when both are ready).
        bool in_pending = t + 1 < Tt, copy_pending = true;
        const unsigned long long t0 = ptx::globaltimer();
        unsigned spins = 0;
        while (in_pending || copy_pending) {
          if (copy_pending && warp_test_wait(bar(sl, S::kHReady, b), (t >> 1) & 1)) {
            if (tracer && lane == 0) trace_mark(p, rank, t, 2);
            hand_off(t);
            copy_pending = false;
            continue;
          }
          if (in_pending && warp_test_wait(bar(sl, S::kDFree, b), (t >> 1) & 1) &&
              warp_test_wait(bar(sl, S::kFullIn, b ^ 1), ((t + 1) >> 1) & 1)) {
            issue_in(t + 1);
            if (t + 3 < Tt && !x_by_warp && ptx::elect_one())
              ptx::mbar_arrive_expect_tx(bar(sl, S::kFullIn, b ^ 1), in_bytes);
            __syncwarp();
            in_pending = false;
            continue;
          }
          if ((++spins & 31) == 0) {  // abort / timeout checks are slow: every 32 polls
            int bad = 0;
            if (lane == 0) bad = (*abort_flag != 0) || (ptx::globaltimer() - t0 > p.timeout_ns);
            if (__shfl_sync(0xffffffffu, bad, 0)) {
              fail(t);
              break;
            }
          }
        }
      }
      // All MMAs must have completed before TMEM is released.
      if (last_commit >= 0 && lane == 0)
        wait_phase(bar(sl, S::kMma, last_commit & 1), (last_commit >> 1) & 1, abort_flag, p.timeout_ns);
      if (last_lin >= 0 && lane == 0)
        wait_phase(bar(sl, S::kLin, lin_buf(last_lin)), lin_phase(last_lin), abort_flag, p.timeout_ns);
      __syncwarp();
    }
  } else {
    // =========================== compute warps ===========================
    const int sl = warp >> 2, q = warp & 3;
    const bool does_linear = does_lin(sl), sibling_linear = sibling_lin(sl);
    bool active = false, other_active = false;
    const int Tt = slot_len(sl, &active);
    // The slot whose gate math precedes this one's on the MUFU pipes: the nearest active slot
    // before it in the ring.  Skipping inactive slots keeps the ring closed, which bounds how far
    // one slot can run ahead of the next: with an open ring (slot 2 of a partial tile empty) slot
    // 0 could finish step t + 2 before slot 1 polled the parity of step t, and that poll would
    // then wait for step t + 4.  (Rings that open when a slot finishes early are why three-slot
    // tiles take uniform lengths only.)
    int prev_sl = sl;
    for (int k = 1; k < NSL; ++k) {
      const int c = (sl + NSL - k) % NSL;
      bool a = false;
      slot_len(c, &a);
      if (a) {
        prev_sl = c;
        break;
      }
    }
    const int T_other = prev_sl != sl ? slot_len(prev_sl, &other_active) : 0;
    const int j8 = lane >> 2;          // unit within the quadrant's group of 8
    const int cpair = (lane & 3) * 2;  // first of the two batch columns in a chunk
    const bool tracer = sl == p.trace_slot;
    // cells: [tau][chunk jc][e]; column within the slot nn = 8 jc + cpair + e
    float c_st[2][CPW][2];
    uint16_t h_st[2][CPW][2];  // h bits (the frozen value of finished rows)
    int len_c[CPW][2], bidx[CPW][2];
#pragma unroll
    for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = sl * NH + 8 * jc + cpair + e;
        len_c[jc][e] = lens_s[n];
        bidx[jc][e] = perm_s[n];
      }
#pragma unroll
    for (int tau = 0; tau < 2; ++tau) {
      const int u = 64 * s + 8 * (4 * tau + q) + j8;
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int b = bidx[jc][e];
          uint16_t hv = 0;
          float cv = 0.0f;
          if (b >= 0 && p.h0 != nullptr && u < p.hid && bc_ok(st, ((size_t)l * p.B + b) * p.hid + u < state_elems, 12)) {
            hv = static_cast<const uint16_t*>(p.h0)[((size_t)l * p.B + b) * p.hid + u];
            cv = from_bits<BF16>(static_cast<const uint16_t*>(p.c0)[((size_t)l * p.B + b) * p.hid + u]);
          }
          h_st[tau][jc][e] = hv;
          c_st[tau][jc][e] = cv;
        }
    }
    // f32 gate bias of this thread's two units (i, f, o rows pre-scaled by 1/2 like the
    // weights), added to the accumulators in registers.
    float bz[2][4];
    {
      const float* bias_img = reinterpret_cast<const float*>(p.packed + packed_bias_off(p.L)) + rank * 256;
#pragma unroll
      for (int tau = 0; tau < 2; ++tau)
#pragma unroll
        for (int g = 0; g < 4; ++g)
          bz[tau][g] = bc_ok(st, rank * 256 + tau * 128 + 32 * q + 8 * g + j8 < ncta * 256, 13)
                           ? bias_img[tau * 128 + 32 * q + 8 * g + j8] : 0.0f;
    }
    const float* blin = reinterpret_cast<const float*>(p.packed + packed_blin_off(p.L));
    const bool lin_warp = does_linear && q == 0;
    const int o = lane;  // Linear output row handled by this lane (lin_warp only)
    const float blin_o = (lin_warp && o < p.O) ? blin[o] : 0.0f;
    uint16_t* out16 = static_cast<uint16_t*>(p.out);
    const int lin_n0 = sl * NH + (S::kSplitLinear ? s * NL : 0);  // first tile row of this CTA's Linear columns

    // The Linear accumulator of the MMAs issued at step t (lanes = output rows,
    // registers = tile columns), once their commit has completed.
    auto load_linear = [&](int t, auto& r) -> bool {
      if (!wait_phase(bar(sl, S::kLin, lin_buf(t)), lin_phase(t), abort_flag, p.timeout_ns)) return false;
      ptx::tc_fence_after();
      const uint32_t dlin = dlin_at(sl, t);
#pragma unroll
      for (int c = 0; c < NL / 8; ++c) ptx::tmem_ld_32x32b_x8(dlin + (uint32_t)(8 * c), r[c]);
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      return true;
    };
    // Stores the [B][O] result.
    auto write_last = [&](const auto& r) {
      if (o >= p.O) return;
#pragma unroll
      for (int c = 0; c < NL / 8; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int b = perm_s[lin_n0 + 8 * c + i];
          if (b >= 0 && bc_ok(st, b < p.B, 14)) out16[(size_t)b * p.O + o] = to_bits<BF16>(__uint_as_float(r[c][i]) + blin_o);
        }
    };

    if (active) {
      for (int t = 0; t < Tt; ++t) {
        const int b = t & 1;
        if (*abort_flag) break;
        if (!wait_phase(bar(sl, S::kMma, b), (t >> 1) & 1, abort_flag, p.timeout_ns)) {
          if (lane == 0) raise_abort(p, sm + S::kAbort, ncta, t);
          break;
        }
        ptx::tc_fence_after();
        if (tracer && q == 0 && lane == 0) trace_mark(p, rank, t, 4);
        uint32_t rif[2][4 * CPW], rgo[2][4 * CPW];
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const uint32_t col = dcol(sl, tau);
          tmem_ld_chunks<CPW>(col + ((uint32_t)(32 * q) << 16), rif[tau]);
          tmem_ld_chunks<CPW>(col + ((uint32_t)(32 * q + 16) << 16), rgo[tau]);
        }
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        // The accumulator may now be re-initialised by the next step's input MMAs.
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(sl, S::kDFree, b));
        if (tracer && q == 0 && lane == 0) trace_mark(p, rank, t, 5);

        // Layer l+1 must have consumed h_{t-2} (same buffer and copy source) before it is overwritten.
        if (l + 1 < p.L && t >= 2) {
          if (!wait_phase(bar(sl, S::kEmpty, b), ((t - 2) >> 1) & 1, abort_flag, p.timeout_ns)) {
            if (lane == 0) raise_abort(p, sm + S::kAbort, ncta, t);
            break;
          }
        }
        // The slots take turns on the MUFU pipes: a slot runs its gate math after that of
        // the preceding active slot's same step (its previous step if that slot comes later
        // in the ring, i.e. for the first active slot), so that one slot's MMA / hand-off
        // latency overlaps the others' gate math.
        {
          const int tt = prev_sl < sl ? t : t - 1;
          if (other_active && tt >= 0 && tt < T_other &&
              !wait_phase(bar(prev_sl, S::kHReady, tt & 1), (tt >> 1) & 1, abort_flag, p.timeout_ns)) {
            if (lane == 0) raise_abort(p, sm + S::kAbort, ncta, t);
            break;
          }
        }
        uint16_t hw[2][CPW][2];
        lstm_cells<CPW, BF16, VARLEN>(rif, rgo, bz, c_st, h_st, len_c, t, hw);
        uint8_t* dst = sm + S::kB + sl * S::kSlotBytes + (b ^ 1) * S::kBufBytes + (2 + s) * S::kBKB;
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const int ul = 8 * (4 * tau + q) + j8;  // unit within this CTA's 64
#pragma unroll
          for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
            for (int e = 0; e < 2; ++e)
              if (bc_ok(st, (uint32_t)(dst - sm) + sw128_off(8 * jc + cpair + e, ul) + 2 <= (uint32_t)S::kALin, 15))
                *reinterpret_cast<uint16_t*>(dst + sw128_off(8 * jc + cpair + e, ul)) = hw[tau][jc][e];
        }
        ptx::fence_proxy_async_smem();
        if (tracer && q == 0 && lane == 0) trace_mark(p, rank, t, 6);
        if (tracer && q == 3 && lane == 0) trace_mark(p, rank, t, 7);
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive(bar(sl, S::kHReady, b));  // the control warp: own half of the next step's MMAs
          // The slot's last warp to finish pushes the tile (acquire-release counter: the
          // other warps' writes, fenced for the async proxy, are ordered before its copies).
          if (ptx::atom_add_acq_rel_smem(sbase + S::kDone + 4 * sl, 1u) % 4u == 3u) {
            const bool to_sibling = ((t + 1 < Tt) || (sibling_linear && t + 1 == Tt)) &&
                                    !(sl == 0 && rank == p.drop_rank && t == p.drop_step);
            // This step's Linear MMAs read h_{t-1} from the buffer the sibling refills with
            // h_{t+1} once it has h_t: they must be done before h_t leaves.  (The output
            // warp has usually long since seen this commit.)
            if (MODE == kModeSeq && does_linear && t >= 1 &&
                !wait_phase(bar(sl, S::kLin, lin_buf(t)), lin_phase(t), abort_flag, p.timeout_ns)) {
              raise_abort(p, sm + S::kAbort, ncta, t);
            } else if (bc_ok(st, (uint32_t)(b ^ 1) * S::kBufBytes + sl * S::kSlotBytes + (3 + s) * S::kBKB <=
                                     (uint32_t)S::kALin, 20)) {
              push_h(bbuf(sl, b ^ 1) + (uint32_t)((2 + s) * S::kBKB), S::kBKB, rank, to_sibling,
                     bar(sl, S::kFullRec, b ^ 1), l + 1 < p.L, 2 * (l + 1), bbuf(sl, b) + (uint32_t)(s * S::kBKB),
                     bar(sl, S::kFullIn, b));
            }
          }
        }
        // The h sequence output, after the step's arrivals: an arrive has release
        // semantics and would wait for global stores issued before it to complete.
        if (MODE == kModeHSeq && last_layer) {
#pragma unroll
          for (int tau = 0; tau < 2; ++tau) {
            const int ul = 8 * (4 * tau + q) + j8;
#pragma unroll
            for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
              for (int e = 0; e < 2; ++e)
                if (bidx[jc][e] >= 0 && 64 * s + ul < p.hid && bc_ok(st, bidx[jc][e] < p.B, 16))
                  out16[((size_t)bidx[jc][e] * p.T + t) * p.hid + 64 * s + ul] =
                      (!VARLEN || t < len_c[jc][e]) ? hw[tau][jc][e] : (uint16_t)0;
          }
        }
      }
      // [B][O] mode: the Linear of the last step's h (issued at step Tt).
      if (MODE == kModeLast && lin_warp && !*abort_flag) {
        uint32_t r[NL / 8][8];
        if (load_linear(Tt, r))
          write_last(r);
        else if (lane == 0)
          raise_abort(p, sm + S::kAbort, ncta, Tt);
      }
      if (MODE == kModeHSeq && last_layer) {
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const int u = 64 * s + 8 * (4 * tau + q) + j8;
#pragma unroll
          for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int bb = bidx[jc][e];
              if (bb < 0 || u >= p.hid || !bc_ok(st, bb < p.B, 16)) continue;
              for (int ts = Tt; ts < p.T; ++ts) out16[((size_t)bb * p.T + ts) * p.hid + u] = 0;
            }
        }
      }
      // Final state.
#pragma unroll
      for (int tau = 0; tau < 2; ++tau) {
        const int u = 64 * s + 8 * (4 * tau + q) + j8;
#pragma unroll
        for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int bb = bidx[jc][e];
            if (bb < 0 || u >= p.hid) continue;
            const size_t idx = ((size_t)l * p.B + bb) * p.hid + u;
            if (!bc_ok(st, idx < state_elems, 17)) continue;
            if (p.h_n != nullptr) static_cast<uint16_t*>(p.h_n)[idx] = h_st[tau][jc][e];
            if (p.c_n != nullptr) {
              if (p.flags & PLSTM_FLAG_CN_F32)
                static_cast<float*>(p.c_n)[idx] = c_st[tau][jc][e];
              else
                static_cast<uint16_t*>(p.c_n)[idx] = to_bits<BF16>(c_st[tau][jc][e]);
            }
          }
      }
    }
  }

  // ---- teardown -----------------------------------------------------------------
  if (*abort_flag) {
    // Let bulk copies already in flight toward peers land before any CTA leaves.
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

// ---- packing ----------------------------------------------------------------------
// Writes the per-CTA A images, the Linear A image, the permuted bias and b_lin.
struct PackArgs {
  const void* w_ih[kMaxLayers];
  const void* w_hh[kMaxLayers];
  const void* b_ih[kMaxLayers];
  const void* b_hh[kMaxLayers];
  const void* w_lin;
  const void* b_lin;
  int ih_layout, hh_layout, dtype, L, I, O;
  int kx;   // padded layer-0 input width: A columns [0, kx) hold W_ih, [kx, kx + 128) W_hh
  int hid;  // the model's hidden size (<= 128; the rest of the 128 units is zero padding)
};

// Gate rows i, f, o are stored pre-scaled by 1/2 (exact in f16 / bf16 up to
// subnormals) so that the kernel's sigmoid(z) = (1 + tanh(z / 2)) / 2 needs no multiply.
__device__ __forceinline__ float gate_scale(int r) { return ((r & 31) >> 3) == 2 ? 1.0f : 0.5f; }

// PyTorch gate row (of a model with hidden size hid) of row r of tile tau of CTA half s,
// or -1 for a padding unit (unit >= hid).
__device__ __forceinline__ int gate_row(int s, int tau, int r, int hid) {
  const int q = r >> 5, rr = r & 31, gate = rr >> 3, j = rr & 7;
  const int unit = 64 * s + 8 * (4 * tau + q) + j;
  return unit < hid ? gate * hid + unit : -1;
}

__global__ void tc_pack_kernel(const PackArgs a, uint8_t* packed) {
  const int ncta = 2 * a.L;
  const int64_t n_a = (int64_t)ncta * (kABytes / 2);
  const int64_t n_lin = kALinBytes / 2;
  const int64_t n_bias = (int64_t)ncta * 256;
  const int64_t total = n_a + n_lin + n_bias + 32;
  uint16_t* img = reinterpret_cast<uint16_t*>(packed);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n_a) {
      // A image: [tile][row][K] 16-bit, K-major rows of 256 (see the TMEM column map).
      const int rank = (int)(i / (kABytes / 2));
      const int within = (int)(i % (kABytes / 2));
      const int tau = within / (128 * kAK), r = (within / kAK) % 128, k = within % kAK;
      const int l = rank >> 1, s = rank & 1;
      const int row = gate_row(s, tau, r, a.hid);
      const int G = 4 * a.hid;
      float v = 0.0f;
      if (row < 0) {
      } else if (l == 0) {
        if (k < a.kx) {
          if (k < a.I) v = load_any(a.w_ih[0], a.dtype, weight_src_index(a.ih_layout, G, a.I, row, k));
        } else if (k - a.kx < a.hid) {
          v = load_any(a.w_hh[0], a.dtype, weight_src_index(a.hh_layout, G, a.hid, row, k - a.kx));
        }
      } else if (k < kH) {
        if (k < a.hid) v = load_any(a.w_ih[l], a.dtype, weight_src_index(a.ih_layout, G, a.hid, row, k));
      } else if (k - kH < a.hid) {
        v = load_any(a.w_hh[l], a.dtype, weight_src_index(a.hh_layout, G, a.hid, row, k - kH));
      }
      v *= gate_scale(r);
      img[i] = a.dtype == PLSTM_BF16 ? to_bits<true>(v) : to_bits<false>(v);
    } else if (i < n_a + n_lin) {
      const int off = (int)(i - n_a) * 2;
      const int kb = off / kATileKB, within = off % kATileKB;
      const int r = within / 128, chunk = (within % 128) >> 4, e = (within & 15) >> 1;
      const int kk = ((chunk ^ (r & 7)) << 3) + e;
      float v = 0.0f;
      if (r < a.O && a.w_lin != nullptr && kb * 64 + kk < a.hid)
        v = load_any(a.w_lin, a.dtype, (int64_t)r * a.hid + kb * 64 + kk);
      img[i] = a.dtype == PLSTM_BF16 ? to_bits<true>(v) : to_bits<false>(v);
    } else if (i < n_a + n_lin + n_bias) {
      const int64_t j = i - n_a - n_lin;
      const int rank = (int)(j / 256), rr = (int)(j % 256);
      const int l = rank >> 1, s = rank & 1;
      const int row = gate_row(s, rr >> 7, rr & 127, a.hid);
      float v = 0.0f;
      if (row >= 0 && a.b_ih[l] != nullptr) v += load_any(a.b_ih[l], a.dtype, row);
      if (row >= 0 && a.b_hh[l] != nullptr) v += load_any(a.b_hh[l], a.dtype, row);
      reinterpret_cast<float*>(packed + packed_bias_off(a.L))[j] = v * gate_scale(rr & 127);
    } else {
      const int o = (int)(i - n_a - n_lin - n_bias);
      float v = 0.0f;
      if (o < a.O && a.b_lin != nullptr) v = load_any(a.b_lin, a.dtype, o);
      reinterpret_cast<float*>(packed + packed_blin_off(a.L))[o] = v;
    }
  }
}

// ---- per-call preparation -----------------------------------------------------------
// Uniform lengths: tile rows are consecutive batch rows.
__global__ void tc_perm_uniform_kernel(int32_t* perm, int32_t* tile_len, int B, int T, int N, int tiles) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < tiles * N; i += gridDim.x * blockDim.x) {
    perm[i] = i < B ? i : -1;
    if (i < tiles) tile_len[i] = T;
  }
}
// Variable lengths: counting sort by length, longest first.
__global__ void tc_len_hist_kernel(const int32_t* lengths, int B, int T, int32_t* hist) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) {
    const int len = min(max(lengths[b], 0), T);
    atomicAdd(&hist[T - len], 1);
  }
}
__global__ void tc_len_scan_kernel(int32_t* hist, int nbins) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < nbins; ++i) {
      const int v = hist[i];
      hist[i] = acc;
      acc += v;
    }
  }
}
__global__ void tc_len_scatter_kernel(const int32_t* lengths, int B, int T, int32_t* offs, int32_t* sorted) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) {
    const int len = min(max(lengths[b], 0), T);
    sorted[atomicAdd(&offs[T - len], 1)] = b;
  }
}
__global__ void tc_perm_varlen_kernel(const int32_t* sorted, const int32_t* lengths, int32_t* perm,
                                      int32_t* tile_len, int B, int T, int N, int tiles) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < tiles * N; i += gridDim.x * blockDim.x) {
    perm[i] = i < B ? sorted[i] : -1;
    if (i < tiles) tile_len[i] = min(max(lengths[sorted[i * N]], 0), T);
  }
}

// Device-side choice between 32- and 64-row two-slot tiles for a length-sorted batch.
// len32 holds the 32-row tiles' lengths (longest first); the 64-row tile j is 32-row tiles
// 2j and 2j+1, so its length is len32[2j].  Each height's launch is list-scheduled in tile
// order onto its m co-resident clusters (a tile holds a cluster for len + L wavefront
// steps); 32-row tiles step kStep32 times as long as 64-row ones (measured 1.476 / 1.86 ms
// at 480 / 512 rows).  Writes len64 and *choice = 32 or 64.
constexpr float kStep32 = 0.8f;
constexpr int kMaxChoiceClusters = 16;
__global__ void tc_tile_choice_kernel(const int32_t* __restrict__ len32, int tiles32, int tiles64, int L, int m32,
                                      int m64, int32_t* __restrict__ len64, int* __restrict__ choice) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  float end[2][kMaxChoiceClusters];
  const int m[2] = {min(m32, kMaxChoiceClusters), min(m64, kMaxChoiceClusters)};
  for (int h = 0; h < 2; ++h)
    for (int c = 0; c < kMaxChoiceClusters; ++c) end[h][c] = 0.0f;
  float span[2] = {0.0f, 0.0f};
  for (int h = 0; h < 2; ++h) {
    const int tiles = h == 0 ? tiles32 : tiles64;
    const float step = h == 0 ? kStep32 : 1.0f;
    for (int j = 0; j < tiles; ++j) {
      const int len = h == 0 ? len32[j] : len32[2 * j];
      if (h == 1) len64[j] = len;
      int c = 0;
      for (int k = 1; k < m[h]; ++k)
        if (end[h][k] < end[h][c]) c = k;
      end[h][c] += step * (float)(len + L);
      span[h] = fmaxf(span[h], end[h][c]);
    }
  }
  *choice = span[0] < span[1] ? 32 : 64;
}
// x[B][T][I] -> per-tile, per-step K-major no-swizzle tiles of kx columns: 8-row x
// 8-column core matrices of 128 bytes, K groups 128 bytes apart, 8-row groups kx * 16
// bytes apart.  One thread per (tile, step, row, K group).
template <typename T16>
__global__ void tc_xpack_kernel(const T16* __restrict__ x, const int32_t* __restrict__ perm,
                                uint8_t* __restrict__ xp, int B, int T, int I, int N, int tiles, int kx,
                                const int* choice) {
  if (choice != nullptr && *choice != N) return;  // packs for the chosen tile height only
  const int kg_n = kx / 8;
  const int64_t total = (int64_t)tiles * T * N * kg_n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int kg = (int)(i % kg_n);
    const int64_t r = i / kg_n;
    const int n = (int)(r % N);
    const int64_t tt = r / N;
    const int t = (int)(tt % T);
    const int tile = (int)(tt / T);
    const int b = perm[tile * N + n];
    uint16_t v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = 0;
    if (b >= 0) {
      const uint16_t* src = reinterpret_cast<const uint16_t*>(x) + ((size_t)b * T + t) * I;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (8 * kg + k < I) v[k] = src[8 * kg + k];
    }
    uint8_t* dst = xp + (size_t)tt * N * kx * 2 + (size_t)(n >> 3) * kx * 16 + kg * 128 + (n & 7) * 16;
    uint4 q;
    q.x = v[0] | (v[1] << 16); q.y = v[2] | (v[3] << 16); q.z = v[4] | (v[5] << 16); q.w = v[6] | (v[7] << 16);
    *reinterpret_cast<uint4*>(dst) = q;
  }
}

// ---- host side ----------------------------------------------------------------------
// slots = 1: wavefront_kernel with N-row tiles; slots = 2: wavefront2_kernel with
// two slots of N / 2 rows per tile.
struct Plan {
  int N, tiles, slots;
};

template <int N, bool BF16, bool VARLEN, int MODE>
void* kernel_ptr() {
  return reinterpret_cast<void*>(&wavefront_kernel<N, BF16, VARLEN, MODE>);
}

template <int N>
void* pick_kernel(bool bf16, bool varlen, int mode) {
#define PLSTM_TC_K(B, V, M) \
  if (bf16 == B && varlen == V && mode == M) return kernel_ptr<N, B, V, M>();
  PLSTM_TC_K(false, false, kModeSeq) PLSTM_TC_K(false, false, kModeLast) PLSTM_TC_K(false, false, kModeHSeq)
  PLSTM_TC_K(false, true, kModeSeq) PLSTM_TC_K(false, true, kModeLast) PLSTM_TC_K(false, true, kModeHSeq)
  PLSTM_TC_K(true, false, kModeSeq) PLSTM_TC_K(true, false, kModeLast) PLSTM_TC_K(true, false, kModeHSeq)
  PLSTM_TC_K(true, true, kModeSeq) PLSTM_TC_K(true, true, kModeLast) PLSTM_TC_K(true, true, kModeHSeq)
#undef PLSTM_TC_K
  return nullptr;
}

int mode_of(const Problem& p) {
  if (!p.has_linear()) return kModeHSeq;
  return p.out_seq() ? kModeSeq : kModeLast;
}

int smem_bytes_for(int N) {
  switch (N) {
    case 16: return Smem<16>::kDynBytes;
    case 32: return Smem<32>::kDynBytes;
    default: return Smem<48>::kDynBytes;
  }
}

void* pick_kernel_n(int N, bool bf16, bool varlen, int mode) {
  switch (N) {
    case 16: return pick_kernel<16>(bf16, varlen, mode);
    case 32: return pick_kernel<32>(bf16, varlen, mode);
    default: return pick_kernel<48>(bf16, varlen, mode);
  }
}

constexpr int kTileNs[3] = {16, 32, 48};

int threads_for(int N) {
  switch (N) {
    case 16: return Smem<16>::kThreads;
    case 32: return Smem<32>::kThreads;
    default: return Smem<48>::kThreads;
  }
}

template <int NH, int NSL, bool BF16, bool VARLEN, int MODE>
void* kernel2_ptr() {
  return reinterpret_cast<void*>(&wavefront2_kernel<NH, NSL, BF16, VARLEN, MODE>);
}
template <int NH, int NSL>
void* pick_kernel2(bool bf16, bool varlen, int mode) {
#define PLSTM_TC_K(B, V, M) \
  if (bf16 == B && varlen == V && mode == M) return kernel2_ptr<NH, NSL, B, V, M>();
  PLSTM_TC_K(false, false, kModeSeq) PLSTM_TC_K(false, false, kModeLast) PLSTM_TC_K(false, false, kModeHSeq)
  PLSTM_TC_K(false, true, kModeSeq) PLSTM_TC_K(false, true, kModeLast) PLSTM_TC_K(false, true, kModeHSeq)
  PLSTM_TC_K(true, false, kModeSeq) PLSTM_TC_K(true, false, kModeLast) PLSTM_TC_K(true, false, kModeHSeq)
  PLSTM_TC_K(true, true, kModeSeq) PLSTM_TC_K(true, true, kModeLast) PLSTM_TC_K(true, true, kModeHSeq)
#undef PLSTM_TC_K
  return nullptr;
}
// Kernel, dynamic shared memory and block size of a plan's launch.
void* plan_kernel(const Plan& pl, bool bf16, bool varlen, int mode) {
  if (pl.slots == 3) return pick_kernel2<16, 3>(bf16, varlen, mode);
  if (pl.slots == 2)
    return pl.N == 32 ? pick_kernel2<16, 2>(bf16, varlen, mode) : pick_kernel2<32, 2>(bf16, varlen, mode);
  return pick_kernel_n(pl.N, bf16, varlen, mode);
}
int plan_smem(const Plan& pl) {
  if (pl.slots == 3) return Smem2<16, 3>::kDynBytes;
  if (pl.slots == 2) return pl.N == 32 ? Smem2<16, 2>::kDynBytes : Smem2<32, 2>::kDynBytes;
  return smem_bytes_for(pl.N);
}
int plan_threads(const Plan& pl, int mode) {
  if (pl.slots == 3) return Smem2<16, 3>::threads(mode);
  if (pl.slots == 2) return pl.N == 32 ? Smem2<16, 2>::threads(mode) : Smem2<32, 2>::threads(mode);
  return threads_for(pl.N);
}

// Padded layer-0 input width of the H = 128 kernels.
int tc_kx(const Problem& p) { return (p.I + kXK - 1) / kXK * kXK; }

// Clusters of 2L > 8 CTAs need the non-portable cluster size (up to 16 on B200).
cudaError_t allow_cluster(void* k, int L) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 2 * L > 8 ? 1 : 0);
}

// Max clusters of 2L CTAs (one per SM) of a plan's kernel co-resident on `device`
// (0: the cluster does not fit); cached.
int max_active_clusters(int device, int L, const Plan& pl) {
  static std::mutex mu;
  static int cache[64][kMaxLayers + 1][4][3];  // [device][L][tile rows / 16 - 1][slots - 1]
  static bool init = false;
  std::lock_guard<std::mutex> g(mu);
  if (!init) {
    for (auto& a : cache)
      for (auto& b : a)
        for (auto& c : b)
          for (auto& d : c) d = -1;
    init = true;
  }
  const int ni = std::min(pl.N / 16, 4) - 1;
  if (device < 0 || device >= 64 || L < 1 || L > kMaxLayers) return 0;
  int& slot = cache[device][L][ni][pl.slots - 1];
  if (slot >= 0) return slot;
  // The fewest co-resident clusters of the three output modes' kernels (their block sizes and
  // register counts differ), so that the plan does not depend on the output mode.
  int n = 1 << 30;
  for (int mode : {kModeSeq, kModeLast, kModeHSeq}) {
    void* k = plan_kernel(pl, false, false, mode);
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, plan_smem(pl));
    allow_cluster(k, L);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * L * 64, 1, 1);
    cfg.blockDim = dim3((unsigned)plan_threads(pl, mode), 1, 1);
    cfg.dynamicSmemBytes = plan_smem(pl);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2 * L;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int m = 0;
    if (cudaOccupancyMaxActiveClusters(&m, k, &cfg) != cudaSuccess || m < 0) {
      cudaGetLastError();
      m = 0;
    }
    n = std::min(n, m);
  }
  slot = n;
  return n;
}

Plan make_plan(const Problem& p, bool varlen) {
  Plan pl;
  // Multi-slot tiles by default: 32 rows (two 16-row slots), 48 (three 16-row slots) or
  // 64 (two 32-row slots); PLSTM_TC_KERNEL=1 selects the single-slot kernel with 16 / 32 /
  // 48-row tiles.  The smallest tile whose clusters all fit on the GPU at once (one wave);
  // beyond that the widest tile (of those whose cluster fits at all: 16-CTA clusters for
  // L > 4 need one 16-SM group).  Slots of 16 rows have the shortest step (their gate math
  // is half as long), so a batch that 15 clusters of 32 rows cannot hold (B = 512) runs as
  // 11 clusters of three 16-row slots rather than 8 clusters of two 32-row slots.
  pl.slots = 2;
  if (const char* e = std::getenv("PLSTM_TC_KERNEL"))
    if (std::atoi(e) == 1 && tc_kx(p) == kXK) pl.slots = 1;  // the single-slot kernel reads x 16 wide
  static constexpr int kTile2Ns[3] = {32, 48, 64};
  static constexpr int kTile2Slots[3] = {2, 3, 2};
  const bool multi = pl.slots == 2;
  const int* ns = multi ? kTile2Ns : kTileNs;
  const int nn = 3;
  auto slots_of = [&](int i) { return multi ? kTile2Slots[i] : 1; };
  // Three 16-row slots measured faster than two 32-row slots for uniform lengths (B = 512:
  // [B][O] 1.54 against 1.83 ms, [B][T][H] 1.54 against 2.00, [B][T][O] 1.97 against 1.99) but
  // slower for variable lengths, where 32-row tiles whose shortest tiles run in a second wave's
  // slack win (dual_plan).
  const bool allow48 = !varlen;
  int N = ns[0], slots = slots_of(0);
  for (int i = 0; i < nn; ++i) {
    if (multi && ns[i] == 48 && !allow48) continue;
    Plan c = pl;
    c.N = ns[i];
    c.slots = slots_of(i);
    const int m = max_active_clusters(p.device, p.L, c);
    if (m < 1) continue;
    N = ns[i];
    slots = c.slots;
    if ((p.B + ns[i] - 1) / ns[i] <= m) break;
  }
  if (const char* e = std::getenv("PLSTM_TC_NTILE")) {
    const int v = std::atoi(e);
    for (int i = 0; i < nn; ++i)
      if (v == ns[i]) {
        N = v;
        slots = slots_of(i);
      }
  }
  pl.slots = slots;
  pl.N = N;
  pl.tiles = (p.B + N - 1) / N;
  if (const char* dbg = std::getenv("PLSTM_TC_DEBUG"))
    if (std::atoi(dbg) != 0)
      std::fprintf(stderr, "plstm tc: %d-slot kernel, %d-row tiles, %d tiles\n", pl.slots, N, pl.tiles);
  return pl;
}

struct TcWs {
  size_t xp, perm, tile_len, hist, sorted, trace, total;
};

// A variable-length batch whose 32-row tiles need more than one wave (so the plan took
// 64-row tiles) enqueues both heights and lets tc_tile_choice_kernel pick from the sorted
// lengths: with widely spread lengths the tail 32-row tiles fit in the long tiles' slack.
struct DualPlan {
  bool on = false;
  int tiles32 = 0, m32 = 0, m64 = 0;
};
DualPlan dual_plan(const Problem& p, const Plan& pl, bool varlen) {
  DualPlan d;
  if (!varlen || pl.slots != 2 || pl.N != 64 || std::getenv("PLSTM_TC_NTILE") != nullptr) return d;
  if (p.flags & (PLSTM_FLAG_TRACE | PLSTM_FLAG_TEST_DROP)) return d;
  Plan c = pl;
  c.N = 32;
  d.tiles32 = (p.B + 31) / 32;
  d.m32 = max_active_clusters(p.device, p.L, c);
  d.m64 = max_active_clusters(p.device, p.L, pl);
  // Beyond two waves of 32-row tiles the 64-row plan won at every measured length spread
  // (B = 1024, 4096 with lengths in [200, 1000]); there the extra launches would only cost.
  d.on = d.m32 >= 1 && d.m64 >= 1 && d.tiles32 > d.m32 && d.tiles32 <= 2 * d.m32;
  return d;
}

TcWs tc_ws(const Problem& p, const Plan& pl) {
  TcWs w;
  size_t off = kStatusBytes;
  w.xp = off;
  off = align_up(off + (size_t)pl.tiles * std::max(p.T, 1) * pl.N * tc_kx(p) * 2, 256);
  w.perm = off;
  off = align_up(off + (size_t)pl.tiles * pl.N * 4, 256);
  w.tile_len = off;  // [tiles], then (two tile heights enqueued) the 32-row tiles' lengths and the choice word
  off = align_up(off + (size_t)(3 * pl.tiles + 1) * 4, 256);
  w.hist = off;
  off = align_up(off + (size_t)(p.T + 1) * 4, 256);
  w.sorted = off;
  off = align_up(off + (size_t)std::max(p.B, 1) * 4, 256);
  w.trace = off;
  if (p.flags & PLSTM_FLAG_TRACE) off += (size_t)2 * p.L * kTraceSteps * kTraceEvents * 8;
  w.total = off;
  return w;
}

// ---- dependent-step latency probe ---------------------------------------------------
// The dependency chain of one wavefront layer-step, measured alone: a cluster of two
// CTAs, each owning 64 hidden units (256 gate rows: two M = 128 tiles whose A slice,
// K = 64, sits in tensor memory), runs `steps` times
//   sibling's h lands -> 8 MMAs over it (2 tiles x 4 K steps, N = NH) + commit ->
//   mbarrier -> tcgen05.ld -> the kernel's gate math (lstm_cells, 2 x NH / 4 x 2 cells
//   per thread) -> h to shared memory -> one bulk copy of this CTA's NH x 64 units
//   (4 KB at NH = 32) into the sibling, completing on its barrier.
// Nothing else runs: no input MMAs, no own-half MMAs, no layer pipeline, no Linear head,
// no second slot.  It is the north-star "dependent-step microbenchmark": its cycles per
// step are a floor for any step of that shape.  CTA 0 records clock64 stamps of every
// step and writes, for the steps from steps / 4 on:
//   out[0] status (0 ok, 1 a bounded wait gave up), out[1] cycles, out[2] steps counted,
//   out[3..8] summed cycles of: landed -> commit issued, commit -> accumulator seen,
//   seen -> loaded, loaded -> h written (warp 0), h written -> copy issued (last warp),
//   copy issued -> next sibling h landed.
constexpr int kProbeOut = 16;

// `variant` bits select alternatives of the chain's parts (0 = the kernel's current form):
//   1: the control warp spins on mbarrier.test_wait instead of try_wait for the sibling's h;
//   2: the compute warps spin on test_wait for the accumulator;
//   4: the hand-off is st.async 16-byte stores by all 128 compute threads (after a named
//      barrier) instead of one bulk copy;
//   8: the two tiles' accumulators are loaded one after the other, the second load in flight
//      under the first tile's gate math.
//  16: the hand-off is plain 16-byte remote stores (st.shared::cluster) by all 128 compute
//      threads, a proxy fence and one cluster-scope release arrival per warp on the sibling's
//      barrier (no transaction bytes), waited for with cluster-scope acquire.
constexpr int kProbeSpinLanded = 1, kProbeSpinMma = 2, kProbeStAsync = 4, kProbeSplitLoad = 8, kProbeRemoteSt = 16;

__device__ __forceinline__ bool warp_wait_phase_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                        unsigned long long timeout_ns) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) {
    const unsigned long long t0 = ptx::globaltimer();
    while (true) {
      if (ptx::mbar_try_wait_cluster(bar, parity)) {
        ok = 1;
        break;
      }
      if (*abort_flag || ptx::globaltimer() - t0 > timeout_ns) break;
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ bool warp_spin_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                unsigned long long timeout_ns) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) {
    const unsigned long long t0 = ptx::globaltimer();
    unsigned n = 0;
    while (true) {
      if (ptx::mbar_test_wait(bar, parity)) {
        ok = 1;
        break;
      }
      if ((++n & 63) == 0 && (*abort_flag || ptx::globaltimer() - t0 > timeout_ns)) break;
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int NH>
__global__ void __launch_bounds__(160, 1) step_probe_kernel(int steps, int variant, unsigned long long timeout_ns,
                                                             unsigned long long* out) {
  constexpr int CPW = NH / 8;
  constexpr uint32_t kHalf = NH * 128;  // one 64-unit K block of h: NH rows x 128 bytes (128-byte swizzle)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = (int)ptx::cluster_ctarank();
  constexpr uint32_t kBar = 4 * kHalf;  // [parity 2][unit half 2] h buffers, then the barriers
  auto full = [&](int b) { return sbase + kBar + 8u * b; };
  auto mma = [&](int b) { return sbase + kBar + 16u + 8u * b; };
  auto hready = [&](int b) { return sbase + kBar + 32u + 8u * b; };
  auto hbuf = [&](int b, int half) { return sbase + (uint32_t)(2 * b + half) * kHalf; };
  uint32_t* counter = reinterpret_cast<uint32_t*>(sm + kBar + 48);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kBar + 52);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kBar + 56);
  volatile unsigned long long* stamp = reinterpret_cast<volatile unsigned long long*>(sm + kBar + 64);  // [8]

  for (int i = tid; i < (int)(4 * kHalf / 4); i += blockDim.x) reinterpret_cast<uint32_t*>(sm)[i] = 0u;  // h0 = 0
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(full(b), (variant & kProbeRemoteSt) ? 4 : 1);
      ptx::mbar_init(mma(b), 1);
      ptx::mbar_init(hready(b), 4);
    }
    *counter = 0;
    *abort_flag = 0;
    ptx::fence_mbar_init_cluster();
    // The sibling's h of steps 1 and 2.
    if (!(variant & kProbeRemoteSt)) {
      if (steps > 1) ptx::mbar_arrive_expect_tx(full(1), kHalf);
      if (steps > 2) ptx::mbar_arrive_expect_tx(full(0), kHalf);
    }
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + kBar + 56, 128);
    ptx::tmem_relinquish();
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
  if (warp < 4) {  // A = small alternating values, two tiles of 32 columns (K = 64) per lane
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = ((i + lane) & 1) ? 0x20002000u : 0xa000a000u;  // +-2^-7 in f16
#pragma unroll
    for (int tau = 0; tau < 2; ++tau)
      ptx::tmem_st_32x32b_x32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(32 * tau), r);
    ptx::tmem_wait_st();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::cluster_sync();
  const uint32_t dcol = tmem + 64;  // D[tau] at 64 + tau NH
  bool ok = true;
  auto give_up = [&]() {
    if (lane == 0 && !*abort_flag) {
      for (int r = 0; r < 2; ++r) ptx::st_cluster_u32(ptx::mapa(ptx::smem_u32((void*)abort_flag), (uint32_t)r), 1u);
      if (s == 0) out[0] = 1ull;
    }
    ok = false;
  };

  if (warp == 4) {
    // ---- control warp: waits for the sibling's h, issues the 8 MMAs and the commit ----
    constexpr uint32_t idesc = ptx::idesc_f16(128, NH, false);
    const int t0 = steps / 4;
    unsigned long long sum[6] = {0, 0, 0, 0, 0, 0}, first = 0, prev_push = 0, landed = 0;
    int counted = 0;
    for (int t = 0; t < steps && ok; ++t) {
      const int b = t & 1;
      if (t >= 1) {
        const uint32_t par = ((t - 1) >> 1) & 1;
        const bool got = (variant & kProbeRemoteSt)     ? warp_wait_phase_cluster(full(b), par, abort_flag, timeout_ns)
                         : (variant & kProbeSpinLanded) ? warp_spin_phase(full(b), par, abort_flag, timeout_ns)
                                                        : warp_wait_phase(full(b), par, abort_flag, timeout_ns);
        if (!got) {
          give_up();
          break;
        }
        if (!(variant & kProbeRemoteSt) && t + 2 < steps && ptx::elect_one())
          ptx::mbar_arrive_expect_tx(full(b), kHalf);
        __syncwarp();
      }
      landed = clock64();
      if (t == t0) first = landed;
      if (t > t0) sum[5] += landed - prev_push;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        const uint64_t dB = ptx::desc_k_sw128(hbuf(b, 1 - s));
#pragma unroll
        for (int tau = 0; tau < 2; ++tau)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            ptx::mma_f16_ts(dcol + (uint32_t)(tau * NH), tmem + (uint32_t)(32 * tau + 8 * kk),
                            dB + (uint64_t)((kk * 32) >> 4), idesc, kk != 0 ? 1u : 0u);
        ptx::mma_commit(mma(b));
      }
      __syncwarp();
      const unsigned long long committed = clock64();
      if (!warp_wait_phase(hready(b), (t >> 1) & 1, abort_flag, timeout_ns)) {
        give_up();
        break;
      }
      if (t >= t0) {
        sum[0] += committed - landed;
        sum[1] += stamp[0] - committed;
        sum[2] += stamp[1] - stamp[0];
        sum[3] += stamp[2] - stamp[1];
        sum[4] += stamp[3] - stamp[2];
        prev_push = stamp[3];
        ++counted;
      }
    }
    if (s == 0 && lane == 0 && ok) {
      out[0] = 0ull;
      out[1] = landed - first;
      out[2] = (unsigned long long)max(counted - 1, 0);
      for (int i = 0; i < 6; ++i) out[3 + i] = sum[i];
    }
    // The last step's MMAs completed before its gate math ran, so TMEM is idle here.
  } else {
    // ---- compute warps: lane quadrant `warp`, the kernel's gate math ----
    const int q = warp, j8 = lane >> 2, cpair = (lane & 3) * 2;
    float c_st[2][CPW][2];
    uint16_t h_st[2][CPW][2];
    int len_c[CPW][2];
    const float bz[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int tau = 0; tau < 2; ++tau)
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          c_st[tau][jc][e] = 0.f;
          h_st[tau][jc][e] = 0;
          len_c[jc][e] = steps;
        }
    for (int t = 0; t < steps && ok; ++t) {
      const int b = t & 1;
      const bool got = (variant & kProbeSpinMma) ? warp_spin_phase(mma(b), (t >> 1) & 1, abort_flag, timeout_ns)
                                                 : warp_wait_phase(mma(b), (t >> 1) & 1, abort_flag, timeout_ns);
      if (!got) {
        give_up();
        break;
      }
      ptx::tc_fence_after();
      if (q == 0 && lane == 0) stamp[0] = clock64();
      uint32_t rif[2][4 * CPW], rgo[2][4 * CPW];
      uint16_t hw[2][CPW][2];
      if (variant & kProbeSplitLoad) {
        // Tile 0's accumulators first; tile 1's load runs under tile 0's gate math.
        tmem_ld_chunks<CPW>(dcol + ((uint32_t)(32 * q) << 16), rif[0]);
        tmem_ld_chunks<CPW>(dcol + ((uint32_t)(32 * q + 16) << 16), rgo[0]);
        ptx::tmem_wait_ld();
        if (q == 0 && lane == 0) stamp[1] = clock64();
        tmem_ld_chunks<CPW>(dcol + (uint32_t)NH + ((uint32_t)(32 * q) << 16), rif[1]);
        tmem_ld_chunks<CPW>(dcol + (uint32_t)NH + ((uint32_t)(32 * q + 16) << 16), rgo[1]);
        lstm_cells_tile<CPW, false, false>(0, rif, rgo, bz, c_st, h_st, len_c, t, hw);
        ptx::tmem_wait_ld();
        reg_after_wait<4 * CPW>(rif[1]);  // tile 1's registers are read only after the wait
        reg_after_wait<4 * CPW>(rgo[1]);
        ptx::tc_fence_before();
        lstm_cells_tile<CPW, false, false>(1, rif, rgo, bz, c_st, h_st, len_c, t, hw);
      } else {
#pragma unroll
        for (int tau = 0; tau < 2; ++tau) {
          const uint32_t col = dcol + (uint32_t)(tau * NH);
          tmem_ld_chunks<CPW>(col + ((uint32_t)(32 * q) << 16), rif[tau]);
          tmem_ld_chunks<CPW>(col + ((uint32_t)(32 * q + 16) << 16), rgo[tau]);
        }
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        if (q == 0 && lane == 0) stamp[1] = clock64();
        lstm_cells<CPW, false, false>(rif, rgo, bz, c_st, h_st, len_c, t, hw);
      }
      uint8_t* dst = sm + (size_t)(2 * (b ^ 1) + s) * kHalf;
#pragma unroll
      for (int tau = 0; tau < 2; ++tau)
#pragma unroll
        for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            *reinterpret_cast<uint16_t*>(dst + sw128_off(8 * jc + cpair + e, 8 * (4 * tau + q) + j8)) = hw[tau][jc][e];
      if (variant & kProbeRemoteSt) {
        if (q == 0 && lane == 0) stamp[2] = clock64();
        ptx::named_bar_sync(1, 128);
        if (q == 0 && lane == 0) stamp[3] = clock64();
        if (t + 1 < steps) {
          const uint32_t peer = (uint32_t)(s ^ 1);
          const uint32_t src = hbuf(b ^ 1, s);
#pragma unroll
          for (int c = tid; c < (int)(kHalf / 16); c += 128) {
            const uint4 v = *reinterpret_cast<const uint4*>(sm + (src - sbase) + 16 * c);
            ptx::st_cluster_v4(ptx::mapa(src + 16u * c, peer), v);
          }
          ptx::fence_proxy_async_cluster();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive_remote(ptx::mapa(full(b ^ 1), peer));
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(hready(b));
      } else if (variant & kProbeStAsync) {
        // All four warps' h in place, then every thread forwards 16-byte pieces of the tile.
        if (q == 0 && lane == 0) stamp[2] = clock64();
        ptx::named_bar_sync(1, 128);
        if (q == 0 && lane == 0) stamp[3] = clock64();
        if (t + 1 < steps) {
          const uint32_t peer = (uint32_t)(s ^ 1);
          const uint32_t rbar = ptx::mapa(full(b ^ 1), peer);
          const uint32_t src = hbuf(b ^ 1, s);
#pragma unroll
          for (int c = tid; c < (int)(kHalf / 16); c += 128) {
            const uint4 v = *reinterpret_cast<const uint4*>(sm + (src - sbase) + 16 * c);
            ptx::st_async_v4(ptx::mapa(src + 16u * c, peer), v, rbar);
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(hready(b));
      } else {
        ptx::fence_proxy_async_smem();
        if (q == 0 && lane == 0) stamp[2] = clock64();
        __syncwarp();
        if (lane == 0) {
          if (ptx::atom_add_acq_rel_smem(ptx::smem_u32(counter), 1u) % 4u == 3u) {
            stamp[3] = clock64();
            if (t + 1 < steps) {
              const uint32_t src = hbuf(b ^ 1, s);
              ptx::bulk_s2c(ptx::mapa(src, (uint32_t)(s ^ 1)), src, kHalf, ptx::mapa(full(b ^ 1), (uint32_t)(s ^ 1)));
            }
          }
          ptx::mbar_arrive(hready(b));
        }
      }
    }
  }
  if (*abort_flag) {  // copies already in flight toward the sibling land before either CTA leaves
    const unsigned long long w0 = ptx::globaltimer();
    while (ptx::globaltimer() - w0 < 50000ull) {
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 128);
  }
  ptx::cluster_sync();
}

// The same chain with each layer split over four CTAs (variant 32 of the probe): CTA r owns
// 32 hidden units (one M = 128 tile of gate rows); per step it waits for the other three
// CTAs' 32-unit pieces of h (NH rows x 64 bytes each, K-major 8 x 16-byte core matrices, no
// swizzle, so that a piece is contiguous), issues 6 MMAs over them (3 pieces x 2 K steps),
// runs the gate math of its 32 units and pushes its own piece to the three others.
constexpr int kProbeQuad = 32;

template <int NH>
__global__ void __launch_bounds__(160, 1) step_probe4_kernel(int steps, unsigned long long timeout_ns,
                                                              unsigned long long* out) {
  constexpr int CPW = NH / 8;
  constexpr uint32_t kPiece = NH * 64;    // 32 units x NH rows, 16-bit
  constexpr uint32_t kBuf = 4 * kPiece;   // one step parity: the four pieces
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = ptx::smem_align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = (int)ptx::cluster_ctarank();
  constexpr uint32_t kBar = 2 * kBuf;
  auto full = [&](int b) { return sbase + kBar + 8u * b; };
  auto mma = [&](int b) { return sbase + kBar + 16u + 8u * b; };
  auto hready = [&](int b) { return sbase + kBar + 32u + 8u * b; };
  auto piece = [&](int b, int pc) { return sbase + (uint32_t)b * kBuf + (uint32_t)pc * kPiece; };
  uint32_t* counter = reinterpret_cast<uint32_t*>(sm + kBar + 48);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kBar + 52);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kBar + 56);
  volatile unsigned long long* stamp = reinterpret_cast<volatile unsigned long long*>(sm + kBar + 64);

  for (int i = tid; i < (int)(kBar / 4); i += blockDim.x) reinterpret_cast<uint32_t*>(sm)[i] = 0u;
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(full(b), 1);
      ptx::mbar_init(mma(b), 1);
      ptx::mbar_init(hready(b), 4);
    }
    *counter = 0;
    *abort_flag = 0;
    ptx::fence_mbar_init_cluster();
    if (steps > 1) ptx::mbar_arrive_expect_tx(full(1), 3 * kPiece);
    if (steps > 2) ptx::mbar_arrive_expect_tx(full(0), 3 * kPiece);
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + kBar + 56, 128);
    ptx::tmem_relinquish();
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
  if (warp < 4) {  // A: one tile, K = 128 (64 columns)
    uint32_t v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = ((i + lane) & 1) ? 0x20002000u : 0xa000a000u;
#pragma unroll
    for (int c = 0; c < 2; ++c) ptx::tmem_st_32x32b_x32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(32 * c), v);
    ptx::tmem_wait_st();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::cluster_sync();
  const uint32_t dcol = tmem + 64;
  bool ok = true;
  auto give_up = [&]() {
    if (lane == 0 && !*abort_flag) {
      for (int q = 0; q < 4; ++q) ptx::st_cluster_u32(ptx::mapa(ptx::smem_u32((void*)abort_flag), (uint32_t)q), 1u);
      if (r == 0) out[0] = 1ull;
    }
    ok = false;
  };

  if (warp == 4) {
    constexpr uint32_t idesc = ptx::idesc_f16(128, NH, false);
    const int t0 = steps / 4;
    unsigned long long sum[6] = {0, 0, 0, 0, 0, 0}, first = 0, prev_push = 0, landed = 0;
    int counted = 0;
    for (int t = 0; t < steps && ok; ++t) {
      const int b = t & 1;
      if (t >= 1) {
        if (!warp_wait_phase(full(b), ((t - 1) >> 1) & 1, abort_flag, timeout_ns)) {
          give_up();
          break;
        }
        if (t + 2 < steps && ptx::elect_one()) ptx::mbar_arrive_expect_tx(full(b), 3 * kPiece);
        __syncwarp();
      }
      landed = clock64();
      if (t == t0) first = landed;
      if (t > t0) sum[5] += landed - prev_push;
      if (ptx::elect_one()) {
        ptx::tc_fence_after();
        bool acc = false;
        for (int pc = 0; pc < 4; ++pc) {
          if (pc == r) continue;
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            ptx::mma_f16_ts(dcol, tmem + (uint32_t)(16 * pc + 8 * ks),
                            ptx::desc_k_none(piece(b, pc) + 256u * ks, 128, 512), idesc, acc ? 1u : 0u);
            acc = true;
          }
        }
        ptx::mma_commit(mma(b));
      }
      __syncwarp();
      const unsigned long long committed = clock64();
      if (!warp_wait_phase(hready(b), (t >> 1) & 1, abort_flag, timeout_ns)) {
        give_up();
        break;
      }
      if (t >= t0) {
        sum[0] += committed - landed;
        sum[1] += stamp[0] - committed;
        sum[2] += stamp[1] - stamp[0];
        sum[3] += stamp[2] - stamp[1];
        sum[4] += stamp[3] - stamp[2];
        prev_push = stamp[3];
        ++counted;
      }
    }
    if (r == 0 && lane == 0 && ok) {
      out[0] = 0ull;
      out[1] = landed - first;
      out[2] = (unsigned long long)max(counted - 1, 0);
      for (int i = 0; i < 6; ++i) out[3 + i] = sum[i];
    }
  } else {
    const int q = warp, j8 = lane >> 2, cpair = (lane & 3) * 2;
    float c_st[2][CPW][2];
    uint16_t h_st[2][CPW][2];
    int len_c[CPW][2];
    const float bz[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int tau = 0; tau < 2; ++tau)
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          c_st[tau][jc][e] = 0.f;
          h_st[tau][jc][e] = 0;
          len_c[jc][e] = steps;
        }
    const int u = 8 * q + j8;  // unit within this CTA's 32
    for (int t = 0; t < steps && ok; ++t) {
      const int b = t & 1;
      if (!warp_wait_phase(mma(b), (t >> 1) & 1, abort_flag, timeout_ns)) {
        give_up();
        break;
      }
      ptx::tc_fence_after();
      if (q == 0 && lane == 0) stamp[0] = clock64();
      uint32_t rif[2][4 * CPW], rgo[2][4 * CPW];
      tmem_ld_chunks<CPW>(dcol + ((uint32_t)(32 * q) << 16), rif[0]);
      tmem_ld_chunks<CPW>(dcol + ((uint32_t)(32 * q + 16) << 16), rgo[0]);
      ptx::tmem_wait_ld();
      reg_after_wait<4 * CPW>(rif[0]);
      reg_after_wait<4 * CPW>(rgo[0]);
      ptx::tc_fence_before();
      if (q == 0 && lane == 0) stamp[1] = clock64();
      uint16_t hw[2][CPW][2];
      lstm_cells_tile<CPW, false, false>(0, rif, rgo, bz, c_st, h_st, len_c, t, hw);
      uint8_t* dst = sm + (size_t)(b ^ 1) * kBuf + (size_t)r * kPiece;
#pragma unroll
      for (int jc = 0; jc < CPW; ++jc)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int row = 8 * jc + cpair + e;
          *reinterpret_cast<uint16_t*>(dst + (row >> 3) * 512 + (u >> 3) * 128 + (row & 7) * 16 + (u & 7) * 2) =
              hw[0][jc][e];
        }
      ptx::fence_proxy_async_smem();
      if (q == 0 && lane == 0) stamp[2] = clock64();
      __syncwarp();
      if (lane == 0) {
        if (ptx::atom_add_acq_rel_smem(ptx::smem_u32(counter), 1u) % 4u == 3u) {
          stamp[3] = clock64();
          if (t + 1 < steps) {
            const uint32_t src = piece(b ^ 1, r);
            for (int pr = 1; pr < 4; ++pr) {
              const uint32_t peer = (uint32_t)((r + pr) & 3);
              ptx::bulk_s2c(ptx::mapa(src, peer), src, kPiece, ptx::mapa(full(b ^ 1), peer));
            }
          }
        }
        ptx::mbar_arrive(hready(b));
      }
    }
  }
  if (*abort_flag) {
    const unsigned long long w0 = ptx::globaltimer();
    while (ptx::globaltimer() - w0 < 50000ull) {
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 128);
  }
  ptx::cluster_sync();
}

}  // namespace tc

using namespace tc;

int32_t tc_make_perm(const Problem& p, int N, int tiles, const int32_t* lengths, int32_t* perm, int32_t* tile_len,
                     int32_t* hist, int32_t* sorted, cudaStream_t s) {
  const int nthr = 256;
  const int nperm = tiles * N;
  if (lengths == nullptr) {
    tc_perm_uniform_kernel<<<(nperm + nthr - 1) / nthr, nthr, 0, s>>>(perm, tile_len, p.B, p.T, N, tiles);
    note_launches(1);
  } else {
    PLSTM_TRY_CUDA(cudaMemsetAsync(hist, 0, (size_t)(p.T + 1) * 4, s));
    tc_len_hist_kernel<<<(p.B + nthr - 1) / nthr, nthr, 0, s>>>(lengths, p.B, p.T, hist);
    tc_len_scan_kernel<<<1, 32, 0, s>>>(hist, p.T + 1);
    tc_len_scatter_kernel<<<(p.B + nthr - 1) / nthr, nthr, 0, s>>>(lengths, p.B, p.T, hist, sorted);
    tc_perm_varlen_kernel<<<(nperm + nthr - 1) / nthr, nthr, 0, s>>>(sorted, lengths, perm, tile_len, p.B, p.T, N,
                                                                      tiles);
    note_launches(4);
  }
  PLSTM_TRY_CUDA(cudaGetLastError());
  return PLSTM_OK;
}

int32_t tc_xpack(const Problem& p, int N, int tiles, const void* x, const int32_t* perm, uint8_t* xp, int kx,
                 cudaStream_t s, const int* choice) {
  if (p.T <= 0) return PLSTM_OK;
  const int nthr = 256;
  const int64_t total = (int64_t)tiles * p.T * N * (kx / 8);
  const int grid = (int)std::min<int64_t>((total + nthr - 1) / nthr, 148 * 32);
  tc_xpack_kernel<uint16_t><<<grid, nthr, 0, s>>>(static_cast<const uint16_t*>(x), perm, xp, p.B, p.T, p.I, N, tiles,
                                                  kx, choice);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

// Shapes the H = 128 wavefront kernels take; every other tensor-core shape goes to the
// layer-sequential backend (plstm_tcl.cu).
bool wavefront_shape(const Problem& p) {
  return p.H >= 1 && p.H <= kH && p.L >= 1 && p.L <= kMaxLayers && p.I <= kMaxXK && (!p.has_linear() || p.O <= 32);
}

bool tc_supported(const Problem& p, std::string* why) {
  if (!wavefront_shape(p)) return tcl_supported(p, why);
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (p.dtype != PLSTM_F16 && p.dtype != PLSTM_BF16) return no("activation type must be f16 or bf16");
  if (p.H < 1 || p.H > kH) return no("hidden_size must be <= 128");
  if (p.L < 1 || p.L > kMaxLayers) return no("num_layers must be 1..8 (one 2L-CTA cluster)");
  if (p.I > kMaxXK) return no("input_size must be <= 128");
  if (p.has_linear() && p.O > 32) return no("output_size must be <= 32");
  if (p.T > 65535) return no("seq_len must be <= 65535");
  int dev = p.device, major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    cudaGetLastError();
    return no("no CUDA device");
  }
  if (major != 10 || minor != 0) return no("device is not sm_100 (B200)");
  Plan c;
  c.slots = 2;
  c.N = 32;
  if (max_active_clusters(dev, p.L, c) < 1) return no("the 2L-CTA cluster does not fit on this device");
  return true;
}

size_t tc_packed_size(const Problem& p) { return wavefront_shape(p) ? packed_total(p.L) : tcl_packed_size(p); }

size_t tc_workspace_size(const Problem& p) {
  // The workspace is sized before the call says whether lengths come: the larger of the
  // fixed- and variable-length plans.
  if (!wavefront_shape(p)) return tcl_workspace_size(p);
  return std::max(tc_ws(p, make_plan(p, false)).total, tc_ws(p, make_plan(p, true)).total);
}

int32_t tc_pack(const Problem& p, int ih_layout, int hh_layout, const void* const* w_ih,
                const void* const* w_hh, const void* const* b_ih, const void* const* b_hh,
                const void* w_lin, const void* b_lin, void* packed, cudaStream_t s) {
  if (!wavefront_shape(p)) return tcl_pack(p, ih_layout, hh_layout, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, packed, s);
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
  a.O = p.has_linear() ? p.O : 0;
  a.kx = tc_kx(p);
  a.hid = p.H;
  tc_pack_kernel<<<148 * 4, 256, 0, s>>>(a, static_cast<uint8_t*>(packed));
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

int32_t tc_forward(const Problem& p, const void* packed, const void* x, const int32_t* lengths,
                   const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                   cudaStream_t s) {
  if (!wavefront_shape(p)) return tcl_forward(p, packed, x, lengths, h0, c0, out, h_n, c_n, ws, s);
  const Plan pl = make_plan(p, lengths != nullptr);
  const TcWs w = tc_ws(p, pl);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  int32_t* perm = reinterpret_cast<int32_t*>(wsb + w.perm);
  int32_t* tile_len = reinterpret_cast<int32_t*>(wsb + w.tile_len);
  const DualPlan dual = dual_plan(p, pl, lengths != nullptr);
  int32_t* len32 = tile_len + pl.tiles;
  int* choice = dual.on ? reinterpret_cast<int*>(len32 + dual.tiles32) : nullptr;
  int32_t* hist = reinterpret_cast<int32_t*>(wsb + w.hist);
  int32_t* sorted = reinterpret_cast<int32_t*>(wsb + w.sorted);
  // The multi-slot kernels read x[B][T][I] themselves when it is at most 16 columns wide (one
  // 16-wide K step: the layer-0 x warp fills the input tiles); otherwise x is repacked into
  // per-tile K-major tiles first.  PLSTM_TC_XPACK=1 forces the repack (for comparisons).
  const bool fuse_x = pl.slots >= 2 && tc_kx(p) == kXK && !(p.out_seq() && p.L == 1) &&
                      std::getenv("PLSTM_TC_XPACK") == nullptr;
  if (!dual.on) {
    int32_t rc = tc_make_perm(p, pl.N, pl.tiles, lengths, perm, tile_len, hist, sorted, s);
    if (rc == PLSTM_OK && !fuse_x) rc = tc_xpack(p, pl.N, pl.tiles, x, perm, wsb + w.xp, tc_kx(p), s);
    if (rc != PLSTM_OK) return rc;
  } else {
    // One length-sorted order serves both heights (64-row tile j = 32-row tiles 2j, 2j+1);
    // the 64-row launch's last 32 perm entries may be padding.
    const int tail = pl.tiles * 64 - dual.tiles32 * 32;
    if (tail > 0) PLSTM_TRY_CUDA(cudaMemsetAsync(perm + dual.tiles32 * 32, 0xff, (size_t)tail * 4, s));
    int32_t rc = tc_make_perm(p, 32, dual.tiles32, lengths, perm, len32, hist, sorted, s);
    if (rc != PLSTM_OK) return rc;
    tc_tile_choice_kernel<<<1, 32, 0, s>>>(len32, dual.tiles32, pl.tiles, p.L, dual.m32, dual.m64, tile_len, choice);
    PLSTM_TRY_CUDA(cudaGetLastError());
    note_launches(1);
    if (!fuse_x) {
      rc = tc_xpack(p, 32, dual.tiles32, x, perm, wsb + w.xp, tc_kx(p), s, choice);
      if (rc == PLSTM_OK) rc = tc_xpack(p, 64, pl.tiles, x, perm, wsb + w.xp, tc_kx(p), s, choice);
    }
    if (rc != PLSTM_OK) return rc;
  }
  Params kp = {};
  kp.packed = static_cast<const uint8_t*>(packed);
  kp.xp = fuse_x ? nullptr : wsb + w.xp;
  kp.x_raw = static_cast<const uint16_t*>(x);
  kp.I = p.I;
  kp.perm = perm;
  kp.lengths = lengths;
  kp.tile_len = tile_len;
  kp.h0 = h0;
  kp.c0 = c0;
  kp.out = out;
  kp.h_n = h_n;
  kp.c_n = c_n;
  kp.status = reinterpret_cast<int*>(wsb);
  kp.B = p.B;
  kp.T = p.T;
  kp.L = p.L;
  kp.O = p.O;
  kp.flags = p.flags;
  kp.kx = tc_kx(p);
  kp.hid = p.H;
  kp.timeout_ns = (unsigned long long)p.timeout_ms * 1000000ull;
  kp.drop_rank = -1;
  kp.drop_step = -1;
  kp.trace = nullptr;
  kp.trace_t0 = p.T / 2;
  kp.trace_slot = 0;
  kp.choice = choice;
  if (const char* e = std::getenv("PLSTM_TC_TRACE_SLOT")) kp.trace_slot = std::atoi(e) == 1 ? 1 : 0;
  if (p.flags & PLSTM_FLAG_TRACE) {
    kp.trace = reinterpret_cast<unsigned long long*>(wsb + w.trace);
    PLSTM_TRY_CUDA(cudaMemsetAsync(kp.trace, 0, (size_t)2 * p.L * kTraceSteps * kTraceEvents * 8, s));
  }
  if (p.flags & PLSTM_FLAG_TEST_DROP) {
    kp.drop_rank = p.L >= 2 ? 2 : 0;
    kp.drop_step = 0;
  }
  const bool bf16 = p.dtype == PLSTM_BF16;
  const int mode = mode_of(p);
  auto launch = [&](const Plan& lp, const int32_t* lp_tile_len) -> int32_t {
    void* k = plan_kernel(lp, bf16, lengths != nullptr, mode);
    const int smem = plan_smem(lp);
    PLSTM_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    PLSTM_TRY_CUDA(allow_cluster(k, p.L));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(lp.tiles * 2 * p.L), 1, 1);
    cfg.blockDim = dim3((unsigned)plan_threads(lp, mode), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2 * p.L;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    Params lkp = kp;
    lkp.tile_len = lp_tile_len;
    void* args[] = {&lkp};
    PLSTM_TRY_CUDA(cudaLaunchKernelExC(&cfg, k, args));
    note_launches(1);
    return PLSTM_OK;
  };
  profile_begin(s);
  int32_t rc = launch(pl, tile_len);
  if (rc == PLSTM_OK && dual.on) {
    Plan p32 = pl;
    p32.N = 32;
    p32.tiles = dual.tiles32;
    rc = launch(p32, len32);
  }
  profile_end(s);
  return rc;
}

}  // namespace plstm

using namespace plstm;
using namespace plstm::tc;

// Dependent-step latency probe (see step_probe_kernel).  out: device buffer of
// kProbeOut uint64 words.
extern "C" int32_t plstm_diag_step_latency(int32_t rows, int32_t steps, int32_t variant, uint64_t* out,
                                           int32_t timeout_ms, void* stream) {
  clear_error();
  PLSTM_CHECK_ARG(rows == 16 || rows == 32, "rows must be 16 or 32");
  PLSTM_CHECK_ARG(steps >= 8 && steps <= 1000000, "steps must be in [8, 1000000]");
  PLSTM_CHECK_ARG(out != nullptr, "out is NULL");
  PLSTM_CHECK_ARG(timeout_ms >= 0, "timeout_ms must be >= 0");
  PLSTM_CHECK_ARG(variant == kProbeQuad || (variant >= 0 && variant < 32 && !((variant & 4) && (variant & 16))),
                  "variant must be in [0, 32) (not both 4 and 16) or 32");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool quad = variant == kProbeQuad;
  void* k = quad ? (rows == 16 ? (void*)step_probe4_kernel<16> : (void*)step_probe4_kernel<32>)
                 : (rows == 16 ? (void*)step_probe_kernel<16> : (void*)step_probe_kernel<32>);
  const int smem = 4 * rows * 128 + 1024 + 1024;
  PLSTM_TRY_CUDA(cudaMemsetAsync(out, 0, kProbeOut * sizeof(uint64_t), s));
  PLSTM_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(quad ? 4 : 2, 1, 1);
  cfg.blockDim = dim3(160, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = quad ? 4 : 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int st = steps;
  unsigned long long tns = (unsigned long long)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000ull;
  int var = variant;
  void* args2[] = {&st, &var, &tns, &out};
  void* args4[] = {&st, &tns, &out};
  PLSTM_TRY_CUDA(cudaLaunchKernelExC(&cfg, k, quad ? args4 : args2));
  note_launches(1);
  return PLSTM_OK;
}
