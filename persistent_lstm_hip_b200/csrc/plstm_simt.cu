// plstm_simt.cu — generic layer-sequential LSTM backend (FFMA, f32 accumulate).
//
// Serves every shape and element type the tensor-core wavefront kernel does
// not: any I, H, L, O, f32 activations (the north star's 1e-4 path) and the
// generic-shape entry point of the reference
// (persistent_lstm_regressor_forward_generic_projected,
// persistent_lstm_hip.cu:2923-3181).  One persistent launch per layer runs the
// whole T loop for a tile of batch rows; the layer's weights are read from L2
// every step in a transposed [K][4H] layout so that consecutive threads read
// consecutive gate rows.
//
// Packed image (all offsets 256-byte aligned), per layer l:
//   wih_t[l]  [K4_l][4H] activation type   (K_0 = I, K_l = H; K4 = K rounded up to 4, pad rows zero)
//   whh_t[l]  [H4][4H]   activation type   (H4 = H rounded up to 4, pad rows zero)
//   bias[l]   [4H]       f32, b_ih + b_hh summed in f32
// then W_lin [O][H] (activation type) and b_lin [O] (f32).
#include <algorithm>
#include <type_traits>
#include <vector>

#include "plstm_common.cuh"
#include "sm100_ptx.cuh"

namespace plstm {
namespace {

struct SimtLayout {
  std::vector<size_t> wih, whh, bias;
  size_t wlin = 0, blin = 0, total = 0;
};

SimtLayout simt_layout(const Problem& p) {
  SimtLayout lo;
  const size_t es = dtype_size(p.dtype);
  const size_t G = 4 * (size_t)p.H;
  size_t off = 0;
  for (int l = 0; l < p.L; ++l) {
    const size_t K = l == 0 ? p.I : p.H;
    lo.wih.push_back(off);
    off = align_up(off + align_up(K, 4) * G * es, 256);
    lo.whh.push_back(off);
    off = align_up(off + align_up(p.H, 4) * G * es, 256);
    lo.bias.push_back(off);
    off = align_up(off + G * 4, 256);
  }
  lo.wlin = off;
  off = align_up(off + (size_t)std::max(p.O, 1) * p.H * es, 256);
  lo.blin = off;
  off = align_up(off + (size_t)std::max(p.O, 1) * 4, 256);
  lo.total = off;
  return lo;
}

struct SimtWs {
  size_t seq[2], hfin, cfin, total;
};

SimtWs simt_ws(const Problem& p) {
  SimtWs w;
  const size_t es = dtype_size(p.dtype);
  size_t off = kStatusBytes;
  const size_t seq_bytes = align_up((size_t)p.B * p.T * p.H * es, 256);
  w.seq[0] = off;
  off += seq_bytes;
  w.seq[1] = off;
  off += seq_bytes;
  w.hfin = off;
  off = align_up(off + (size_t)p.L * p.B * p.H * es, 256);
  w.cfin = off;
  off = align_up(off + (size_t)p.L * p.B * p.H * 4, 256);
  w.total = off;
  return w;
}

// dst[k][r] = W[r][k] (transposed to [K4][rows], K4 = K rounded up to 4, rows k >= K zero) converted to
// the activation type.
__global__ void pack_transposed_kernel(const void* src, int src_dtype, int layout, int rows, int K,
                                       void* dst, int dst_dtype) {
  const int64_t n = (int64_t)rows * ((K + 3) & ~3);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i / rows);
    const int r = (int)(i % rows);
    store_any(dst, dst_dtype, i, k < K ? load_any(src, src_dtype, weight_src_index(layout, rows, K, r, k)) : 0.0f);
  }
}

// dst[r][k] = W[r][k] (native [rows][K]).
__global__ void pack_native_kernel(const void* src, int src_dtype, int layout, int rows, int K,
                                   void* dst, int dst_dtype) {
  const int64_t n = (int64_t)rows * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / K);
    const int k = (int)(i % K);
    store_any(dst, dst_dtype, i, load_any(src, src_dtype, weight_src_index(layout, rows, K, r, k)));
  }
}

// dst[i] = a[i] + b[i] in f32 (either may be null).
__global__ void pack_bias_kernel(const void* a, const void* b, int dtype, int n, float* dst) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (a != nullptr) v += load_any(a, dtype, i);
    if (b != nullptr) v += load_any(b, dtype, i);
    dst[i] = v;
  }
}

constexpr int kSimtThreads = 512;
constexpr size_t kSimtSmemMax = 227 * 1024 - 256;  // dynamic shared memory; the static lens[] needs the rest

// Four consecutive gate rows of one transposed weight row, as f32.
__device__ __forceinline__ float4 ld_w4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld_w4(const __half* p) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float4 ld_w4(const __nv_bfloat16* p) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// acc[n][i] += sum_{k < nk} w[k * G + i] * v[n * ld + k] for the four rows i of one quad, in increasing
// k; nk, v and ld are multiples of 4 (zero-padded rows), so each group of four k takes four vector weight
// loads and one 16-byte shared load per batch row.  The loop is bound by the latency of the L2 weight
// reads: each round issues the loads of U groups before any of their FMAs.
template <typename T, int NB>
__device__ __forceinline__ void quad_dot(const T* __restrict__ w, int G, const float* v, int ld, int nk,
                                         float (&acc)[NB][4]) {
  constexpr int U = NB >= 8 ? 2 : 4;  // groups of four k per round
  for (int k = 0; k < nk; k += 4 * U) {
    float4 wv[U][4];
#pragma unroll
    for (int g = 0; g < U; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        wv[g][j] = k + 4 * g < nk ? ld_w4(w + (int64_t)(k + 4 * g + j) * G) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int g = 0; g < U; ++g) {
      if (k + 4 * g >= nk) break;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float4 x = *reinterpret_cast<const float4*>(v + n * ld + k + 4 * g);
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[n][0] = fmaf(wv[g][j].x, xs[j], acc[n][0]);
          acc[n][1] = fmaf(wv[g][j].y, xs[j], acc[n][1]);
          acc[n][2] = fmaf(wv[g][j].z, xs[j], acc[n][2]);
          acc[n][3] = fmaf(wv[g][j].w, xs[j], acc[n][3]);
        }
      }
    }
  }
}

// Launch shape of one layer: NB batch rows per CTA, the combined [x_t ; h_{t-1}] contraction
// split into `ks` k-slices whose partial gate sums are added in slice order.
struct SimtShape {
  int nb, ks;
  size_t smem;
};

size_t simt_smem(int nb, int ks, int K, int H) {
  const size_t ldx = align_up(K, 4) + align_up(H, 4);
  return sizeof(float) * (nb * (ldx + (size_t)ks * 4 * H + H) + 4 * (size_t)H);
}

// Fewest batch rows per CTA that keep the grid within one wave of 148 CTAs (the per-step cost
// of a CTA is set by streaming the layer's weights from L2, not by its row count), then the
// k-split that best fills whole rounds of kSimtThreads quad-slices with at least 16 k per slice.
SimtShape simt_shape(int B, int K, int H) {
  int nb = 1;
  while (nb < 8 && (B + nb - 1) / nb > 148) nb *= 2;
  while (nb > 1 && simt_smem(nb, 1, K, H) > kSimtSmemMax) nb /= 2;
  int best = 1;
  double best_eff = 0.0;
  for (int ks = 1; ks <= 8; ++ks) {
    if (ks > 1 && (K + H) / ks < 16) break;  // at least 16 k per slice
    if (simt_smem(nb, ks, K, H) > kSimtSmemMax) break;
    const int items = ks * H;
    const int rounds = (items + kSimtThreads - 1) / kSimtThreads;
    const double eff = (double)items / ((double)rounds * kSimtThreads);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = ks;
    }
  }
  return {nb, best, simt_smem(nb, best, K, H)};
}

// One layer, whole sequence, NB batch rows per CTA.
// xin: layer input [B][T][K] (activation type T).  seq_out[b * out_sb + t * out_st + u].
// gin: optional precomputed input projection added to the gates, gin[b * gin_sb + t * gin_st + r]
// (the hidden-update entry point runs with K = 0 and gin set).
// hfin/cfin: final state of this layer [B][H] (T / f32).
// Each step a work item (quad q, slice s) accumulates gate rows 4q..4q+3 over the slice's k range
// of [x_t ; 0 ; h_{t-1} ; 0] (x and h each zero-padded to a multiple of 4, like the weight rows),
// reading each transposed weight row as one vector; the gate phase adds bias, gin and the slices'
// partial sums in that order.
template <typename T, int NB>
__global__ void __launch_bounds__(kSimtThreads)
    simt_layer_kernel(const T* __restrict__ xin, int K, const T* __restrict__ wih_t,
                      const T* __restrict__ whh_t, const float* __restrict__ bias,
                      const int32_t* __restrict__ lengths, const T* __restrict__ h0,
                      const T* __restrict__ c0, T* __restrict__ seq_out, T* __restrict__ hfin,
                      float* __restrict__ cfin, int B, int Tn, int H, const T* __restrict__ gin,
                      int64_t gin_sb, int64_t gin_st, int64_t out_sb, int64_t out_st, int ks_n) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int G = 4 * H;
  const int K4 = (K + 3) & ~3;
  const int ldx = K4 + ((H + 3) & ~3);
  float* xh = smem;                        // [NB][ldx]: x_t at 0, h_{t-1} at K4, pads zero
  float* part = xh + NB * ldx;             // [ks_n][NB][4H] partial gate sums
  float* cst = part + (size_t)ks_n * NB * G;  // [NB][H]
  float* bsm = cst + NB * H;                // [4H] bias
  __shared__ int lens[NB];
  const int b0 = blockIdx.x * NB;
  const int tid = threadIdx.x;
  const int chunk = ((ldx + ks_n - 1) / ks_n + 3) & ~3;

  if (tid < NB) {
    const int b = b0 + tid;
    int len = 0;
    if (b < B) len = lengths != nullptr ? min(max(lengths[b], 0), Tn) : Tn;
    lens[tid] = len;
  }
  for (int i = tid; i < NB * ldx; i += blockDim.x) xh[i] = 0.0f;
  for (int r = tid; r < G; r += blockDim.x) bsm[r] = bias != nullptr ? bias[r] : 0.0f;
  __syncthreads();
  for (int i = tid; i < NB * H; i += blockDim.x) {
    const int n = i / H, u = i % H, b = b0 + n;
    float hv = 0.0f, cv = 0.0f;
    if (b < B) {
      if (h0 != nullptr) hv = to_f32(h0[(int64_t)b * H + u]);
      if (c0 != nullptr) cv = to_f32(c0[(int64_t)b * H + u]);
    }
    xh[n * ldx + K4 + u] = hv;
    cst[i] = cv;
  }
  __syncthreads();
  int tmax = 0;
#pragma unroll
  for (int n = 0; n < NB; ++n) tmax = max(tmax, lens[n]);

  // x_t of batch row n, element k (zero for rows past B).
  auto x_at = [&](int i, int t) {
    const int n = i / K, k = i % K, b = b0 + n;
    return b < B ? to_f32(xin[((int64_t)b * Tn + t) * K + k]) : 0.0f;
  };
  if (tmax > 0) {
    for (int i = tid; i < NB * K; i += blockDim.x) xh[(i / K) * ldx + i % K] = x_at(i, 0);
    __syncthreads();
  }
  constexpr int kXPre = 2;  // x_{t+1} items per thread loaded under step t's contraction
  for (int t = 0; t < tmax; ++t) {
    const bool next = t + 1 < tmax;
    float xr[kXPre];
#pragma unroll
    for (int m = 0; m < kXPre; ++m) {
      const int i = tid + m * blockDim.x;
      xr[m] = next && i < NB * K ? x_at(i, t + 1) : 0.0f;
    }
    for (int item = tid; item < ks_n * H; item += blockDim.x) {
      const int q = item % H, s = item / H;
      const int k0 = s * chunk, k1 = min(ldx, k0 + chunk);
      float acc[NB][4];
#pragma unroll
      for (int n = 0; n < NB; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
      if (k0 < K4) quad_dot<T, NB>(wih_t + (int64_t)k0 * G + 4 * q, G, xh + k0, ldx, min(k1, K4) - k0, acc);
      const int j0 = max(k0, K4);
      if (j0 < k1) quad_dot<T, NB>(whh_t + (int64_t)(j0 - K4) * G + 4 * q, G, xh + j0, ldx, k1 - j0, acc);
#pragma unroll
      for (int n = 0; n < NB; ++n)
        *reinterpret_cast<float4*>(part + ((size_t)s * NB + n) * G + 4 * q) =
            make_float4(acc[n][0], acc[n][1], acc[n][2], acc[n][3]);
    }
    __syncthreads();
    for (int i = tid; i < NB * H; i += blockDim.x) {
      const int n = i / H, u = i % H, b = b0 + n;
      if (t < lens[n]) {
        float g[4];
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
          const int r = gi * H + u;
          float v = bsm[r];
          if (gin != nullptr) v += to_f32(gin[(int64_t)b * gin_sb + (int64_t)t * gin_st + r]);
          for (int s = 0; s < ks_n; ++s) v += part[((size_t)s * NB + n) * G + r];
          g[gi] = v;
        }
        const float ig = sigmoid_acc(g[0]);
        const float fg = sigmoid_acc(g[1]);
        const float gg = tanh_acc(g[2]);
        const float og = sigmoid_acc(g[3]);
        const float c = fg * cst[i] + ig * gg;
        cst[i] = c;
        const T hq = from_f32<T>(og * tanh_acc(c));  // h is kept in the activation type
        xh[n * ldx + K4 + u] = to_f32(hq);
        seq_out[(int64_t)b * out_sb + (int64_t)t * out_st + u] = hq;
      } else if (b < B) {
        seq_out[(int64_t)b * out_sb + (int64_t)t * out_st + u] = from_f32<T>(0.0f);
      }
    }
    if (next) {  // the x part of xh is not read by the gate phase
#pragma unroll
      for (int m = 0; m < kXPre; ++m) {
        const int i = tid + m * blockDim.x;
        if (i < NB * K) xh[(i / K) * ldx + i % K] = xr[m];
      }
      for (int i = tid + kXPre * blockDim.x; i < NB * K; i += blockDim.x) xh[(i / K) * ldx + i % K] = x_at(i, t + 1);
    }
    __syncthreads();
  }
  // Rows of this tile are all done at tmax; zero their remaining outputs.
  for (int n = 0; n < NB; ++n) {
    const int b = b0 + n;
    if (b >= B) break;
    const int64_t cnt = (int64_t)(Tn - tmax) * H;
    for (int64_t i = tid; i < cnt; i += blockDim.x)
      seq_out[(int64_t)b * out_sb + (int64_t)(tmax + i / H) * out_st + i % H] = from_f32<T>(0.0f);
  }
  for (int i = tid; i < NB * H; i += blockDim.x) {
    const int n = i / H, u = i % H, b = b0 + n;
    if (b < B) {
      hfin[(int64_t)b * H + u] = from_f32<T>(xh[n * ldx + K4 + u]);
      cfin[(int64_t)b * H + u] = cst[i];
    }
  }
}

// Launches simt_layer_kernel with the shape simt_shape picks.
template <typename T>
int32_t launch_simt_layer(const T* xin, int K, const T* wih_t, const T* whh_t, const float* bias,
                          const int32_t* lengths, const T* h0, const T* c0, T* seq_out, T* hfin, float* cfin,
                          int B, int Tn, int H, const T* gin, int64_t gin_sb, int64_t gin_st, int64_t out_sb,
                          int64_t out_st, cudaStream_t s) {
  const SimtShape sh = simt_shape(B, K, H);
  if (sh.smem > kSimtSmemMax) {
    set_error("hidden size too large for the FFMA backend's shared-memory tile");
    return PLSTM_ENOTSUP;
  }
  auto kern = simt_layer_kernel<T, 1>;
  if (sh.nb == 2) kern = simt_layer_kernel<T, 2>;
  if (sh.nb == 4) kern = simt_layer_kernel<T, 4>;
  if (sh.nb == 8) kern = simt_layer_kernel<T, 8>;
  PLSTM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.smem));
  kern<<<(B + sh.nb - 1) / sh.nb, kSimtThreads, sh.smem, s>>>(xin, K, wih_t, whh_t, bias, lengths, h0, c0,
                                                              seq_out, hfin, cfin, B, Tn, H, gin, gin_sb, gin_st,
                                                              out_sb, out_st, sh.ks);
  PLSTM_TRY_CUDA(cudaGetLastError());
  return PLSTM_OK;
}

// ---- cluster-resident f32 layer kernel (H <= 128, K <= 128) -------------------------------
// A cluster of kClC CTAs runs one layer for NB batch rows.  CTA c owns the units
// [c U, (c + 1) U), U = ceil(H / 16) * 4 (units >= H are zero padding), with all four gates:
// its LR = 4U gate rows of W_ih^T / W_hh^T (local row g U + j = global row g H + c U + j;
// zero for padding units) stay in shared memory for
// the whole sequence instead of streaming from L2 every step.  Each step every CTA
// contracts [x_t ; h_{t-1}] (its own full copy) against its rows in k-slices, applies the
// gate math to its units and stores h_t into the next step's buffer of every CTA of the
// cluster (distributed shared memory); one cluster barrier per step orders those stores.
// The contraction order per row (k-slices of the same width, partial sums added in slice
// order) does not depend on the row's companions, the batch size or the tile.
constexpr int kClC = 4;
constexpr int kClThreads = 512;
constexpr int kClRowGroups = 2;  // a work item holds NB / 2 batch rows, so 512 threads fit the registers

// Units per CTA: a multiple of 4, so quads of local rows stay inside one gate.
__host__ __device__ inline int cl_units(int H) { return (H + 15) / 16 * 4; }

struct ClShape {
  int nb, slices;
  size_t smem;
};

// Floats: w [K4 + H4][LR] | part [slices][NB][LR] | xh [2][NB][K4 + H4] | cst [NB][U] | bias [LR].
size_t simt_cl_smem(int nb, int slices, int K, int H) {
  const size_t ldx = align_up(K, 4) + align_up(H, 4);
  const size_t U = cl_units(H), LR = 4 * U;
  return sizeof(float) * (ldx * LR + (size_t)slices * nb * LR + 2 * (size_t)nb * ldx + (size_t)nb * U + LR);
}

// Shapes the cluster kernel serves, for batches it runs in one wave of 37 clusters of at
// most 16 rows; larger batches stream the weights from L2 (simt_layer_kernel), which is
// faster there (f32, H = 128, L = 4, B = 1024: 45.8 ms against 58.7 ms in two waves).
bool simt_cl_supported(int dtype, int K, int H, int route_batch) {
  return dtype == PLSTM_F32 && H >= 1 && H <= 128 && K >= 0 && K <= 128 &&
         route_batch <= 148 / kClC * 16;
}

// Quads of consecutive local rows (U of them) times k-slices times the two row groups fill
// the CTA's threads (at most 16 slices).
int simt_cl_slices(int H) { return std::min(kClThreads / kClRowGroups / cl_units(H), 16); }

// Fewest batch rows per cluster (4, 8 or 16) that keep the clusters within 37 (148 SMs /
// 4), then fewer while the shared memory does not fit.
ClShape simt_cl_shape(int B, int K, int H) {
  const int slices = simt_cl_slices(H);
  int nb = 4;
  while (nb < 16 && (B + nb - 1) / nb > 148 / kClC) nb *= 2;
  while (nb > 4 && simt_cl_smem(nb, slices, K, H) > kSimtSmemMax) nb /= 2;
  return {nb, slices, simt_cl_smem(nb, slices, K, H)};
}

template <int NB>
__global__ void __cluster_dims__(kClC, 1, 1) __launch_bounds__(kClThreads)
    simt_cl_layer_kernel(const float* __restrict__ xin, int K, const float* __restrict__ wih_t,
                         const float* __restrict__ whh_t, const float* __restrict__ bias,
                         const int32_t* __restrict__ lengths, const float* __restrict__ h0,
                         const float* __restrict__ c0, float* __restrict__ seq_out, float* __restrict__ hfin,
                         float* __restrict__ cfin, int B, int Tn, int H, int slices, int64_t out_sb, int64_t out_st) {
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  const int G = 4 * H;
  const int U = cl_units(H);  // units of this CTA (c U + j >= H: padding)
  const int LR = 4 * U;       // its gate rows
  const int K4 = (K + 3) & ~3;
  const int ldx = K4 + ((H + 3) & ~3);
  float* w = smem;                               // [ldx][LR]
  float* part = w + (size_t)ldx * LR;            // [slices][NB][LR]
  float* xh = part + (size_t)slices * NB * LR;   // [2][NB][ldx]
  float* cst = xh + 2 * NB * ldx;                // [NB][U]
  float* bsm = cst + NB * U;                     // [LR]
  __shared__ int lens[NB];
  const int c = (int)ptx::cluster_ctarank();
  const int b0 = (blockIdx.x / kClC) * NB;
  const int tid = threadIdx.x;
  const int chunk = ((ldx + slices - 1) / slices + 3) & ~3;
  auto grow = [&](int lr) { return (lr / U) * H + c * U + lr % U; };  // local -> global gate row
  auto real = [&](int lr) { return c * U + lr % U < H; };

  if (tid < NB) {
    const int b = b0 + tid;
    lens[tid] = b < B ? (lengths != nullptr ? min(max(lengths[b], 0), Tn) : Tn) : 0;
  }
  for (int i = tid; i < ldx * LR; i += blockDim.x) {
    const int k = i / LR, lr = i % LR;
    float v = 0.0f;
    if (real(lr)) {
      if (k < K) v = wih_t[(int64_t)k * G + grow(lr)];
      else if (k >= K4) v = whh_t[(int64_t)(k - K4) * G + grow(lr)];
    }
    w[i] = v;
  }
  for (int i = tid; i < LR; i += blockDim.x) bsm[i] = real(i) ? bias[grow(i)] : 0.0f;
  for (int i = tid; i < 2 * NB * ldx; i += blockDim.x) xh[i] = 0.0f;
  __syncthreads();
  for (int i = tid; i < NB * H; i += blockDim.x) {
    const int n = i / H, u = i % H, b = b0 + n;
    if (b < B && h0 != nullptr) xh[n * ldx + K4 + u] = h0[(int64_t)b * H + u];
  }
  for (int i = tid; i < NB * U; i += blockDim.x) {
    const int n = i / U, j = i % U, b = b0 + n;
    cst[i] = (b < B && c0 != nullptr && c * U + j < H) ? c0[(int64_t)b * H + c * U + j] : 0.0f;
  }
  int tmax = 0;
#pragma unroll
  for (int n = 0; n < NB; ++n) tmax = max(tmax, lens[n]);
  for (int i = tid; i < NB * K; i += blockDim.x) {
    const int n = i / K, k = i % K, b = b0 + n;
    if (b < B && tmax > 0) xh[n * ldx + k] = xin[((int64_t)b * Tn) * K + k];
  }
  // Every CTA's buffers are initialised before any sibling stores into them.
  ptx::cluster_sync();
  const uint32_t xh_u32 = ptx::smem_u32(xh);
  constexpr int NR = NB / kClRowGroups;  // batch rows of one work item
  constexpr int kXPre = 4;                // NB * K <= 16 * 128 = kXPre * kClThreads
  for (int t = 0; t < tmax; ++t) {
    const float* xc = xh + (t & 1) * NB * ldx;
    const int nxt = ((t + 1) & 1) * NB * ldx;  // float offset of the next step's buffer
    float xr[kXPre];                           // x_{t+1}, loaded under the contraction
#pragma unroll
    for (int m = 0; m < kXPre; ++m) {
      const int i = tid + m * kClThreads;
      const int n = i / max(K, 1), b = b0 + n;
      xr[m] = (t + 1 < tmax && i < NB * K && b < B) ? xin[((int64_t)b * Tn + t + 1) * K + i % K] : 0.0f;
    }
    for (int item = tid; item < U * slices * kClRowGroups; item += blockDim.x) {
      const int q = item % U, s = (item / U) % slices, n0 = item / (U * slices) * NR;
      const int k0 = s * chunk, k1 = min(ldx, k0 + chunk);
      float acc[NR][4];
#pragma unroll
      for (int n = 0; n < NR; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
      for (int k = k0; k < k1; k += 4) {
        float4 wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const float4*>(w + (size_t)(k + j) * LR + 4 * q);
#pragma unroll
        for (int n = 0; n < NR; ++n) {
          const float4 xv = *reinterpret_cast<const float4*>(xc + (n0 + n) * ldx + k);
          const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[n][0] = fmaf(wv[j].x, xs[j], acc[n][0]);
            acc[n][1] = fmaf(wv[j].y, xs[j], acc[n][1]);
            acc[n][2] = fmaf(wv[j].z, xs[j], acc[n][2]);
            acc[n][3] = fmaf(wv[j].w, xs[j], acc[n][3]);
          }
        }
      }
#pragma unroll
      for (int n = 0; n < NR; ++n)
        *reinterpret_cast<float4*>(part + ((size_t)s * NB + n0 + n) * LR + 4 * q) =
            make_float4(acc[n][0], acc[n][1], acc[n][2], acc[n][3]);
    }
    __syncthreads();
    for (int i = tid; i < NB * U; i += blockDim.x) {
      const int n = i / U, j = i % U, b = b0 + n, u = c * U + j;
      if (u >= H) continue;  // padding unit
      float hv;
      if (t < lens[n]) {
        float g[4];
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
          const int lr = gi * U + j;
          float v = bsm[lr];
          for (int s = 0; s < slices; ++s) v += part[((size_t)s * NB + n) * LR + lr];
          g[gi] = v;
        }
        const float cn = sigmoid_acc(g[1]) * cst[i] + sigmoid_acc(g[0]) * tanh_acc(g[2]);
        cst[i] = cn;
        hv = sigmoid_acc(g[3]) * tanh_acc(cn);
        seq_out[(int64_t)b * out_sb + (int64_t)t * out_st + u] = hv;
      } else {
        hv = xc[n * ldx + K4 + u];  // finished rows keep h
        if (b < B) seq_out[(int64_t)b * out_sb + (int64_t)t * out_st + u] = 0.0f;
      }
      const uint32_t addr = xh_u32 + (uint32_t)(nxt + n * ldx + K4 + u) * 4u;
#pragma unroll
      for (int r = 0; r < kClC; ++r) ptx::st_cluster_u32(ptx::mapa(addr, (uint32_t)r), __float_as_uint(hv));
    }
#pragma unroll
    for (int m = 0; m < kXPre; ++m) {
      const int i = tid + m * kClThreads;
      if (t + 1 < tmax && i < NB * K) xh[nxt + (i / K) * ldx + i % K] = xr[m];
    }
    // h_t of every unit is in every CTA's next buffer before the step after reads it.
    ptx::cluster_sync();
  }
  const float* xl = xh + (tmax & 1) * NB * ldx;
  for (int n = 0; n < NB; ++n) {
    const int b = b0 + n;
    if (b >= B) break;
    const int64_t cnt = (int64_t)(Tn - tmax) * U;
    for (int64_t i = tid; i < cnt; i += blockDim.x)
      if (c * U + i % U < H) seq_out[(int64_t)b * out_sb + (int64_t)(tmax + i / U) * out_st + c * U + i % U] = 0.0f;
  }
  for (int i = tid; i < NB * U; i += blockDim.x) {
    const int n = i / U, j = i % U, b = b0 + n;
    if (b < B && c * U + j < H) {
      hfin[(int64_t)b * H + c * U + j] = xl[n * ldx + K4 + c * U + j];
      cfin[(int64_t)b * H + c * U + j] = cst[i];
    }
  }
}

int32_t launch_simt_cl_layer(const float* xin, int K, const float* wih_t, const float* whh_t, const float* bias,
                             const int32_t* lengths, const float* h0, const float* c0, float* seq_out, float* hfin,
                             float* cfin, int B, int Tn, int H, int64_t out_sb, int64_t out_st, cudaStream_t s) {
  const ClShape sh = simt_cl_shape(B, K, H);
  if (sh.smem > kSimtSmemMax) {
    set_error("cluster FFMA kernel: shared-memory tile too large");
    return PLSTM_ENOTSUP;
  }
  auto kern = simt_cl_layer_kernel<4>;
  if (sh.nb == 8) kern = simt_cl_layer_kernel<8>;
  if (sh.nb == 16) kern = simt_cl_layer_kernel<16>;
  PLSTM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.smem));
  const int grid = (B + sh.nb - 1) / sh.nb * kClC;
  kern<<<grid, kClThreads, sh.smem, s>>>(xin, K, wih_t, whh_t, bias, lengths, h0, c0, seq_out, hfin, cfin, B, Tn, H,
                                         sh.slices, out_sb, out_st);
  PLSTM_TRY_CUDA(cudaGetLastError());
  return PLSTM_OK;
}

// out[b][t][o] (SEQ) or out[b][o] (LAST) = b_lin[o] + W_lin[o] . h, zero past each length (SEQ).
template <typename T>
__global__ void simt_linear_kernel(const T* __restrict__ hseq, const T* __restrict__ hlast,
                                   const T* __restrict__ wlin, const float* __restrict__ blin,
                                   const int32_t* __restrict__ lengths, T* __restrict__ out, int B,
                                   int Tn, int H, int O, int seq_mode) {
  const int64_t rows = seq_mode ? (int64_t)B * Tn : B;
  const int64_t n = rows * O;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / O;
    const int o = (int)(i % O);
    const int b = seq_mode ? (int)(row / Tn) : (int)row;
    const int t = seq_mode ? (int)(row % Tn) : 0;
    const int len = lengths != nullptr ? min(max(lengths[b], 0), Tn) : Tn;
    float acc = 0.0f;
    if (!seq_mode || t < len) {
      const T* h = seq_mode ? hseq + row * H : hlast + (int64_t)b * H;
      acc = blin[o];
      const T* w = wlin + (int64_t)o * H;
      for (int u = 0; u < H; ++u) acc = fmaf(to_f32(w[u]), to_f32(h[u]), acc);
    }
    out[i] = from_f32<T>(acc);
  }
}

template <typename T>
__global__ void copy_state_kernel(const T* __restrict__ hsrc, const float* __restrict__ csrc,
                                  void* h_n, void* c_n, int c_f32, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (h_n != nullptr) static_cast<T*>(h_n)[i] = hsrc[i];
    if (c_n != nullptr) {
      if (c_f32)
        static_cast<float*>(c_n)[i] = csrc[i];
      else
        static_cast<T*>(c_n)[i] = from_f32<T>(csrc[i]);
    }
  }
}

int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16));
}

template <typename T>
int32_t simt_forward_t(const Problem& p, const void* packed, const void* x, const int32_t* lengths,
                       const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                       cudaStream_t s) {
  const SimtLayout lo = simt_layout(p);
  const SimtWs w = simt_ws(p);
  const char* pk = static_cast<const char*>(packed);
  char* wsb = static_cast<char*>(ws);
  T* seq[2] = {reinterpret_cast<T*>(wsb + w.seq[0]), reinterpret_cast<T*>(wsb + w.seq[1])};
  T* hfin = reinterpret_cast<T*>(wsb + w.hfin);
  float* cfin = reinterpret_cast<float*>(wsb + w.cfin);
  const T* layer_in = static_cast<const T*>(x);
  int K = p.I;
  for (int l = 0; l < p.L; ++l) {
    const bool last = l == p.L - 1;
    T* dst = (last && !p.has_linear()) ? static_cast<T*>(out) : seq[l & 1];
    const T* h0l = h0 ? static_cast<const T*>(h0) + (size_t)l * p.B * p.H : nullptr;
    const T* c0l = c0 ? static_cast<const T*>(c0) + (size_t)l * p.B * p.H : nullptr;
    if (l == 0) profile_begin(s);
    int32_t rc;
    if constexpr (std::is_same<T, float>::value) {
      if (simt_cl_supported(p.dtype, K, p.H, p.route_batch())) {
        rc = launch_simt_cl_layer(layer_in, K, reinterpret_cast<const float*>(pk + lo.wih[l]),
                                  reinterpret_cast<const float*>(pk + lo.whh[l]),
                                  reinterpret_cast<const float*>(pk + lo.bias[l]), lengths, h0l, c0l, dst,
                                  hfin + (size_t)l * p.B * p.H, cfin + (size_t)l * p.B * p.H, p.B, p.T, p.H,
                                  (int64_t)p.T * p.H, p.H, s);
        if (rc != PLSTM_OK) return rc;
        note_launches(1);
        if (l == p.L - 1) profile_end(s);
        layer_in = dst;
        K = p.H;
        continue;
      }
    }
    rc = launch_simt_layer<T>(
        layer_in, K, reinterpret_cast<const T*>(pk + lo.wih[l]), reinterpret_cast<const T*>(pk + lo.whh[l]),
        reinterpret_cast<const float*>(pk + lo.bias[l]), lengths, h0l, c0l, dst, hfin + (size_t)l * p.B * p.H,
        cfin + (size_t)l * p.B * p.H, p.B, p.T, p.H, nullptr, 0, 0, (int64_t)p.T * p.H, p.H, s);
    if (rc != PLSTM_OK) return rc;
    note_launches(1);
    if (l == p.L - 1) profile_end(s);
    layer_in = dst;
    K = p.H;
  }
  if (p.has_linear()) {
    const int seq_mode = p.out_seq() ? 1 : 0;
    const int64_t n = (seq_mode ? (int64_t)p.B * p.T : p.B) * p.O;
    simt_linear_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(
        layer_in, hfin + (size_t)(p.L - 1) * p.B * p.H, reinterpret_cast<const T*>(pk + lo.wlin),
        reinterpret_cast<const float*>(pk + lo.blin), lengths, static_cast<T*>(out), p.B, p.T, p.H,
        p.O, seq_mode);
    PLSTM_TRY_CUDA(cudaGetLastError());
    note_launches(1);
  }
  if (h_n != nullptr || c_n != nullptr) {
    const int64_t n = (int64_t)p.L * p.B * p.H;
    copy_state_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(hfin, cfin, h_n, c_n,
                                                           (p.flags & PLSTM_FLAG_CN_F32) ? 1 : 0, n);
    PLSTM_TRY_CUDA(cudaGetLastError());
    note_launches(1);
  }
  return PLSTM_OK;
}

// ---- hidden update (plstm_hidden_update) --------------------------------------------
struct HuWs {
  size_t whh, bias, seq, total;
};
HuWs hu_ws(const HuProblem& p) {
  HuWs w;
  const size_t es = dtype_size(p.dtype);
  size_t off = kStatusBytes;
  w.whh = off;
  off = align_up(off + align_up(p.H, 4) * 4 * p.H * es, 256);
  w.bias = off;
  off = align_up(off + (size_t)4 * p.H * 4, 256);
  w.seq = off;
  if (!p.write_seq()) off = align_up(off + (size_t)p.B * p.T * p.H * es, 256);
  w.total = off;
  return w;
}

template <typename T>
int32_t simt_hu_t(const HuProblem& p, const void* gate_proj, const void* w_hh, const void* bias, void* h_state,
                  float* c_state, void* out, void* ws, cudaStream_t s) {
  const HuWs w = hu_ws(p);
  char* wsb = static_cast<char*>(ws);
  const int G = 4 * p.H;
  pack_transposed_kernel<<<grid_for((int64_t)G * (p.H + 3), 256), 256, 0, s>>>(w_hh, p.dtype, p.w_layout, G, p.H,
                                                                          wsb + w.whh, p.dtype);
  pack_bias_kernel<<<grid_for(G, 256), 256, 0, s>>>(bias, nullptr, p.dtype, G, reinterpret_cast<float*>(wsb + w.bias));
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(2);
  const bool sm = p.seq_major();
  T* seq = p.write_seq() ? static_cast<T*>(out) : reinterpret_cast<T*>(wsb + w.seq);
  const int64_t out_sb = (p.write_seq() && sm) ? p.H : (int64_t)p.T * p.H;
  const int64_t out_st = (p.write_seq() && sm) ? (int64_t)p.B * p.H : p.H;
  const int64_t gin_sb = sm ? G : (int64_t)p.T * G;
  const int64_t gin_st = sm ? (int64_t)p.B * G : G;
  profile_begin(s);
  const int32_t rc = launch_simt_layer<T>(
      nullptr, 0, nullptr, reinterpret_cast<const T*>(wsb + w.whh), reinterpret_cast<const float*>(wsb + w.bias),
      nullptr, nullptr, nullptr, seq, static_cast<T*>(h_state), c_state, p.B, p.T, p.H,
      static_cast<const T*>(gate_proj), gin_sb, gin_st, out_sb, out_st, s);
  if (rc != PLSTM_OK) return rc;
  profile_end(s);
  note_launches(1);
  if (!p.write_seq())
    PLSTM_TRY_CUDA(cudaMemcpyAsync(out, h_state, (size_t)p.B * p.H * sizeof(T), cudaMemcpyDeviceToDevice, s));
  return PLSTM_OK;
}

}  // namespace

size_t simt_hu_workspace_size(const HuProblem& p) { return hu_ws(p).total; }

int32_t simt_hidden_update(const HuProblem& p, const void* gate_proj, const void* w_hh, const void* bias,
                           void* h_state, float* c_state, void* out, void* ws, cudaStream_t s) {
  switch (p.dtype) {
    case PLSTM_F32:
      return simt_hu_t<float>(p, gate_proj, w_hh, bias, h_state, c_state, out, ws, s);
    case PLSTM_F16:
      return simt_hu_t<__half>(p, gate_proj, w_hh, bias, h_state, c_state, out, ws, s);
    default:
      return simt_hu_t<__nv_bfloat16>(p, gate_proj, w_hh, bias, h_state, c_state, out, ws, s);
  }
}

size_t simt_packed_size(const Problem& p) { return simt_layout(p).total; }
size_t simt_workspace_size(const Problem& p) { return simt_ws(p).total; }

int32_t simt_pack(const Problem& p, int ih_layout, int hh_layout, const void* const* w_ih, const void* const* w_hh,
                  const void* const* b_ih, const void* const* b_hh, const void* w_lin,
                  const void* b_lin, void* packed, cudaStream_t s) {
  const SimtLayout lo = simt_layout(p);
  char* pk = static_cast<char*>(packed);
  const int G = 4 * p.H;
  for (int l = 0; l < p.L; ++l) {
    const int K = l == 0 ? p.I : p.H;
    pack_transposed_kernel<<<grid_for((int64_t)G * (K + 3), 256), 256, 0, s>>>(
        w_ih[l], p.dtype, ih_layout, G, K, pk + lo.wih[l], p.dtype);
    pack_transposed_kernel<<<grid_for((int64_t)G * (p.H + 3), 256), 256, 0, s>>>(
        w_hh[l], p.dtype, hh_layout, G, p.H, pk + lo.whh[l], p.dtype);
    pack_bias_kernel<<<grid_for(G, 256), 256, 0, s>>>(b_ih ? b_ih[l] : nullptr,
                                                       b_hh ? b_hh[l] : nullptr, p.dtype, G,
                                                       reinterpret_cast<float*>(pk + lo.bias[l]));
  }
  if (p.has_linear()) {
    pack_native_kernel<<<grid_for((int64_t)p.O * p.H, 256), 256, 0, s>>>(
        w_lin, p.dtype, PLSTM_W_NATIVE, p.O, p.H, pk + lo.wlin, p.dtype);
    pack_bias_kernel<<<grid_for(p.O, 256), 256, 0, s>>>(b_lin, nullptr, p.dtype, p.O,
                                                         reinterpret_cast<float*>(pk + lo.blin));
    note_launches(2);
  }
  note_launches(3 * p.L);
  PLSTM_TRY_CUDA(cudaGetLastError());
  return PLSTM_OK;
}

int32_t simt_forward(const Problem& p, const void* packed, const void* x, const int32_t* lengths,
                     const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                     cudaStream_t s) {
  switch (p.dtype) {
    case PLSTM_F32:
      return simt_forward_t<float>(p, packed, x, lengths, h0, c0, out, h_n, c_n, ws, s);
    case PLSTM_F16:
      return simt_forward_t<__half>(p, packed, x, lengths, h0, c0, out, h_n, c_n, ws, s);
    default:
      return simt_forward_t<__nv_bfloat16>(p, packed, x, lengths, h0, c0, out, h_n, c_n, ws, s);
  }
}

}  // namespace plstm
