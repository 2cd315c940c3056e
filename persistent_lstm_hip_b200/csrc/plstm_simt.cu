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
//   wih_t[l]  [K_l][4H]  activation type   (K_0 = I, K_l = H)
//   whh_t[l]  [H][4H]    activation type
//   bias[l]   [4H]       f32, b_ih + b_hh summed in f32
// then W_lin [O][H] (activation type) and b_lin [O] (f32).
#include <algorithm>
#include <vector>

#include "plstm_common.cuh"

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
    off = align_up(off + K * G * es, 256);
    lo.whh.push_back(off);
    off = align_up(off + (size_t)p.H * G * es, 256);
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

// dst[k][r] = W[r][k] (transposed to [K][rows]) converted to the activation type.
__global__ void pack_transposed_kernel(const void* src, int src_dtype, int layout, int rows, int K,
                                       void* dst, int dst_dtype) {
  const int64_t n = (int64_t)rows * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i / rows);
    const int r = (int)(i % rows);
    store_any(dst, dst_dtype, i, load_any(src, src_dtype, weight_src_index(layout, rows, K, r, k)));
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

constexpr int kSimtThreads = 256;

// One layer, whole sequence, NB batch rows per CTA.
// xin: layer input [B][T][K] (activation type T).  seq_out[b * out_sb + t * out_st + u].
// gin: optional precomputed input projection added to the gates, gin[b * gin_sb + t * gin_st + r]
// (the hidden-update entry point runs with K = 0 and gin set).
// hfin/cfin: final state of this layer [B][H] (T / f32).
template <typename T, int NB>
__global__ void __launch_bounds__(kSimtThreads)
    simt_layer_kernel(const T* __restrict__ xin, int K, const T* __restrict__ wih_t,
                      const T* __restrict__ whh_t, const float* __restrict__ bias,
                      const int32_t* __restrict__ lengths, const T* __restrict__ h0,
                      const T* __restrict__ c0, T* __restrict__ seq_out, T* __restrict__ hfin,
                      float* __restrict__ cfin, int B, int Tn, int H, const T* __restrict__ gin,
                      int64_t gin_sb, int64_t gin_st, int64_t out_sb, int64_t out_st) {
  extern __shared__ float smem[];
  const int G = 4 * H;
  const int KH = K + H;
  float* xh = smem;                 // [NB][K + H]: x_t then h_{t-1}
  float* gates = xh + NB * KH;      // [NB][4H]
  float* cst = gates + NB * G;      // [NB][H]
  __shared__ int lens[NB];
  const int b0 = blockIdx.x * NB;
  const int tid = threadIdx.x;

  if (tid < NB) {
    const int b = b0 + tid;
    int len = 0;
    if (b < B) len = lengths != nullptr ? min(max(lengths[b], 0), Tn) : Tn;
    lens[tid] = len;
  }
  for (int i = tid; i < NB * H; i += blockDim.x) {
    const int n = i / H, u = i % H, b = b0 + n;
    float hv = 0.0f, cv = 0.0f;
    if (b < B) {
      if (h0 != nullptr) hv = to_f32(h0[(int64_t)b * H + u]);
      if (c0 != nullptr) cv = to_f32(c0[(int64_t)b * H + u]);
    }
    xh[n * KH + K + u] = hv;
    cst[i] = cv;
  }
  __syncthreads();
  int tmax = 0;
#pragma unroll
  for (int n = 0; n < NB; ++n) tmax = max(tmax, lens[n]);

  for (int t = 0; t < tmax; ++t) {
    for (int i = tid; i < NB * K; i += blockDim.x) {
      const int n = i / K, k = i % K, b = b0 + n;
      xh[n * KH + k] = (b < B) ? to_f32(xin[((int64_t)b * Tn + t) * K + k]) : 0.0f;
    }
    __syncthreads();
    for (int r = tid; r < G; r += blockDim.x) {
      float acc[NB];
      const float bv = bias != nullptr ? bias[r] : 0.0f;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        acc[n] = bv;
        if (gin != nullptr && b0 + n < B) acc[n] += to_f32(gin[(int64_t)(b0 + n) * gin_sb + (int64_t)t * gin_st + r]);
      }
      int k = 0;
      for (; k + 4 <= K; k += 4) {
        const float w0 = to_f32(wih_t[(int64_t)(k + 0) * G + r]);
        const float w1 = to_f32(wih_t[(int64_t)(k + 1) * G + r]);
        const float w2 = to_f32(wih_t[(int64_t)(k + 2) * G + r]);
        const float w3 = to_f32(wih_t[(int64_t)(k + 3) * G + r]);
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const float* v = xh + n * KH + k;
          acc[n] = fmaf(w0, v[0], acc[n]);
          acc[n] = fmaf(w1, v[1], acc[n]);
          acc[n] = fmaf(w2, v[2], acc[n]);
          acc[n] = fmaf(w3, v[3], acc[n]);
        }
      }
      for (; k < K; ++k) {
        const float w = to_f32(wih_t[(int64_t)k * G + r]);
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[n] = fmaf(w, xh[n * KH + k], acc[n]);
      }
      int j = 0;
      for (; j + 4 <= H; j += 4) {
        const float w0 = to_f32(whh_t[(int64_t)(j + 0) * G + r]);
        const float w1 = to_f32(whh_t[(int64_t)(j + 1) * G + r]);
        const float w2 = to_f32(whh_t[(int64_t)(j + 2) * G + r]);
        const float w3 = to_f32(whh_t[(int64_t)(j + 3) * G + r]);
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const float* v = xh + n * KH + K + j;
          acc[n] = fmaf(w0, v[0], acc[n]);
          acc[n] = fmaf(w1, v[1], acc[n]);
          acc[n] = fmaf(w2, v[2], acc[n]);
          acc[n] = fmaf(w3, v[3], acc[n]);
        }
      }
      for (; j < H; ++j) {
        const float w = to_f32(whh_t[(int64_t)j * G + r]);
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[n] = fmaf(w, xh[n * KH + K + j], acc[n]);
      }
#pragma unroll
      for (int n = 0; n < NB; ++n) gates[n * G + r] = acc[n];
    }
    __syncthreads();
    for (int i = tid; i < NB * H; i += blockDim.x) {
      const int n = i / H, u = i % H, b = b0 + n;
      const float* g = gates + n * G;
      if (t < lens[n]) {
        const float ig = sigmoid_acc(g[u]);
        const float fg = sigmoid_acc(g[H + u]);
        const float gg = tanh_acc(g[2 * H + u]);
        const float og = sigmoid_acc(g[3 * H + u]);
        const float c = fg * cst[i] + ig * gg;
        cst[i] = c;
        const T hq = from_f32<T>(og * tanh_acc(c));  // h is kept in the activation type
        xh[n * KH + K + u] = to_f32(hq);
        seq_out[(int64_t)b * out_sb + (int64_t)t * out_st + u] = hq;
      } else if (b < B) {
        seq_out[(int64_t)b * out_sb + (int64_t)t * out_st + u] = from_f32<T>(0.0f);
      }
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
      hfin[(int64_t)b * H + u] = from_f32<T>(xh[n * KH + K + u]);
      cfin[(int64_t)b * H + u] = cst[i];
    }
  }
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
  constexpr int NB = 4;
  const int grid = (p.B + NB - 1) / NB;
  const T* layer_in = static_cast<const T*>(x);
  int K = p.I;
  for (int l = 0; l < p.L; ++l) {
    const bool last = l == p.L - 1;
    T* dst = (last && !p.has_linear()) ? static_cast<T*>(out) : seq[l & 1];
    const size_t smem = sizeof(float) * NB * ((size_t)(K + p.H) + 4 * (size_t)p.H + p.H);
    auto kern = simt_layer_kernel<T, NB>;
    PLSTM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const T* h0l = h0 ? static_cast<const T*>(h0) + (size_t)l * p.B * p.H : nullptr;
    const T* c0l = c0 ? static_cast<const T*>(c0) + (size_t)l * p.B * p.H : nullptr;
    if (l == 0) profile_begin(s);
    kern<<<grid, kSimtThreads, smem, s>>>(
        layer_in, K, reinterpret_cast<const T*>(pk + lo.wih[l]),
        reinterpret_cast<const T*>(pk + lo.whh[l]), reinterpret_cast<const float*>(pk + lo.bias[l]),
        lengths, h0l, c0l, dst, hfin + (size_t)l * p.B * p.H, cfin + (size_t)l * p.B * p.H, p.B,
        p.T, p.H, nullptr, 0, 0, (int64_t)p.T * p.H, p.H);
    PLSTM_TRY_CUDA(cudaGetLastError());
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
  off = align_up(off + (size_t)p.H * 4 * p.H * es, 256);
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
  pack_transposed_kernel<<<grid_for((int64_t)G * p.H, 256), 256, 0, s>>>(w_hh, p.dtype, p.w_layout, G, p.H,
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
  constexpr int NB = 4;
  const size_t smem = sizeof(float) * NB * ((size_t)p.H + 4 * (size_t)p.H + p.H);
  auto kern = simt_layer_kernel<T, NB>;
  PLSTM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  profile_begin(s);
  kern<<<(p.B + NB - 1) / NB, kSimtThreads, smem, s>>>(
      nullptr, 0, nullptr, reinterpret_cast<const T*>(wsb + w.whh), reinterpret_cast<const float*>(wsb + w.bias),
      nullptr, nullptr, nullptr, seq, static_cast<T*>(h_state), c_state, p.B, p.T, p.H,
      static_cast<const T*>(gate_proj), gin_sb, gin_st, out_sb, out_st);
  PLSTM_TRY_CUDA(cudaGetLastError());
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
    pack_transposed_kernel<<<grid_for((int64_t)G * K, 256), 256, 0, s>>>(
        w_ih[l], p.dtype, ih_layout, G, K, pk + lo.wih[l], p.dtype);
    pack_transposed_kernel<<<grid_for((int64_t)G * p.H, 256), 256, 0, s>>>(
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
