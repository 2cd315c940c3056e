// plstm_dedupe.cu — duplicate-row elimination for the forward.
//
// The reference has one special case of this: when every row of x equals the
// first, it runs a single sequence and broadcasts the result
// (persistent_lstm_hip/model.py:493-530, the uniform kernels of
// persistent_lstm_hip.cu:2399-2821).  Here any set of identical rows is
// found on the device and computed once:
//
//   1. row_hash_kernel   one CTA per row: a 64-bit hash of the row's identity
//                        (x up to the row's length, the length, its h0 / c0
//                        rows), inserted into an open-addressing table that
//                        keeps the smallest row index per hash (atomicMin);
//   2. row_rep_kernel    one CTA per row: looks its hash up and compares the
//                        row with the table's row element by element, so a
//                        hash collision never merges different rows;
//   3. row_compact_kernel one CTA: deterministic scan giving each distinct row
//                        (its representative = the first occurrence) a dense
//                        index, the list of representatives and the row map;
//   4. the forward on the distinct rows, gathered with copy_rows_kernel, and
//      the results scattered back to every row with the same kernel.
//
// The distinct count decides the inner forward's batch, so the host reads it
// once (one stream synchronisation), as the reference's torch.equal check
// does.  Rows are distinct or not bit for bit: +0 and -0, or two NaN payloads,
// count as different, which only costs work, never correctness.
//
// The hash mixes each 16-bit unit with its position through the SplitMix64
// finaliser (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) and sums the mixed values.
#include <climits>
#include <cstring>
#include <string>

#include "plstm_common.cuh"

namespace plstm {
namespace {

constexpr int kDedupeThreads = 256;
constexpr int kCompactThreads = 1024;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// The rows' identity: x[B][T][I] and, optionally, lengths[B], h0/c0[L][B][H];
// every element size is a multiple of 16 bits, so rows are read as u16 units.
struct RowSet {
  const uint16_t* x;
  const int32_t* lengths;
  const uint16_t* h0;
  const uint16_t* c0;
  int64_t x_row;   // u16 units of one x row (T * I * elem / 2)
  int64_t x_step;  // u16 units of one time step (I * elem / 2)
  int64_t s_row;   // u16 units of one h0 / c0 row (H * elem / 2)
  int B, T, L;
};

__device__ __forceinline__ int row_len(const RowSet& a, int b) {
  if (a.lengths == nullptr) return a.T;
  return min(max(a.lengths[b], 0), a.T);
}

__device__ __forceinline__ uint64_t block_sum_u64(uint64_t v, uint64_t* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  uint64_t s = 0;
  if (threadIdx.x == 0)
    for (int i = 0; i < nw; ++i) s += red[i];
  return s;  // valid in thread 0
}

__global__ void __launch_bounds__(kDedupeThreads)
    row_hash_kernel(RowSet a, unsigned long long* keys, int* vals, uint32_t mask, uint64_t* hash) {
  __shared__ uint64_t red[kDedupeThreads / 32];
  const int b = blockIdx.x;
  const int len = row_len(a, b);
  const uint16_t* xr = a.x + (int64_t)b * a.x_row;
  const int64_t n = (int64_t)len * a.x_step;
  uint64_t s = 0;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) s += mix64(((uint64_t)j << 16) ^ xr[j]);
  if (a.h0 != nullptr) {
    for (int l = 0; l < a.L; ++l) {
      const int64_t off = ((int64_t)l * a.B + b) * a.s_row;
      for (int64_t j = threadIdx.x; j < a.s_row; j += blockDim.x) {
        const uint64_t pos = ((uint64_t)l * a.s_row + j) << 17;
        s += mix64((1ull << 62) ^ pos ^ a.h0[off + j]);
        s += mix64((1ull << 61) ^ pos ^ a.c0[off + j]);
      }
    }
  }
  s = block_sum_u64(s, red);
  if (threadIdx.x != 0) return;
  uint64_t h = mix64(s ^ mix64(0x9e3779b97f4a7c15ull + (uint64_t)len));
  if (h == 0) h = 1;  // 0 marks an empty table slot
  hash[b] = h;
  uint32_t slot = (uint32_t)h & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe) {  // the table has more slots than rows
    const unsigned long long prev = atomicCAS(&keys[slot], 0ull, (unsigned long long)h);
    if (prev == 0ull || prev == (unsigned long long)h) {
      atomicMin(&vals[slot], b);
      return;
    }
    slot = (slot + 1) & mask;
  }
}

__global__ void __launch_bounds__(kDedupeThreads)
    row_rep_kernel(RowSet a, const unsigned long long* keys, const int* vals, uint32_t mask,
                   const uint64_t* hash, int* rep) {
  const int b = blockIdx.x;
  const unsigned long long h = hash[b];
  uint32_t slot = (uint32_t)h & mask;
  int cand = b;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    if (keys[slot] == h) {
      cand = vals[slot];
      break;
    }
    slot = (slot + 1) & mask;
  }
  if (cand == b || cand < 0 || cand >= a.B) {
    if (threadIdx.x == 0) rep[b] = b;
    return;
  }
  const int len = row_len(a, b);
  int same = len == row_len(a, cand);
  if (same) {
    const uint16_t* xb = a.x + (int64_t)b * a.x_row;
    const uint16_t* xc = a.x + (int64_t)cand * a.x_row;
    const int64_t n = (int64_t)len * a.x_step;
    for (int64_t j = threadIdx.x; j < n && same; j += blockDim.x) same = xb[j] == xc[j];
    if (a.h0 != nullptr) {
      for (int l = 0; l < a.L && same; ++l) {
        const int64_t ob = ((int64_t)l * a.B + b) * a.s_row, oc = ((int64_t)l * a.B + cand) * a.s_row;
        for (int64_t j = threadIdx.x; j < a.s_row && same; j += blockDim.x)
          same = a.h0[ob + j] == a.h0[oc + j] && a.c0[ob + j] == a.c0[oc + j];
      }
    }
  }
  same = __syncthreads_and(same);
  if (threadIdx.x == 0) rep[b] = same ? cand : b;
}

// One CTA: representatives (rep[b] == b) get dense indices in row order.
// pos[] holds them; row_map[b] = pos[rep[b]]; unique_index[0..count) lists the
// representatives ascending.
__global__ void __launch_bounds__(kCompactThreads)
    row_compact_kernel(const int* rep, int B, int* pos, int* row_map, int* unique_index, int* count) {
  __shared__ int warp_tot[kCompactThreads / 32];
  const int t = threadIdx.x;
  const int chunk = (B + kCompactThreads - 1) / kCompactThreads;
  const int lo = min(B, t * chunk), hi = min(B, lo + chunk);
  int n = 0;
  for (int i = lo; i < hi; ++i) n += rep[i] == i;
  // Exclusive scan of n over the CTA.
  int incl = n;
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if ((t & 31) >= o) incl += v;
  }
  if ((t & 31) == 31) warp_tot[t >> 5] = incl;
  __syncthreads();
  if (t < 32) {
    int w = warp_tot[t];
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (t >= o) w += v;
    }
    warp_tot[t] = w;  // inclusive over warps
  }
  __syncthreads();
  int off = incl - n + ((t >> 5) > 0 ? warp_tot[(t >> 5) - 1] : 0);
  for (int i = lo; i < hi; ++i) {
    if (rep[i] == i) {
      pos[i] = off;
      unique_index[off] = i;
      ++off;
    }
  }
  if (t == kCompactThreads - 1) *count = warp_tot[31];
  __syncthreads();
  for (int i = lo; i < hi; ++i) row_map[i] = pos[rep[i]];
}

// dst row r of group g <- src row idx[r] of group g; rows are `units` U wide.
template <typename U>
__global__ void copy_rows_kernel(U* __restrict__ dst, const U* __restrict__ src, const int* __restrict__ idx,
                                 int64_t units, int64_t src_group_rows, int64_t dst_group_rows) {
  const int64_t r = blockIdx.x, g = blockIdx.y;
  const U* s = src + (g * src_group_rows + idx[r]) * units;
  U* d = dst + (g * dst_group_rows + r) * units;
  for (int64_t j = threadIdx.x; j < units; j += blockDim.x) d[j] = s[j];
}

int32_t copy_rows(void* dst, const void* src, const int* idx, int nrows, size_t row_bytes, int groups,
                  int64_t src_group_rows, int64_t dst_group_rows, cudaStream_t s) {
  if (nrows == 0 || row_bytes == 0 || groups == 0) return PLSTM_OK;
  const uintptr_t al = (uintptr_t)dst | (uintptr_t)src | (uintptr_t)row_bytes;
  const dim3 grid((unsigned)nrows, (unsigned)groups);
  const int thr = 128;
  if (al % 16 == 0)
    copy_rows_kernel<uint4><<<grid, thr, 0, s>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), idx,
                                                 (int64_t)(row_bytes / 16), src_group_rows, dst_group_rows);
  else if (al % 8 == 0)
    copy_rows_kernel<uint2><<<grid, thr, 0, s>>>(static_cast<uint2*>(dst), static_cast<const uint2*>(src), idx,
                                                 (int64_t)(row_bytes / 8), src_group_rows, dst_group_rows);
  else if (al % 4 == 0)
    copy_rows_kernel<uint32_t><<<grid, thr, 0, s>>>(static_cast<uint32_t*>(dst), static_cast<const uint32_t*>(src),
                                                    idx, (int64_t)(row_bytes / 4), src_group_rows, dst_group_rows);
  else
    copy_rows_kernel<uint16_t><<<grid, thr, 0, s>>>(static_cast<uint16_t*>(dst), static_cast<const uint16_t*>(src),
                                                    idx, (int64_t)(row_bytes / 2), src_group_rows, dst_group_rows);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(1);
  return PLSTM_OK;
}

uint32_t table_slots(int B) {
  uint32_t n = 64;
  while (n < 2u * (uint32_t)B) n <<= 1;
  return n;
}

size_t out_row_bytes(const Problem& p) {
  const size_t es = dtype_size(p.dtype);
  if (!p.has_linear()) return (size_t)p.T * p.H * es;
  return p.out_seq() ? (size_t)p.T * p.O * es : (size_t)p.O * es;
}

size_t cn_elem(const Problem& p) { return (p.flags & PLSTM_FLAG_CN_F32) ? 4 : dtype_size(p.dtype); }

// Scratch of the row grouping and of the distinct-row copies, all 256-aligned.
struct DedupeWs {
  size_t keys, vals, hash, rep, pos, map, uniq, count, x, len, h0, c0, out, hn, cn, total;
};

DedupeWs dedupe_layout(const Problem& p, bool copies) {
  DedupeWs w = {};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  const size_t B = (size_t)p.B, es = dtype_size(p.dtype), slots = table_slots(p.B);
  const size_t state = (size_t)p.L * B * p.H;
  w.keys = take(slots * 8);
  w.vals = take(slots * 4);
  w.hash = take(B * 8);
  w.rep = take(B * 4);
  w.pos = take(B * 4);
  w.map = take(B * 4);
  w.uniq = take(B * 4);
  w.count = take(16);
  if (copies) {
    w.x = take(B * p.T * p.I * es);
    w.len = take(B * 4);
    w.h0 = take(state * es);
    w.c0 = take(state * es);
    w.out = take(B * out_row_bytes(p));
    w.hn = take(state * es);
    w.cn = take(state * cn_elem(p));
  }
  w.total = o;
  return w;
}

// Groups the rows; writes row_map / unique_index (device, B entries) and the
// distinct count (host).  `scratch` holds dedupe_layout(p, false).total bytes.
int32_t group_rows(const Problem& p, const void* x, const int32_t* lengths, const void* h0, const void* c0,
                   int* row_map, int* unique_index, int* count, char* scratch, cudaStream_t s) {
  const DedupeWs w = dedupe_layout(p, false);
  const uint32_t slots = table_slots(p.B);
  auto* keys = reinterpret_cast<unsigned long long*>(scratch + w.keys);
  auto* vals = reinterpret_cast<int*>(scratch + w.vals);
  auto* hash = reinterpret_cast<uint64_t*>(scratch + w.hash);
  auto* rep = reinterpret_cast<int*>(scratch + w.rep);
  auto* pos = reinterpret_cast<int*>(scratch + w.pos);
  auto* dcount = reinterpret_cast<int*>(scratch + w.count);
  PLSTM_TRY_CUDA(cudaMemsetAsync(keys, 0, (size_t)slots * 8, s));
  PLSTM_TRY_CUDA(cudaMemsetAsync(vals, 0x7f, (size_t)slots * 4, s));  // 0x7f7f7f7f: above every row index
  RowSet a;
  a.x = static_cast<const uint16_t*>(x);
  a.lengths = lengths;
  a.h0 = static_cast<const uint16_t*>(h0);
  a.c0 = static_cast<const uint16_t*>(c0);
  const int64_t eu = (int64_t)dtype_size(p.dtype) / 2;
  a.x_row = (int64_t)p.T * p.I * eu;
  a.x_step = (int64_t)p.I * eu;
  a.s_row = (int64_t)p.H * eu;
  a.B = p.B;
  a.T = p.T;
  a.L = p.L;
  row_hash_kernel<<<p.B, kDedupeThreads, 0, s>>>(a, keys, vals, slots - 1, hash);
  PLSTM_TRY_CUDA(cudaGetLastError());
  row_rep_kernel<<<p.B, kDedupeThreads, 0, s>>>(a, keys, vals, slots - 1, hash, rep);
  PLSTM_TRY_CUDA(cudaGetLastError());
  row_compact_kernel<<<1, kCompactThreads, 0, s>>>(rep, p.B, pos, row_map, unique_index, dcount);
  PLSTM_TRY_CUDA(cudaGetLastError());
  note_launches(3);
  int host = 0;
  PLSTM_TRY_CUDA(cudaMemcpyAsync(&host, dcount, sizeof(int), cudaMemcpyDeviceToHost, s));
  PLSTM_TRY_CUDA(cudaStreamSynchronize(s));
  *count = host;
  return PLSTM_OK;
}

int32_t refuse_capture(cudaStream_t s, const char* what) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  PLSTM_TRY_CUDA(cudaStreamIsCapturing(s, &st));
  if (st != cudaStreamCaptureStatusNone) {
    set_error(std::string(what) + " reads the distinct-row count on the host and cannot run under stream capture");
    return PLSTM_EINVAL;
  }
  return PLSTM_OK;
}

}  // namespace

int32_t dedupe_stream_ok(cudaStream_t s) { return refuse_capture(s, "PLSTM_FLAG_DEDUPE"); }

size_t unique_rows_scratch_size(const Problem& p) { return dedupe_layout(p, false).total; }

size_t dedupe_scratch_size(const Problem& p) { return dedupe_layout(p, true).total; }

int32_t unique_rows(const Problem& p, const void* x, const int32_t* lengths, const void* h0, const void* c0,
                    int* row_map, int* unique_index, int* count, void* scratch, cudaStream_t s) {
  int32_t rc = refuse_capture(s, "plstm_unique_rows");
  if (rc != PLSTM_OK) return rc;
  return group_rows(p, x, lengths, h0, c0, row_map, unique_index, count, static_cast<char*>(scratch), s);
}

int32_t dedupe_forward(const Problem& p, const DedupeInner& inner, const void* x, const int32_t* lengths,
                       const void* h0, const void* c0, void* out, void* h_n, void* c_n, void* ws,
                       size_t inner_ws_bytes, cudaStream_t s) {
  int32_t rc = refuse_capture(s, "PLSTM_FLAG_DEDUPE");
  if (rc != PLSTM_OK) return rc;
  char* scratch = static_cast<char*>(ws) + align_up(inner_ws_bytes, 256);
  const DedupeWs w = dedupe_layout(p, true);
  int* row_map = reinterpret_cast<int*>(scratch + w.map);
  int* uniq = reinterpret_cast<int*>(scratch + w.uniq);
  int U = 0;
  if ((rc = group_rows(p, x, lengths, h0, c0, row_map, uniq, &U, scratch, s)) != PLSTM_OK) return rc;
  Problem q = p;
  q.flags &= ~PLSTM_FLAG_DEDUPE;
  if (U == p.B) return inner.run(inner.ctx, q, x, lengths, h0, c0, out, h_n, c_n, ws, s);
  if (U <= 0 || U > p.B) {
    set_error("duplicate-row grouping returned an impossible distinct count " + std::to_string(U));
    return PLSTM_ECUDA;
  }
  q.route_B = p.route_batch();
  q.B = U;
  const size_t es = dtype_size(p.dtype);
  const size_t srow = (size_t)p.H * es, crow = (size_t)p.H * cn_elem(p);
  void* xu = scratch + w.x;
  int32_t* lu = lengths ? reinterpret_cast<int32_t*>(scratch + w.len) : nullptr;
  void* h0u = h0 ? scratch + w.h0 : nullptr;
  void* c0u = c0 ? scratch + w.c0 : nullptr;
  void* ou = scratch + w.out;
  void* hnu = h_n ? scratch + w.hn : nullptr;
  void* cnu = c_n ? scratch + w.cn : nullptr;
  if (p.T > 0 && (rc = copy_rows(xu, x, uniq, U, (size_t)p.T * p.I * es, 1, 0, 0, s)) != PLSTM_OK) return rc;
  if (lu && (rc = copy_rows(lu, lengths, uniq, U, 4, 1, 0, 0, s)) != PLSTM_OK) return rc;
  if (h0u && (rc = copy_rows(h0u, h0, uniq, U, srow, p.L, p.B, U, s)) != PLSTM_OK) return rc;
  if (c0u && (rc = copy_rows(c0u, c0, uniq, U, srow, p.L, p.B, U, s)) != PLSTM_OK) return rc;
  if ((rc = inner.run(inner.ctx, q, xu, lu, h0u, c0u, ou, hnu, cnu, ws, s)) != PLSTM_OK) return rc;
  if ((rc = copy_rows(out, ou, row_map, p.B, out_row_bytes(p), 1, 0, 0, s)) != PLSTM_OK) return rc;
  if (hnu && (rc = copy_rows(h_n, hnu, row_map, p.B, srow, p.L, U, p.B, s)) != PLSTM_OK) return rc;
  if (cnu && (rc = copy_rows(c_n, cnu, row_map, p.B, crow, p.L, U, p.B, s)) != PLSTM_OK) return rc;
  return PLSTM_OK;
}

}  // namespace plstm
