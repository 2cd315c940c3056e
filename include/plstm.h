/*
 * plstm.h — C ABI of the B200-native persistent LSTM + Linear inference path.
 *
 * This is the drop-in boundary for the fused `nn.LSTM + nn.Linear` forward of
 * mantuoluozk/persistent_lstm_hip.  The reference exposes that path as two
 * pybind11 modules taking torch tensors:
 *   - `persistent_lstm_hip_ext`          (persistent_lstm_hip/csrc/bindings.cpp:154-165)
 *   - `miopen_adaptive_lstm_hip._C`      (miopen_adaptive_lstm_hip/csrc/bindings.cpp:5-78)
 * Every entry point below takes plain device pointers, sizes and a
 * `cudaStream_t` passed as `void*`; no torch type crosses this boundary.  The
 * caller owns every buffer (inputs, outputs, workspace); packed images and
 * workspaces must be 16-byte aligned (cudaMalloc and torch allocations are),
 * else the call returns PLSTM_EINVAL.  Each function only
 * enqueues work on `stream` and returns; device-side failures (a bounded
 * inter-CTA wait that ran out) are recorded in the workspace status word and
 * reported by `plstm_read_status` or, with PLSTM_FLAG_SYNC_CHECK, by the call
 * itself.
 *
 * Return codes are PLSTM_OK or one of the PLSTM_E* values; the message of the
 * last failure on the calling thread is returned by `plstm_last_error()`.
 * Unlike the reference (persistent_lstm_op.cpp:55-70, model.py:656-658), no
 * entry point silently falls back to a CPU implementation.
 */
#ifndef PLSTM_H_
#define PLSTM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PLSTM_API __attribute__((visibility("default")))
#else
#define PLSTM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PLSTM_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------- */
#define PLSTM_OK 0
#define PLSTM_EINVAL 1     /* bad shape, dtype, pointer or flag */
#define PLSTM_ENOTSUP 2    /* valid request this build cannot serve */
#define PLSTM_ETIMEOUT 3   /* a bounded inter-CTA wait gave up (device status) */
#define PLSTM_ECUDA 4      /* a CUDA runtime call failed */
#define PLSTM_EWORKSPACE 5 /* workspace smaller than plstm_workspace_size() */
#define PLSTM_EBOUNDS 6    /* bounds-check build only: an index was outside its buffer (device status; the
                              detail word is the checking site) */

/* ---- element types ------------------------------------------------------ */
#define PLSTM_F32 0
#define PLSTM_F16 1
#define PLSTM_BF16 2

/* ---- weight layouts accepted by plstm_pack ------------------------------ */
/* nn.LSTM native: W[4H][K] row-major (packing.py:45-52 keeps this layout). */
#define PLSTM_W_NATIVE 0
/* transposed: W^T[K][4H] (the `_t` arguments of persistent_lstm_op.cpp:73-124). */
#define PLSTM_W_TRANSPOSED 1
/* k-pair interleaved: [ceil(K/2)][4H][2], odd K zero-padded
 * (`_pack_recurrent_weight_kpairs`, persistent_lstm_hip/model.py:20-27). */
#define PLSTM_W_KPAIR 2
/* MMAC-packed recurrent weight (plstm_hidden_update only, K = H): flat
 * [H/16 unit tiles][H/16 k tiles][16 k][4 unit groups][4 gates][4 units]
 * (`_pack_mmac_weight`, miopen_adaptive_lstm_hip/model.py:259-286). */
#define PLSTM_W_MMAC 3

/* ---- backends ----------------------------------------------------------- */
#define PLSTM_BACKEND_AUTO 0 /* tensor-core wavefront kernel when it applies, else SIMT */
#define PLSTM_BACKEND_SIMT 1 /* generic layer-sequential FFMA kernel (any shape, f32) */
#define PLSTM_BACKEND_TC 2   /* tcgen05 kernels, f16/bf16: H<=128 with L<=8, I<=128, O<=32 (wavefront); else any H<=512, L<=16, I<=128 */

/* ---- flags -------------------------------------------------------------- */
#define PLSTM_FLAG_OUT_SEQ 0x1      /* out is [B][T][O]: Linear on every step, zero past each length */
#define PLSTM_FLAG_OUT_LAST 0x2     /* out is [B][O]: Linear on each row's last valid step */
#define PLSTM_FLAG_NO_LINEAR 0x4    /* out is the last layer's h sequence [B][T][H] (no Linear head) */
#define PLSTM_FLAG_BIAS_SUMMED 0x8  /* b_ih already holds b_ih + b_hh; b_hh must be NULL */
#define PLSTM_FLAG_SYNC_CHECK 0x10  /* synchronise `stream` and turn the device status into the return code */
#define PLSTM_FLAG_CN_F32 0x20      /* c_n is written as f32 instead of the activation type */
/* Duplicate-row elimination: rows with the same identity (x up to the row's
 * length, the length, the row's h0 / c0 in every layer; bit for bit) are
 * computed once and their results copied to every duplicate.  The general
 * form of the reference's uniform-batch shortcut (persistent_lstm_hip/model.py:
 * 493-530).  Synchronises `stream` once to read the distinct-row count, so the
 * call is refused under stream capture. */
#define PLSTM_FLAG_DEDUPE 0x40
#define PLSTM_FLAG_TEST_DROP 0x100  /* fault injection: one producer CTA skips one h hand-off (tests only) */
/* Diagnostics: the tensor-core kernel records SM clock (clock64) timestamps of
 * 8 events for 64 steps starting at T/2, for every CTA of the first cluster,
 * into the last 2L*64*8*8 bytes of the workspace (u64 [2L][64][8]). */
#define PLSTM_FLAG_TRACE 0x200

/* Problem descriptor.  All sizes are element counts. */
typedef struct plstm_desc {
  int32_t batch;       /* B */
  int32_t seq_len;     /* T */
  int32_t input_size;  /* I */
  int32_t hidden_size; /* H */
  int32_t num_layers;  /* L */
  int32_t output_size; /* O (ignored with PLSTM_FLAG_NO_LINEAR) */
  int32_t dtype;       /* PLSTM_F32 / PLSTM_F16 / PLSTM_BF16: x, weights, outputs */
  int32_t w_layout;    /* PLSTM_W_* of w_ih / w_hh given to plstm_pack / plstm_forward */
  int32_t flags;       /* PLSTM_FLAG_* */
  int32_t backend;     /* PLSTM_BACKEND_* */
  int32_t timeout_ms;  /* bound of every inter-CTA wait; 0 = $PLSTM_TIMEOUT_MS, else 2000 ms */
  int32_t device;      /* CUDA device ordinal the pointers live on */
} plstm_desc;

/* ---- library info ------------------------------------------------------- */
PLSTM_API int32_t plstm_abi_version(void);
/* Message of the last failed call on this thread ("" if none). */
PLSTM_API const char* plstm_last_error(void);
/* Backend that plstm_forward would run for `d` (PLSTM_BACKEND_SIMT or _TC). */
PLSTM_API int32_t plstm_select_backend(const plstm_desc* d);

/* ---- packed weights ------------------------------------------------------ */
/* Bytes of the device-side packed weight image for `d`.  Replaces the
 * per-weight-version cache the reference builds in Python
 * (persistent_lstm_hip/model.py:542-582, miopen_adaptive_lstm_hip/model.py:403-430). */
PLSTM_API int32_t plstm_packed_size(const plstm_desc* d, size_t* bytes);
/* Converts w_ih[l], w_hh[l] (layout d->w_layout), biases and the Linear head
 * into the backend's packed image.  b_hh may be NULL with PLSTM_FLAG_BIAS_SUMMED
 * (the reference passes one pre-summed bias, model.py:552-561); biases may be
 * NULL for a bias-free LSTM; w_lin/b_lin are ignored with PLSTM_FLAG_NO_LINEAR. */
PLSTM_API int32_t plstm_pack(const plstm_desc* d, const void* const* w_ih, const void* const* w_hh,
                   const void* const* b_ih, const void* const* b_hh, const void* w_lin,
                   const void* b_lin, void* packed, size_t packed_bytes, void* stream);

/* ---- forward -------------------------------------------------------------- */
/* Scratch bytes plstm_forward_packed needs (plstm_forward needs
 * plstm_workspace_size + plstm_packed_size). */
PLSTM_API int32_t plstm_workspace_size(const plstm_desc* d, size_t* bytes);

/* The hot path.  x[B][T][I]; lengths[B] (int32, device, may be NULL = all T);
 * h0/c0[L][B][H] (may be NULL = zeros); out per the OUT_* flag; h_n/c_n
 * [L][B][H] (may be NULL).  Semantics follow nn.LSTM(batch_first=True) +
 * nn.Linear; with `lengths` they follow pack_padded_sequence: state freezes
 * after each row's length, outputs past it are zero, h_n/c_n are taken at the
 * last valid step. */
PLSTM_API int32_t plstm_forward_packed(const plstm_desc* d, const void* packed, const void* x,
                             const int32_t* lengths, const void* h0, const void* c0, void* out,
                             void* h_n, void* c_n, void* workspace, size_t workspace_bytes,
                             void* stream);
/* Same, packing the weights into the tail of `workspace` first (workspace_bytes
 * >= plstm_workspace_size + plstm_packed_size rounded up to 256). */
PLSTM_API int32_t plstm_forward(const plstm_desc* d, const void* x, const void* const* w_ih,
                      const void* const* w_hh, const void* const* b_ih, const void* const* b_hh,
                      const void* w_lin, const void* b_lin, const int32_t* lengths, const void* h0,
                      const void* c0, void* out, void* h_n, void* c_n, void* workspace,
                      size_t workspace_bytes, void* stream);

/* The forward for callers that cannot hand the library a device workspace
 * (no counterpart in the reference): plugin hosts whose execute hook must not
 * allocate device memory, and programs on a fixed device-memory budget after
 * start-up.  Same contract as plstm_forward_packed for the f16 / bf16
 * tensor-core path, but the scratch comes from a 24 MiB array the library
 * keeps on every device it is loaded on; it allocates nothing.  Problems that
 * need more scratch (plstm_workspace_size) are rejected with PLSTM_EINVAL.
 * The first call on a device looks up that array's device address (make it
 * before any stream capture).  All calls share the array: calls whose GPU work
 * overlaps race and must be serialised by the caller. */
PLSTM_API int32_t plstm_forward_packed_noalloc(const plstm_desc* d, const void* packed, const void* x,
                                               const int32_t* lengths, const void* h0, const void* c0,
                                               void* out, void* h_n, void* c_n, void* stream);

/* Groups identical rows as PLSTM_FLAG_DEDUPE does, without running the
 * forward (the generalisation of the reference's uniform-batch check,
 * persistent_lstm_hip/model.py:493-520).  row_map[B] (device) receives each
 * row's distinct-row index in 0..count-1, unique_index[B] (device) in its
 * first *count entries the first row of each distinct row, ascending; *count
 * (host) the number of distinct rows.  Synchronises `stream`; refused under
 * stream capture.  The workspace needs plstm_unique_rows_workspace_size bytes. */
PLSTM_API int32_t plstm_unique_rows_workspace_size(const plstm_desc* d, size_t* bytes);
PLSTM_API int32_t plstm_unique_rows(const plstm_desc* d, const void* x, const int32_t* lengths, const void* h0,
                                    const void* c0, int32_t* row_map, int32_t* unique_index, int32_t* count,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Reads (and clears) the device status word the kernels of the last forward
 * using `workspace` left, synchronising `stream`.  *status receives PLSTM_OK
 * or PLSTM_ETIMEOUT; *detail the first failing (cta << 16 | step & 0xffff). */
PLSTM_API int32_t plstm_read_status(const void* workspace, void* stream, int32_t* status, int32_t* detail);

/* ---- entry points of `persistent_lstm_hip_ext` ------------------------------
 * The fixed 4-layer regressor calls (x[B][T][I] f16 in, out[B][O] f16).  Each
 * takes the 13 LSTM tensors in the reference's order (W_ih, W_hh, pre-summed
 * bias per layer) plus the Linear head, and a caller workspace of
 * plstm_ref4_workspace_size() bytes.  H and O are read from the arguments the
 * reference derives them from; I from x. */
PLSTM_API int32_t plstm_ref4_workspace_size(int32_t batch, int32_t seq_len, int32_t input_size,
                                  int32_t hidden_size, int32_t output_size, size_t* bytes);

/* persistent_lstm4_forward (bindings.cpp:155; persistent_lstm_op.cpp:15-71):
 * native [4H][K] weights. */
PLSTM_API int32_t plstm_persistent_lstm4_forward(const void* x, int32_t batch, int32_t seq_len,
                                       int32_t input_size, int32_t hidden_size,
                                       int32_t output_size, const void* const* w_ih4,
                                       const void* const* w_hh4, const void* const* bias4,
                                       const void* w_lin, const void* b_lin, void* out,
                                       void* workspace, size_t workspace_bytes, void* stream);
/* persistent_lstm4_forward_packed (bindings.cpp:156; persistent_lstm_op.cpp:73-124):
 * transposed [K][4H] weights. */
PLSTM_API int32_t plstm_persistent_lstm4_forward_packed(const void* x, int32_t batch, int32_t seq_len,
                                              int32_t input_size, int32_t hidden_size,
                                              int32_t output_size, const void* const* w_ih4_t,
                                              const void* const* w_hh4_t, const void* const* bias4,
                                              const void* w_lin, const void* b_lin, void* out,
                                              void* workspace, size_t workspace_bytes,
                                              void* stream);
/* persistent_lstm4_forward_interleaved (bindings.cpp:157; persistent_lstm_op.cpp:126-186):
 * k-pair packed W_ih and W_hh. */
PLSTM_API int32_t plstm_persistent_lstm4_forward_interleaved(
    const void* x, int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
    int32_t output_size, const void* const* w_ih4_kpair, const void* const* w_hh4_kpair,
    const void* const* bias4, const void* w_lin, const void* b_lin, void* out, void* workspace,
    size_t workspace_bytes, void* stream);
/* persistent_lstm4_forward_monolithic (bindings.cpp:162; persistent_lstm_op.cpp:250-310):
 * k-pair packed W_ih and W_hh, all layers in one kernel. */
PLSTM_API int32_t plstm_persistent_lstm4_forward_monolithic(
    const void* x, int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
    int32_t output_size, const void* const* w_ih4_kpair, const void* const* w_hh4_kpair,
    const void* const* bias4, const void* w_lin, const void* b_lin, void* out, void* workspace,
    size_t workspace_bytes, void* stream);
/* persistent_lstm4_forward_projected (bindings.cpp:158; persistent_lstm_op.cpp:188-248):
 * native W_ih, k-pair packed W_hh.  Also serves
 * persistent_lstm4_forward_projected_uniform{,_p4,_p8} (bindings.cpp:159-161,
 * persistent_lstm_hip.cu:2399-2821), whose `virtual_batch_size` only chose how
 * many redundant blocks the DCU kernel ran and has no meaning here. */
PLSTM_API int32_t plstm_persistent_lstm4_forward_projected(
    const void* x, int32_t batch, int32_t seq_len, int32_t input_size, int32_t hidden_size,
    int32_t output_size, const void* const* w_ih4, const void* const* w_hh4_kpair,
    const void* const* bias4, const void* w_lin, const void* b_lin, void* out, void* workspace,
    size_t workspace_bytes, void* stream);
/* persistent_lstm_regressor_forward_generic_projected (bindings.cpp:163;
 * persistent_lstm_hip.cu:2923-3181): any L, native weights, pre-summed bias. */
PLSTM_API int32_t plstm_regressor_forward_generic(const void* x, int32_t batch, int32_t seq_len,
                                        int32_t input_size, int32_t hidden_size,
                                        int32_t num_layers, int32_t output_size,
                                        const void* const* w_ih, const void* const* w_hh,
                                        const void* const* bias, const void* w_lin,
                                        const void* b_lin, void* out, void* workspace,
                                        size_t workspace_bytes, void* stream);
/* repeat_first_row (bindings.cpp:164; persistent_lstm_hip.cu:1684-1809):
 * output[r][c] = input[0][c] for r < out_rows. */
PLSTM_API int32_t plstm_repeat_first_row(const void* input, int32_t cols, int32_t out_rows, int32_t dtype,
                               void* output, void* stream);

/* ---- entry points of `miopen_adaptive_lstm_hip._C` ------------------------- */
/* adaptive_lstm_input_gemm_forward_workspace (bindings.cpp:38-41;
 * adaptive_lstm_hip.cu:389-433, 2355-2385): gate[M][N] = x[M][K] . w_t[K][N]
 * (no bias), f16 or bf16 in and out, f32 accumulation, on tcgen05 tensor cores. */
PLSTM_API int32_t plstm_input_gemm(const void* x, int32_t m, int32_t k, const void* w_t, int32_t n,
                         int32_t dtype, void* gate, void* stream);

/* Hidden update: the LSTM recurrence over precomputed input projections, from
 * h = c = 0.  For every row b and step t:
 *   gates = gate_proj[b, t] + bias + W_hh . h_{t-1}   (gate order i, f, g, o)
 *   c_t = sigmoid(f) c_{t-1} + sigmoid(i) tanh(g),  h_t = sigmoid(o) tanh(c_t)
 * Replaces every hidden-update function of `miopen_adaptive_lstm_hip._C`
 * (bindings.cpp:6-36, 42-78; adaptive_lstm_hip.h:5-170: the generic, partitioned,
 * cached, GEMM-scan, gate-accumulate, seq-major, persistent and MMAC-packed
 * variants all compute this).
 *   gate_proj [B][T][4H] (or [T][B][4H] with PLSTM_HU_SEQ_MAJOR), activation type
 *   w_hh      [4H][H] (PLSTM_W_NATIVE), [H][4H] (PLSTM_W_TRANSPOSED) or PLSTM_W_MMAC
 *   bias      [4H] activation type, or NULL
 *   h_state   [B][H] activation type, c_state [B][H] f32: the final state
 *   out       h sequence [B][T][H] ([T][B][H] with PLSTM_HU_SEQ_MAJOR) with
 *             PLSTM_HU_WRITE_SEQUENCE, else the final h [B][H]
 * f16 / bf16 with H = 128, 256 or 512 run the tcgen05 cluster recurrence; other
 * sizes and f32 run the FFMA kernel.  The workspace is caller-owned
 * (plstm_hidden_update_workspace_size). */
#define PLSTM_HU_SEQ_MAJOR 0x1
#define PLSTM_HU_WRITE_SEQUENCE 0x2
PLSTM_API int32_t plstm_hidden_update_workspace_size(int32_t batch, int32_t seq_len, int32_t hidden, int32_t dtype,
                                           int32_t flags, int32_t device, size_t* bytes);
PLSTM_API int32_t plstm_hidden_update(const void* gate_proj, int32_t batch, int32_t seq_len, int32_t hidden,
                            const void* w_hh, int32_t w_layout, const void* bias, int32_t dtype, int32_t flags,
                            void* h_state, float* c_state, void* out, void* workspace, size_t workspace_bytes,
                            void* stream);

/* ---- instrumentation (no counterpart in the reference beyond its
 * MIOPEN_ADAPTIVE_LSTM_PROFILE per-layer CUDA-event timings,
 * miopen_adaptive_lstm_hip/model.py:685-690, 1025-1052) ----------------------- */
/* Number of kernels this library has launched in this process. */
PLSTM_API int64_t plstm_launch_count(void);
/* enable != 0: every forward records CUDA events around its recurrent kernel
 * (the dominant one) on the caller's stream. */
PLSTM_API int32_t plstm_profile(int32_t enable);
/* Synchronises on the recorded events and returns the summed recurrent-kernel
 * time (ms) and the number of timed launches since the last read; clears them. */
PLSTM_API int32_t plstm_profile_read(float* ms, int32_t* launches);

/* ---- diagnostics ------------------------------------------------------------ */
/* Hardware self-check used by the test suite (no counterpart in the
 * reference): writes a known pattern into tensor memory and reads it back with
 * the tcgen05.ld shapes the wavefront kernel relies on.  out must hold
 * 128 * 24 uint32 (device memory): for thread (warp w, lane t), out[(32w+t)*24 + i]
 * = registers of ld.16x256b.x2 at lane 32w (i < 8), at lane 32w+16 (8 <= i < 16)
 * and of ld.32x32b.x8 at column 8 (16 <= i < 24); each value is
 * (tmem lane << 8 | column). */
PLSTM_API int32_t plstm_diag_tmem_layout(uint32_t* out, void* stream);

/* Dependent-step latency probe (no counterpart in the reference; its serial
 * per-step loop is persistent_lstm_hip.cu:493-558): one cluster of two CTAs runs
 * the wavefront kernel's per-step dependency chain alone for `steps` steps of a
 * `rows`-row (16 or 32) slot: the sibling's h lands, 8 tcgen05 MMAs over it
 * (two M = 128 tiles x K = 64) and their commit, one tcgen05.ld, the kernel's gate
 * math, h written to shared memory and one bulk copy of this CTA's 64 units into
 * the sibling.  out (device, 16 uint64) receives [0] status (0 ok, 1 a bounded
 * wait gave up), [1] SM cycles over [2] steps (from steps / 4 on), [3..8] summed
 * cycles of the phases landed -> commit issued -> accumulator seen -> loaded ->
 * h written -> copy issued -> next h landed.  The latency floor of the roofline.
 * `variant` 0 runs the chain as the kernel does; its bits select alternatives
 * (1: spin on mbarrier.test_wait for the sibling's h, 2: spin for the
 * accumulator, 4: hand-off by st.async 16-byte stores from all compute threads,
 * 8: the two tiles' accumulators loaded one after the other under the gate math). */
PLSTM_API int32_t plstm_diag_step_latency(int32_t rows, int32_t steps, int32_t variant, uint64_t* out,
                                          int32_t timeout_ms, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PLSTM_H_ */
