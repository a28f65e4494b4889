/*
 * bnbq.h -- C ABI of the B200 (sm_100a) blockwise-quantization kernels.
 *
 * This is the boundary that replaces the reference's `cutejax.call(...)`
 * custom calls (bnb_jax 0.2.0, src/bnb_jax/kernels/{quantize,dequantize,gemv}.py).
 * Every entry point takes raw device pointers, element counts and a CUDA
 * stream (as `void*`, i.e. a `cudaStream_t`), enqueues its kernels on that
 * stream and returns immediately: no allocation, no host synchronisation.
 * The caller owns every buffer. Outputs are written at their exact sizes
 * (ceil(n/2) NF4 bytes, n 8-bit bytes, ceil(n/bs) absmax values, n decoded
 * elements): the reference's host-side pad and slice copies do not exist here.
 *
 * Numerics follow bitsandbytes' fast-math arithmetic exactly as the reference
 * restates it (src/bnb_jax/kernels/_ptx.py:15-33): mul.ftz.f32, abs/max.ftz,
 * rcp.approx.ftz.f32, round-to-nearest conversions. Codes, absmax and decoded
 * values are bitwise those of the reference.
 *
 * Pointer alignment: element buffers (x, out, y) and code buffers must be
 * 16-byte aligned; absmax / codebook pointers 4-byte aligned. A misaligned
 * pointer returns BNBQ_ERR_MISALIGNED without launching anything.
 *
 * Return value: BNBQ_OK (0) or a negative status; bnbq_error_string() names it.
 * Nothing here calls exit(), traps on the device, or leaves work half-queued
 * on an argument error.
 */
#ifndef BNBQ_H_
#define BNBQ_H_

#include <stdint.h>

#if defined(__GNUC__)
#define BNBQ_API __attribute__((visibility("default")))
#else
#define BNBQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types (the reference's _DTYPES, kernels/quantize.py:35) */
enum bnbq_dtype { BNBQ_F32 = 0, BNBQ_F16 = 1, BNBQ_BF16 = 2 };

enum bnbq_status {
  BNBQ_OK = 0,
  BNBQ_ERR_INVALID = -1,     /* bad size / blocksize / null pointer (ValueError in Python) */
  BNBQ_ERR_UNSUPPORTED = -2, /* dtype or shape outside what the kernel implements (NotImplementedError) */
  BNBQ_ERR_MISALIGNED = -3,  /* a pointer breaks the alignment rule above */
  BNBQ_ERR_CUDA = -4,        /* a CUDA runtime call or launch failed */
  BNBQ_ERR_DEVICE = -5,      /* the current device is not sm_100 */
  BNBQ_ERR_TOO_LARGE = -6    /* more than a no-allocation entry point's fixed scratch holds */
};

/* Largest batch the CUDA-core GEMV handles; bnbq_matmul_nf4 uses the tcgen05
 * GEMM above it. Same value as the reference's GEMV_MAX_M (kernels/gemv.py:42). */
#define BNBQ_GEMV_MAX_M 20

/* ---------------------------------------------------------------- quantize */

/* NF4 blockwise quantize of n elements of `dtype` at `x`.
 * q: ceil(n/2) bytes, two codes per byte, high nibble first; absmax: ceil(n/bs) floats.
 * blocksize: power of two, 8 <= bs <= 4096 (the reference accepts any power of
 * two >= 8, kernels/dequantize.py:87-90; bitsandbytes uses 32..4096).
 * Replaces: cutejax.call(_quant_launch, ..., nf4=True) at kernels/quantize.py:226-233
 * behind quantize_nf4 (kernels/quantize.py:238-248). A partial last block reads
 * as zero-padded, as the reference's jnp.pad does (kernels/quantize.py:221-225). */
BNBQ_API int bnbq_quantize_nf4(int dtype, const void* x, int64_t n, int32_t blocksize,
                      uint8_t* q, float* absmax, void* stream);

/* 8-bit blockwise quantize with a 256-entry float32 codebook `code` (device).
 * q: n bytes; absmax: ceil(n/bs) floats. blocksize: power of two, 8..4096.
 * `offset` (device, one float, may be NULL): when given, every element is first
 * replaced by fl32(x - *offset) -- the centring step of double quantization,
 * array.py:200-201 (`quantize(absmax - offset, "8bit", 256)`), fused here.
 * Replaces: cutejax.call(_quant_launch, ..., nf4=False) at kernels/quantize.py:226-233
 * behind quantize_blockwise (kernels/quantize.py:251-262). */
BNBQ_API int bnbq_quantize_blockwise(int dtype, const void* x, int64_t n, int32_t blocksize,
                            const float* code, const float* offset,
                            uint8_t* q, float* absmax, void* stream);

/* offset[0] = mean(absmax[0..nb)) as float32 (double accumulation, one rounding;
 * deterministic). Replaces the XLA reduction `jnp.mean(absmax)` at array.py:200. */
BNBQ_API int bnbq_absmax_mean(const float* absmax, int64_t nb, float* offset, void* stream);

/* NF4 quantization with double-quantized scales in ONE kernel launch (plus a
 * 12-byte memset of the workspace's barrier counters): bitwise the chain
 *   bnbq_quantize_nf4(x -> q, absmax);
 *   bnbq_absmax_mean(absmax -> offset);
 *   bnbq_quantize_blockwise(absmax with *offset subtracted, code2, blocksize2
 *                           -> absmax_q, absmax2).
 * absmax (ceil(n/blocksize) floats, 16-byte aligned) is written too: it is the
 * nested pass's input. blocksize2: power of two, 8..256 (the format's 256).
 * workspace: at least bnbq_quantize_nf4_dq_workspace_bytes() bytes, 16-byte
 * aligned, any contents (the call clears it on the stream); calls sharing it
 * must be ordered on one stream. The kernel is a cooperative launch whose two
 * grid-wide barriers are bounded in time (an expiry is counted by
 * bnbq_wait_timeouts and leaves the outputs wrong). n must be > 0.
 * Replaces: quantize(x, "nf4", bs, double_quant=True) at array.py:199-202
 * (quantize_nf4, then jnp.mean, then quantize_blockwise: three launches). */
BNBQ_API int bnbq_quantize_nf4_dq(int dtype, const void* x, int64_t n, int32_t blocksize,
                                  const float* code2, int32_t blocksize2, uint8_t* q, float* absmax,
                                  uint8_t* absmax_q, float* absmax2, float* offset,
                                  void* workspace, int64_t workspace_bytes, void* stream);
BNBQ_API int64_t bnbq_quantize_nf4_dq_workspace_bytes(void);

/* -------------------------------------------------------------- dequantize */

/* out[i] = dtype(mul.ftz(NF4_TABLE[nibble_i], absmax[i / bs])), i < n.
 * Replaces: cutejax.call(_dequant_launch, ..., nf4=True) at kernels/dequantize.py:110-116
 * behind dequantize_nf4 (kernels/dequantize.py:120-134). */
BNBQ_API int bnbq_dequantize_nf4(int dtype, const uint8_t* q, const float* absmax,
                        int64_t n, int32_t blocksize, void* out, void* stream);

/* out[i] = dtype(mul.ftz(code[q_i], absmax[i / bs])) (+ *offset, float32 add, when
 * offset != NULL and dtype is F32: the offset add of a nested absmax, array.py:107-108).
 * Replaces: cutejax.call(_dequant_launch, ..., nf4=False) at kernels/dequantize.py:110-116
 * behind dequantize_blockwise (kernels/dequantize.py:137-148). */
BNBQ_API int bnbq_dequantize_blockwise(int dtype, const uint8_t* q, const float* absmax,
                              const float* code, int64_t n, int32_t blocksize,
                              const float* offset, void* out, void* stream);

/* Double-quantized NF4 decode in one pass: the block scale is decoded in-kernel as
 *   a_b = fl32(mul.ftz(code2[absmax_q[b]], absmax2[b / bs2]) + offset[0])
 * and out[i] = dtype(mul.ftz(NF4_TABLE[nibble_i], a_{i/bs})).
 * Bitwise equal to the reference's three-step chain QuantizedArray.dequantize
 * (array.py:95-104: nested 8-bit dequantize, XLA add of the offset, NF4 dequantize). */
BNBQ_API int bnbq_dequantize_nf4_nested(int dtype, const uint8_t* q, const uint8_t* absmax_q,
                               const float* absmax2, const float* code2, const float* offset,
                               int64_t n, int32_t blocksize, int32_t blocksize2,
                               void* out, void* stream);

/* Double-quantized 8-bit decode in one pass (same nested scale decode as above, then
 * the 8-bit codebook `code`). Replaces array.py:95-97 + :103-104 for qtype "8bit". */
BNBQ_API int bnbq_dequantize_blockwise_nested(int dtype, const uint8_t* q, const float* code,
                                     const uint8_t* absmax_q, const float* absmax2,
                                     const float* code2, const float* offset,
                                     int64_t n, int32_t blocksize, int32_t blocksize2,
                                     void* out, void* stream);

/* ------------------------------------------------------------------ matmul */

/* y[m, j] = sum_k x[m, k] * W[j, k] for an NF4 weight W of n_rows x k, never
 * materialised. x: m x k row-major, dtype F16 or BF16; y: m x n_rows of the same
 * dtype with row stride ldy (>= n_rows) elements.
 * w: the weight's packed codes, row-major, n_rows*k/2 bytes (high nibble first).
 * Scales: `absmax` (n_rows*k/bs floats) when absmax_q == NULL; otherwise the
 * double-quantized triple absmax_q (n_rows*k/bs bytes), absmax2, code2 (256) and
 * offset (1 float), with absmax2 indexed by the GLOBAL block number
 * (absmax2_block0 + local block) / blocksize2, so that a row shard of a weight can
 * pass its own slices of w / absmax_q and the whole absmax2.
 * Numerics: per block, t = sum table[q]*x in float32; acc += a*t; one rounding
 * to dtype at the end (kernels/gemv.py:97-123). A one-hot x returns the decoded
 * weights bitwise.
 * Requires k % 32 == 0 and 32 <= blocksize (a power of two), like the reference
 * (kernels/gemv.py:172-181). bnbq_gemv_nf4 handles 1 <= m <= BNBQ_GEMV_MAX_M.
 * Replaces: cutejax.call(_gemv_launch, ...) at kernels/gemv.py:195-204 (gemv_nf4). */
BNBQ_API int bnbq_gemv_nf4(int dtype, const void* x, int32_t m, int32_t k,
                  const uint8_t* w, int64_t n_rows, int32_t blocksize,
                  const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                  const float* code2, const float* offset, int32_t blocksize2,
                  int64_t absmax2_block0, void* y, int64_t ldy, void* stream);

/* Same contract for any m >= 1: the GEMV for m <= BNBQ_GEMV_MAX_M, the tcgen05/TMEM
 * fused dequantize-GEMM above it (weights decoded to dtype in tensor memory, i.e.
 * the reference fallback's precision `x @ w.dequantize(x.dtype).T`, _matmul.py:58-59,
 * accumulated in float32 in tensor memory).
 * Replaces: the router _matmul_2d (_matmul.py:46-60) for NF4 weights. */
BNBQ_API int bnbq_matmul_nf4(int dtype, const void* x, int32_t m, int32_t k,
                    const uint8_t* w, int64_t n_rows, int32_t blocksize,
                    const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                    const float* code2, const float* offset, int32_t blocksize2,
                    int64_t absmax2_block0, void* y, int64_t ldy, void* stream);

/* bnbq_gemv_nf4 / bnbq_matmul_nf4 with a workspace: device memory the caller
 * allocates once (bnbq_gemv_workspace_bytes gives its size for a shape; one
 * buffer as large as the largest serves every shape; its contents need no
 * initial value) and passes to every call. With it, 1 <= m <= 4 runs the
 * shared-memory pair-table GEMV, which splits K across the SMs and writes
 * its partial sums there; a second kernel adds them in a fixed order (the
 * results are deterministic). Other shapes, or a workspace that is NULL or
 * too small, run the kernels of bnbq_gemv_nf4. Calls that share a workspace
 * must be ordered on one stream. Same numerics contract and one-hot
 * exactness as bnbq_gemv_nf4. The weight codes and scales are read before
 * the kernel waits for the preceding kernel on the stream (programmatic
 * dependent launch); x is read and y written after it. */
BNBQ_API int bnbq_gemv_nf4_ws(int dtype, const void* x, int32_t m, int32_t k,
                     const uint8_t* w, int64_t n_rows, int32_t blocksize,
                     const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                     const float* code2, const float* offset, int32_t blocksize2,
                     int64_t absmax2_block0, void* y, int64_t ldy,
                     void* workspace, int64_t workspace_bytes, void* stream);
BNBQ_API int bnbq_matmul_nf4_ws(int dtype, const void* x, int32_t m, int32_t k,
                       const uint8_t* w, int64_t n_rows, int32_t blocksize,
                       const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                       const float* code2, const float* offset, int32_t blocksize2,
                       int64_t absmax2_block0, void* y, int64_t ldy,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* The backward of the fused matmul for a few rows of g: out[m, k] =
 * sum_n g[m, n] * W[n, k] for an NF4 weight W (n_rows x k), never
 * materialised, 1 <= m <= 4, k % 256 == 0, blocksize >= 32. g: m x n_rows
 * (row stride ldg elements), out: m x k (row stride ldo), both F16 or BF16;
 * scales and absmax2 indexing as bnbq_gemv_nf4. Every weight is its exact
 * dequantized float32 value, times g in float32, summed in a fixed order and
 * rounded once: a one-hot g returns the dequantized weight row bitwise. The
 * workspace (any contents, 16-byte aligned, at least
 * bnbq_gemv_t_nf4_workspace_bytes for that m, k and n_rows on this device)
 * takes per-warp partial sums of each column group that a second kernel adds
 * in a fixed order. Calls sharing it must be ordered on one stream.
 * Replaces: the custom VJP's backward g @ w.dequantize(g.dtype)
 * (_matmul.py:67-68) for those shapes. */
BNBQ_API int bnbq_gemv_t_nf4_ws(int dtype, const void* g, int32_t m, int64_t n_rows, int64_t ldg, int32_t k,
                                const uint8_t* w, int32_t blocksize, const float* absmax,
                                const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                                void* out, int64_t ldo, void* workspace, int64_t workspace_bytes, void* stream);
BNBQ_API int bnbq_gemv_t_nf4_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes);

/* Which kernels bnbq_matmul_nf4_ws runs for a call of this shape with this
 * workspace (the scales' pointer matters only through its alignment):
 * BNBQ_ROUTE_TABLE_GEMV (the pair-table GEMV, 1 <= m <= 4), BNBQ_ROUTE_GEMV
 * (the other GEMV kernels, m <= BNBQ_GEMV_MAX_M) or BNBQ_ROUTE_GEMM (the
 * tcgen05 GEMM). Host-only. No counterpart in the reference. */
enum bnbq_route { BNBQ_ROUTE_TABLE_GEMV = 1, BNBQ_ROUTE_GEMV = 2, BNBQ_ROUTE_GEMM = 3 };
BNBQ_API int bnbq_gemv_route(int32_t m, int32_t k, int64_t n_rows, int32_t blocksize, const uint8_t* absmax_q,
                             int32_t blocksize2, const void* workspace, int64_t workspace_bytes, int32_t* route);

/* Which GEMV bnbq_gemv_nf4_ws / bnbq_matmul_nf4_ws use when both apply:
 * 0 (default) by shape -- the pair-table GEMV for weights with at least 1.5
 * output rows per element of K, the streaming row kernels otherwise --, 1 the
 * pair-table GEMV whenever it applies, 2 never. Process-wide; for tests and
 * tuning. No counterpart in the reference. */
BNBQ_API int bnbq_set_gemv_policy(int32_t policy);

/* Workspace bytes bnbq_gemv_nf4_ws / bnbq_matmul_nf4_ws use for an (m x k) x
 * and an n_rows x k weight (0: that shape needs none). */
BNBQ_API int bnbq_gemv_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes);

/* y[m, j] = sum_k x[m, k] * W[j, k] for an 8-bit blockwise-quantized weight W
 * (bnbq_quantize_blockwise's format: one code byte per element, row-major
 * n_rows x k, decoded through the 256-float codebook `code`), never
 * materialised, for 1 <= m <= BNBQ_GEMV8_MAX_M rows of x (F16 or BF16).
 * Scales, absmax2 indexing, y's row stride, numerics (float32 products of x
 * with code[q], the block's scale applied once per block, one rounding) and
 * the one-hot exactness are those of bnbq_gemv_nf4. Requires k % 128 == 0
 * and a power-of-two blocksize >= 32; the workspace (any contents, at least
 * bnbq_gemv_blockwise_workspace_bytes, 256-byte aligned) takes the split-K
 * partial sums, which a second kernel adds in a fixed order.
 * The reference has no fused path for 8-bit weights: this replaces its
 * fallback x @ w.dequantize(x.dtype).T for them (_matmul.py:58-59, chosen by
 * _fused_applies, _matmul.py:74-79). */
#define BNBQ_GEMV8_MAX_M 4
BNBQ_API int bnbq_gemv_blockwise_ws(int dtype, const void* x, int32_t m, int32_t k,
                                    const uint8_t* w, int64_t n_rows, int32_t blocksize, const float* code,
                                    const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                                    const float* code2, const float* offset, int32_t blocksize2,
                                    int64_t absmax2_block0, void* y, int64_t ldy,
                                    void* workspace, int64_t workspace_bytes, void* stream);
BNBQ_API int bnbq_gemv_blockwise_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes);

/* ------------------------------------------------------------ diagnostics */

/* All-gather of a row-sharded matmul output over NVLink peer memory (the
 * exchange of the N-sharded GEMV/GEMM; the reference has no counterpart -- it
 * runs on one device -- and NCCL's all-gather is the portable alternative).
 * y_local: this rank's m x n_local slice (row stride ld_local, dtype F16/BF16),
 * columns [col0, col0 + n_local) of the m x n_total output (the ranks'
 * slices tile [0, n_total); with world 1, col0 = 0 and n_local = n_total,
 * else BNBQ_ERR_INVALID). y_full: this
 * rank's output (row stride ldy >= n_total; written only by this rank).
 * inbox: device array of `world` pointers, rank d's inbox of inbox_words
 * uint64 words (IPC-mapped peer memory for d != rank; 8-byte aligned; zeroed
 * once before the first call; the same inbox_words on every rank, at least
 * 2 * m * n_total, else BNBQ_ERR_TOO_LARGE). state: this rank's uint32[2]
 * (zeroed once; the kernel keeps it). 1 <= world <= 64. Enqueued on `stream`
 * after the matmul that wrote y_local (it waits for it): it stores the slice
 * into every peer's inbox as words {value, epoch} (one 8-byte store each,
 * halves alternating by call), copies it into y_full, and fills the other
 * columns of y_full from this rank's own inbox once their words carry the
 * call's epoch. Every rank must make the same sequence of calls with the same
 * n_total. y_full stays unchanged until this rank's next call on `stream`.
 * The waits for peers are bounded (10 s by default); an expiry is counted by
 * bnbq_wait_timeouts and leaves those columns of y_full unwritten. */
/* CUDA IPC of the buffers the peer all-gather writes (no counterpart in the
 * reference). bnbq_ipc_handle exports the allocation containing `ptr`: 64
 * bytes into handle_out and ptr's offset from the allocation base.
 * bnbq_ipc_open maps such a handle from another process into the current
 * device's context (peer access enabled as needed) and returns the base;
 * bnbq_ipc_close unmaps it. */
BNBQ_API int bnbq_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out);
BNBQ_API int bnbq_ipc_open(const void* handle, void** base_out);
BNBQ_API int bnbq_ipc_close(void* base);

/* Let kernels on the current device access memory of `peer_device` (CUDA peer
 * access of this process's context; needed before bnbq_peer_allgather_rows
 * stores into IPC mappings of another device's memory). BNBQ_OK if enabled or
 * already enabled, BNBQ_ERR_UNSUPPORTED if the devices cannot be peers. No
 * counterpart in the reference. */
BNBQ_API int bnbq_enable_peer_access(int peer_device);

BNBQ_API int bnbq_peer_allgather_rows(int dtype, const void* y_local, int32_t m, int64_t n_local, int64_t ld_local,
                                      int64_t col0, void* y_full, int64_t n_total, int64_t ldy,
                                      uint64_t* const* inbox, int64_t inbox_words, uint32_t* state, int32_t world,
                                      int32_t rank, void* stream);

/* The row-sharded matmul and its all-gather in one call (no counterpart in
 * the reference, which runs on one device): y_full[:, col0 : col0 + n_local]
 * = x @ W_rank.T for this rank's n_local rows of the weight (the arguments of
 * bnbq_matmul_nf4_ws, with n_rows = n_local), and the other columns from the
 * peers, as bnbq_peer_allgather_rows would assemble them (same inbox, state,
 * world and rank arguments; one call per rank in the same order). For M <= 2
 * the matmul kernel itself stores its rows into the peers' inboxes and
 * collects theirs in its epilogue (one kernel chain, no separate exchange
 * launch); other shapes run the matmul, then the exchange kernel. A rank
 * with n_local = 0 only collects. Results bitwise those of
 * bnbq_matmul_nf4_ws on the rank's rows. */
BNBQ_API int bnbq_matmul_nf4_allgather(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                                       int64_t n_local, int32_t blocksize, const float* absmax,
                                       const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                       const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                                       void* y_full, int64_t n_total, int64_t ldy, int64_t col0,
                                       uint64_t* const* inbox, int64_t inbox_words, uint32_t* state, int32_t world,
                                       int32_t rank, void* workspace, int64_t workspace_bytes, void* stream);

/* bnbq_peer_allgather_rows for a caller that may not allocate device memory:
 * code that runs the exchange inside a compiled program whose runtime owns
 * the device memory (an XLA FFI handler receives only its operand and result
 * buffers; cudaMalloc there can fail against the runtime's preallocation and
 * would synchronise the device), or a serving loop held to a fixed memory
 * plan. Such a caller has nowhere to keep `state`, which must outlive every
 * call and start at zero. Here the library keeps it: a fixed 256-byte array
 * per device (held by every device that loads the library until the process
 * exits) with one state pair per exchange slot. Every rank of a group names
 * the same `exchange` slot on every call; limit 32 slots (0..31), a larger
 * slot returns BNBQ_ERR_TOO_LARGE. A slot belongs to one group and one set of
 * zeroed inboxes: before another group (or new inboxes) uses it,
 * every rank calls bnbq_peer_allgather_noalloc_reset. The other arguments and
 * the result are bnbq_peer_allgather_rows's. The first call on a device looks
 * up the array's device address (bnbq_peer_allgather_noalloc_setup does only
 * that: make it before capturing exchanges into a graph). The address is
 * cached per device for the life of the process, so it does not survive a
 * cudaDeviceReset. Calls whose kernels overlap on one device with the same
 * slot race. No counterpart in the reference. */
BNBQ_API int bnbq_peer_allgather_rows_noalloc(int dtype, const void* y_local, int32_t m, int64_t n_local,
                                              int64_t ld_local, int64_t col0, void* y_full, int64_t n_total,
                                              int64_t ldy, uint64_t* const* inbox, int64_t inbox_words,
                                              int32_t exchange, int32_t world, int32_t rank, void* stream);

/* The no-allocation exchange's set-up for the current device (the device
 * address of the library's state array), with no exchange; BNBQ_OK when done.
 * No counterpart in the reference. */
BNBQ_API int bnbq_peer_allgather_noalloc_setup(void);

/* Zero slot `exchange` of the current device's no-allocation state, enqueued
 * on `stream`. No counterpart in the reference. */
BNBQ_API int bnbq_peer_allgather_noalloc_reset(int32_t exchange, void* stream);

/* out[i] = rcp.approx.ftz.f32(in[i]): the hardware reciprocal the quantize kernels
 * use for 1/absmax (kernels/_ptx.py:20-22). Lets a CPU checker take the device's
 * own reciprocal instead of modelling it. */
BNBQ_API int bnbq_rcp_approx_ftz(const float* in, float* out, int64_t n, void* stream);

/* Number of bounded device-side waits that expired on the current device since
 * the library was loaded (pipelined kernels wait on their own bulk copies;
 * each wait gives up after a fixed spin count instead of hanging, and the
 * kernel then stops early). 0 in normal operation. Synchronous. */
BNBQ_API int bnbq_wait_timeouts(unsigned int* count);

/* Test hook: the time limit of every bounded device-side wait on the current
 * device (the pipelined kernels' waits on their own copies, 1 s by default;
 * the peer all-gather's waits for other ranks, 10 s by default), in
 * nanoseconds; 0 restores the defaults. A test shortens it to make a wait run
 * out on purpose and checks that the kernel returns and counts the expiry.
 * Synchronous. No counterpart in the reference. */
BNBQ_API int bnbq_set_wait_limit_ns(uint64_t ns);

/* Human-readable name of a status code (static storage). */
BNBQ_API const char* bnbq_error_string(int status);

/* Library version: major*10000 + minor*100 + patch. */
BNBQ_API int bnbq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BNBQ_H_ */
