/*
 * kvq.h - C ABI of the B200 (sm_100a) 4-bit KV-cache library (libkvq.so).
 *
 * Drop-in native layer under the Python entry points of the reference
 * sztlink/krea-realtime-bench (quant_kv.py, quant_kv_kernels.py). Every entry
 * point takes plain device pointers, sizes and a CUDA stream (passed as void*,
 * a cudaStream_t; NULL = legacy default stream), launches asynchronously on that
 * stream and returns 0 or a negative status. No exception crosses the ABI;
 * kvq_last_error() returns the message of the calling thread's last failure.
 *
 * Cache storage (identical to the reference, quant_kv.py:107-111 and
 * quant_kv_kernels.py:13-16):
 *   codes   uint8 [S, H, D/2] int4: byte i = code(2i) | code(2i+1) << 4, code = q + 8
 *           uint8 [S, H, D]   int8: code = q + 128
 *   scales  bf16  [S, H, G]   one scale per (token, head, channel group)
 *   sink    bf16  [sink, H, D] exact copy of the first `sink` tokens (optional)
 * Channel groups are given by a HOST int32 array chan_band[D] (group index per
 * channel, values in [0, G)), the array the reference builds on the device with
 * build_chan_band (quant_kv_kernels.py:114-119). The five layouts the reference
 * uses (bands, bands2, bands4, blind32, blind64; quant_kv.py:62-82) run on
 * specialised kernels; any other map runs on a generic kernel with the same
 * results.
 */
#ifndef KVQ_H_
#define KVQ_H_

#include <stdint.h>

#if defined(__GNUC__)
#define KVQ_API __attribute__((visibility("default")))
#else
#define KVQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define KVQ_OK 0
#define KVQ_ERR_ARG (-1)         /* invalid argument: shape, pointer, group map */
#define KVQ_ERR_UNSUPPORTED (-2) /* valid but not supported by this build (e.g. head_dim) */
#define KVQ_ERR_CUDA (-3)        /* a CUDA runtime call failed (message has the CUDA error) */
#define KVQ_ERR_ALIGN (-4)       /* a pointer or stride is not aligned as required */
#define KVQ_ERR_DEVICE (-5)      /* the current device is not an sm_100 part */

/* ABI version of this header; bumped on any signature change. */
#define KVQ_ABI_VERSION 3

/* Size of the opaque handle kvq_ipc_export() writes (a cudaIpcMemHandle_t). */
#define KVQ_IPC_HANDLE_BYTES 64

KVQ_API int kvq_abi_version(void);

/* Message of the calling thread's last failing call ("" if none). */
KVQ_API const char* kvq_last_error(void);

/*
 * Quantize rows of bf16 K or V into codes + scales, in place.
 * Replaces: quant_kv_kernels.quantize (quant_kv_kernels.py:102-111), the Triton
 * _quant_kernel launch (quant_kv_kernels.py:57-84) and the torch oracle
 * QuantKVTensor._quantize (quant_kv.py:142-159). Codes and scales are bit-exact
 * to the torch path (round half to even, IEEE divides), not to the Triton kernel.
 *
 *   x          bf16 [n_tokens][n_heads][head_dim], token stride x_token_stride
 *              elements (>= n_heads*head_dim); 16-byte aligned rows
 *   codes      uint8 out, [n_tokens][n_heads][head_dim/2] (bits 4) or [..][head_dim] (bits 8)
 *   scales     bf16 out, [n_tokens][n_heads][n_groups]
 *   sink       bf16 out or NULL: rows of x whose token index is < sink_tokens are
 *              also copied verbatim to sink ([sink_tokens][n_heads][head_dim]),
 *              as QuantKVTensor.__setitem__ does (quant_kv.py:213-215)
 *   chan_band  HOST int32[head_dim], group of each channel
 *   bits       4 or 8 (qmax 7 or 127)
 */
KVQ_API int kvq_quantize(const void* x, int64_t x_token_stride, void* codes, void* scales,
                 void* sink, int64_t sink_tokens, int64_t n_tokens, int n_heads,
                 int head_dim, const int32_t* chan_band, int n_groups, int bits,
                 void* stream);

/*
 * Dequantize rows to bf16, optionally overlaying the exact sink copy.
 * Replaces: quant_kv_kernels.dequantize (quant_kv_kernels.py:91-99), the Triton
 * _dequant_kernel (quant_kv_kernels.py:33-55) and, with a sink, the read
 * QuantKVTensor.__getitem__ (quant_kv.py:189-199). Bit-exact to the torch path.
 *
 *   codes, scales  as produced by kvq_quantize, first row = first token read
 *   sink           bf16 or NULL; tokens < sink_tokens are copied from sink
 *                  (sink points at the sink row of the first token read)
 *   out            bf16 out [n_tokens][n_heads][head_dim], token stride
 *                  out_token_stride elements
 */
KVQ_API int kvq_dequantize(const void* codes, const void* scales, const void* sink,
                   int64_t sink_tokens, void* out, int64_t out_token_stride,
                   int64_t n_tokens, int n_heads, int head_dim,
                   const int32_t* chan_band, int n_groups, int bits, void* stream);

/*
 * The requantizing move of the reference's eviction `kv[:, a:b] = kv[:, c:d].clone()`
 * (quant_kv.py:13; the clone dequantizes, quant_kv.py:189-199, and the slice write
 * quantizes, quant_kv.py:201-215) in one pass over packed rows: for each of
 * n_tokens x n_heads rows, value = the row's bf16 from src_exact for the first
 * exact_tokens tokens (a source window's sink rows), else kvq_dequantize() of
 * src_codes / src_scales; then dst_codes / dst_scales := kvq_quantize(value), and the
 * first sink_tokens tokens' values also go to dst_sink. Bit-identical to
 * kvq_dequantize() followed by kvq_quantize(), without the bf16 window in memory.
 * int4 codes, head_dim 128 and the five specialised group maps (KVQ_ERR_UNSUPPORTED
 * otherwise: take the two-call path). Source and destination must not overlap.
 */
KVQ_API int kvq_requantize(const void* src_codes, const void* src_scales, const void* src_exact,
                           int64_t exact_tokens, void* dst_codes, void* dst_scales, void* dst_sink,
                           int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim,
                           const int32_t* chan_band, int n_groups, int bits, void* stream);

/*
 * Fused int4-KV attention over a cache window, reading K and V packed.
 * Replaces the read path `attention(q, kv_cache["k"][:, lo:hi], kv_cache["v"][:, lo:hi])`
 * (quant_kv.py:14): QuantKVTensor.__getitem__'s dequantize + bf16 sink overlay
 * (quant_kv.py:189-199) followed by the upstream attention() call that
 * probe_attention.py:97-124 hooks (softmax(q k^T / sqrt(D)) v, non-causal).
 *
 *   q          bf16 [batch][n_q][n_heads][head_dim], token stride q_token_stride
 *   k_*, v_*   cache storage of K and V as written by kvq_quantize, streams
 *              stacked: stream b owns cache rows [b*cache_tokens, (b+1)*cache_tokens)
 *              and sink rows [b*sink_tokens, (b+1)*sink_tokens)
 *   lo, hi     window of cache tokens; tokens < sink_tokens come from the sinks
 *   out        bf16 [batch][n_q][n_heads][head_dim], token stride out_token_stride
 *   softmax_scale  <= 0 selects 1/sqrt(head_dim)
 *   workspace  NULL, or device memory of workspace_bytes bytes (256-byte aligned)
 *              that kvq_attention_workspace_bytes() asks for: with it, the units
 *              of the launch's last wave are cut along the KV window into parts
 *              whose partial results the last part to finish merges (the
 *              workspace holds them, and a counter per unit that the launch
 *              clears first); launches that share a workspace must be ordered
 *              (one stream). Without it, or when it is too small, every unit
 *              runs whole; the results agree within the attention tolerance.
 * head_dim 128; K int4 (k_bits 4) or int8 (k_bits 8, the K8V4 mode of
 * bench_qkv.py:160) and V int4; the five reference group layouts.
 */
KVQ_API int kvq_attention(const void* q, int64_t q_token_stride,
                          const void* k_codes, const void* k_scales, const void* k_sink,
                          const void* v_codes, const void* v_scales, const void* v_sink,
                          int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi,
                          void* out, int64_t out_token_stride, int batch, int64_t n_q,
                          int n_heads, int head_dim, const int32_t* chan_band, int n_groups,
                          int k_bits, int v_bits, float softmax_scale, void* workspace,
                          int64_t workspace_bytes, void* stream);

/*
 * Bytes of workspace kvq_attention() / kvq_attention_gather() use for a launch
 * of this shape on the current device (0: the launch runs every unit whole), in
 * *bytes. No counterpart in the reference (its attention is a library call).
 */
KVQ_API int kvq_attention_workspace_bytes(int batch, int64_t n_q, int n_heads, int64_t n_kv_tokens,
                                          int64_t* bytes);

/*
 * kvq_attention() for callers that cannot allocate device memory or hand over a
 * workspace: a frame loop in which a cudaMalloc or cudaFree would synchronize the
 * device and stall the frame, or a host framework that owns the device memory
 * through its own pool and gives a plugin no way to ask for more. No counterpart
 * in the reference (its attention is a library call with no workspace).
 * The workspace is KVQ_NOALLOC_SCRATCH_BYTES of device memory inside the library,
 * one instance per device, held by every GPU that loads the library's device code
 * until the process exits; no call allocates. It keeps the last call's contents:
 * each launch first clears the part counters that must start at zero (the partial
 * results are always written before they are read). The first call on a device looks
 * the scratch up (and loads the library's device code if that has not happened
 * yet): make it before any stream capture. A shape whose workspace would be
 * larger (kvq_attention_workspace_bytes) is rejected with KVQ_ERR_UNSUPPORTED.
 * All calls on one device share the scratch: calls that may overlap on the GPU
 * (streams not ordered with one another) race and corrupt each other's output.
 * Arguments and results as kvq_attention() with a workspace.
 */
#define KVQ_NOALLOC_SCRATCH_BYTES (32ll << 20)
KVQ_API int kvq_attention_noalloc(const void* q, int64_t q_token_stride,
                                  const void* k_codes, const void* k_scales, const void* k_sink,
                                  const void* v_codes, const void* v_scales, const void* v_sink,
                                  int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi,
                                  void* out, int64_t out_token_stride, int batch, int64_t n_q,
                                  int n_heads, int head_dim, const int32_t* chan_band, int n_groups,
                                  int k_bits, int v_bits, float softmax_scale, void* stream);

/*
 * kvq_attention() that also writes, per (stream, query, head), four fp32 row
 * statistics of the attention distribution p = softmax(q k^T * scale) to
 * stats[batch][n_q][n_heads][4] (16-byte aligned): log-sum-exp of the scaled
 * logits, entropy -sum p ln p (nats), max p, and the mass sum p over cache
 * tokens below sink_tokens. The reference's attention probe computes the last
 * three on a sample of queries in fp32 (probe_attention.py:102-121: entropia,
 * peso_max, massa_ancora; adaptive_reset.py uses them as its spread sensor);
 * here they come out of the fused kernel for every query.
 */
KVQ_API int kvq_attention_stats(const void* q, int64_t q_token_stride,
                                const void* k_codes, const void* k_scales, const void* k_sink,
                                const void* v_codes, const void* v_scales, const void* v_sink,
                                int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi,
                                void* out, int64_t out_token_stride, float* stats, int batch, int64_t n_q,
                                int n_heads, int head_dim, const int32_t* chan_band, int n_groups,
                                int k_bits, int v_bits, float softmax_scale, void* stream);

/*
 * kvq_quantize() of keys before their rotary embedding: each row is rotated
 * first, exactly as the upstream runtime does before its cache write (Wan's
 * rope_apply, not vendored; band split quant_kv.py:26-31): channel pairs
 * (2i, 2i+1) as complex128 times freqs[positions[t][a(i)]][i] = (cos, sin)
 * (a(i) = 0/1/2 for pairs [0,22)/[22,43)/[43,64): frame/height/width axis),
 * rounded to fp32 and then to bf16; then quantized, and the sink rows receive the
 * rotated bf16 values. freqs: device float64 [max_pos][64][2] (16-byte aligned);
 * positions: device int32 [n_tokens][3] (values outside [0, max_pos) clamp).
 * head_dim 128 and the five specialised group layouts. Replaces the separate
 * rotary kernel and cache write (quant_kv.py:12) of an append.
 */
KVQ_API int kvq_rope_quantize(const void* x, int64_t x_token_stride, void* codes, void* scales, void* sink,
                              int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim,
                              const int32_t* chan_band, int n_groups, int bits, const double* freqs,
                              int max_pos, const int32_t* positions, void* stream);

/*
 * kvq_quantize() of the same token range of n_tensors tensors (1..96, e.g. the
 * 40 layers x {K, V} of a window rebuild) in one launch: tensor i reads x[i]
 * and writes codes[i], scales[i] and, for its first sink_tokens tokens,
 * sink[i] (sink may be NULL for no sink copy; single entries may be NULL too).
 * All tensors share n_tokens, n_heads, head_dim, x_token_stride, the group map
 * and bits; every pointer has the alignment kvq_quantize() requires. Results are
 * bit-identical to n_tensors kvq_quantize() calls. Replaces the per-layer
 * quantize launches of a rebuild (quant_kv_kernels.py:102-111 called once per
 * layer and tensor through quant_kv.py:212-215).
 */
KVQ_API int kvq_rebuild_layers(int n_tensors, const void* const* x, int64_t x_token_stride,
                               void* const* codes, void* const* scales, void* const* sink,
                               int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim,
                               const int32_t* chan_band, int n_groups, int bits, void* stream);

/*
 * kvq_attention() for one rank of a head-sharded job: the n_heads heads of this
 * launch are written at heads [out_head0, out_head0 + n_heads) of each of the
 * n_outs output buffers outs[0..n_outs) (1 <= n_outs <= 8), all of layout
 * [batch, n_q, out_heads, head_dim] bf16 with token stride out_token_stride
 * (elements, >= out_heads * head_dim, multiple of 8; buffers 16-byte aligned).
 * With outs = every rank's output buffer (peers mapped by kvq_ipc_import()),
 * the epilogue is the all-gather of the output over NVLink: when every rank's
 * launch has completed, every rank holds the full [batch, n_q, out_heads, D].
 * To read the gathered output without a host barrier, follow the launch on
 * every rank by kvq_gather_barrier() on the same stream.
 * Other arguments and errors as kvq_attention(). No counterpart in the
 * reference (single GPU); replaces the attention + NCCL all-gather pair of a
 * head-sharded deployment.
 */
KVQ_API int kvq_attention_gather(const void* q, int64_t q_token_stride,
                                 const void* k_codes, const void* k_scales, const void* k_sink,
                                 const void* v_codes, const void* v_scales, const void* v_sink,
                                 int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi,
                                 void* const* outs, int n_outs, int out_head0, int out_heads,
                                 int64_t out_token_stride, int batch, int64_t n_q,
                                 int n_heads, int head_dim, const int32_t* chan_band, int n_groups,
                                 int k_bits, int v_bits, float softmax_scale, void* workspace,
                                 int64_t workspace_bytes, void* stream);

/*
 * Device-side barrier of the ranks of a head-sharded job, stream-ordered: one
 * thread on `stream`, after the work before it on the stream (e.g. the rank's
 * kvq_attention_gather()) has completed, adds 1 to every rank's counter
 * counters[0..n_ranks) (unsigned 32-bit, 4-byte aligned, counters[self] in this
 * GPU's memory, the others peers' counters mapped by kvq_ipc_import()) with
 * release semantics at system scope, then waits until its own counter reaches
 * target (compared modulo 2^32; target = n_ranks x the number of barriers so
 * far) with acquire semantics. Work launched after it reads every rank's stores
 * made before their barrier, without a host barrier. Gives up after wait_cycles
 * (>= 1000, at most about a second), raising the device status word
 * (kvq_device_status()). No counterpart in the reference (single GPU).
 */
KVQ_API int kvq_gather_barrier(unsigned int* const* counters, int n_ranks, int self, unsigned int target,
                               int64_t wait_cycles, void* stream);

/*
 * CUDA IPC for the output buffers of kvq_attention_gather(). kvq_ipc_export()
 * writes KVQ_IPC_HANDLE_BYTES bytes naming the device allocation that contains
 * ptr and the byte offset of ptr in it; another process passes both to
 * kvq_ipc_import(), which maps the allocation (*base) and returns the address of
 * ptr there (*ptr); kvq_ipc_close(base) unmaps it. No counterpart in the
 * reference (single GPU).
 */
KVQ_API int kvq_ipc_export(const void* ptr, void* handle, int64_t* offset);
KVQ_API int kvq_ipc_import(const void* handle, int64_t offset, void** base, void** ptr);
KVQ_API int kvq_ipc_close(void* base);

/*
 * Test hook of the bounded waits (no counterpart in the reference, whose Triton
 * kernels have no waits): kvq_attention() with the K tiles from stall_tile on
 * withheld by the producer and every wait limited to wait_cycles (>= 1000 and at
 * most the default of about a second). The waits for the withheld tile give up,
 * the kernel raises the device status word (kvq_device_status() returns 1), lets
 * its in-flight copies and MMAs finish, frees its tensor memory and returns; the
 * output is invalid. Used by the tests to show that a timed-out launch leaves
 * the context usable.
 */
KVQ_API int kvq_test_attention_timeout(const void* q, int64_t q_token_stride,
                                       const void* k_codes, const void* k_scales, const void* k_sink,
                                       const void* v_codes, const void* v_scales, const void* v_sink,
                                       int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi,
                                       void* out, int64_t out_token_stride, int batch, int64_t n_q,
                                       int n_heads, int head_dim, const int32_t* chan_band, int n_groups,
                                       int k_bits, int v_bits, float softmax_scale, int stall_tile,
                                       int64_t wait_cycles, void* stream);

/*
 * Synchronizes the current device and returns the library's device status word:
 * 0 = no kernel gave up, 1 = a kernel's bounded wait timed out (its output is
 * invalid). reset != 0 clears it. No counterpart in the reference (its Triton
 * kernels have no waits).
 */
KVQ_API int kvq_device_status(int reset);

#ifdef __cplusplus
}
#endif

#endif /* KVQ_H_ */
