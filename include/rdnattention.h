/*
 * rdnattention for B200 (sm_100a) — stable C ABI of librdnattention.so.
 *
 * Drop-in replacement for the reference library's C ABI
 * (src/c_api.hpp:16-87 of dmonkman/RDNAttention): identical symbol names,
 * argument order, argument meaning and return codes, so the reference's own
 * ctypes binding (rdnattention/__init__.py:94-130) loads this library
 * unchanged.  Device pointers are CUDA device pointers and `stream` is a
 * cudaStream_t (the reference's hipStream_t slot).
 *
 * Every function operates on caller-owned device memory and keeps no handle
 * table.  Launches are enqueued on `stream` and never block the host.  The
 * only device memory the library obtains itself is the RoPE workspace of
 * rdna_attention_forward (stream-ordered; see rdna_attention_forward_ws for
 * the variant that takes it from the caller).
 */
#ifndef RDNATTENTION_H_
#define RDNATTENTION_H_

#include <stdint.h>

#if defined(_WIN32)
#define RDNA_API_EXPORT __declspec(dllexport)
#else
#define RDNA_API_EXPORT __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
#define RDNA_API extern "C" RDNA_API_EXPORT
#else
#define RDNA_API RDNA_API_EXPORT
#endif

/* 1 if at least one CUDA device is visible, else 0.
 * Replaces src/c_api.hpp:16 (rdna_has_device). */
RDNA_API int32_t rdna_has_device(void);

/* Reason the most recent failing call on this thread failed ("" if none
 * has).  Thread-local, never cleared by a successful call.
 * Replaces src/c_api.hpp:18-19 (rdna_get_error). */
RDNA_API const char* rdna_get_error(void);

/* FP16 forward attention.  q/k/v/output: fp16, head_dim contiguous, strides
 * in ELEMENTS for the batch/head/seq axes.  head_dim: any multiple of 32 in
 * [32, 512].  rot_cos/rot_sin (read when has_rope != 0): fp32
 * [max(seq_len, key_seq_len), head_dim/2], contiguous, interleaved-pair RoPE
 * applied to Q and K in-kernel.  num_kv_heads < num_heads selects GQA
 * (num_heads % num_kv_heads == 0).  causal != 0 aligns the causal diagonal
 * to the end of the key sequence; window_size > 0 limits each query to a
 * one-sided (causal) or two-sided (|q+delta-k| <= window_size/2) band.
 * Returns 0, or -3 with rdna_get_error() set.
 * Replaces src/c_api.hpp:36-57 (rdna_attention_forward). */
RDNA_API int32_t rdna_attention_forward(
    const void* q, const void* k, const void* v, void* output,
    const void* rot_cos, const void* rot_sin,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, int32_t causal, int32_t has_rope, int32_t window_size,
    void* stream);

/* INT8 forward attention (both GEMMs in int8, s32 accumulation), fp16
 * output.  head_dim 64 or 128; causal, window, GQA; no RoPE.  Dequant:
 * S = float(q.k) * q_scale_i * k_scale_j * scale; q_scale_vec (B, H, S) /
 * k_scale_vec (B, Hkv, KS) fp32 per-token scales override q_scale / k_scale
 * when non-NULL; v_scale is per-tensor.  P is quantised min(127,
 * lround(p * 127)).  Returns 0, or -3 with rdna_get_error() set.
 * Replaces src/c_api.hpp:64-87 (rdna_attention_forward_int8qk). */
RDNA_API int32_t rdna_attention_forward_int8qk(
    const void* q, const void* k, const void* v, void* output,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, float q_scale, float k_scale, float v_scale,
    const void* q_scale_vec, const void* k_scale_vec,
    int32_t causal, int32_t window_size, void* stream);

/* ---- Extensions beyond the reference ABI (no counterpart there) ---- */

/* Bytes of device workspace rdna_attention_forward_ws() needs for this
 * problem: 0 without RoPE; with RoPE, room for the rotated K (fp16), which a
 * pre-pass writes once per call so the attention kernel's K tiles arrive
 * rotated, plus the rotated Q for head_dim > 128 (head_dim <= 128 kernels
 * rotate Q themselves).  Each part is rounded up to 256 bytes.  0 for
 * decode-shaped problems (seq_len x GQA group <= 64, head_dim 64 or 128),
 * whose kernel rotates in place.  (rdna_attention_forward itself obtains the
 * workspace with cudaMallocAsync/cudaFreeAsync on `stream`.) */
RDNA_API uint64_t rdna_attention_forward_workspace_size(
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim, int32_t has_rope);

/* rdna_attention_forward with a caller-owned workspace (256-byte aligned,
 * at least rdna_attention_forward_workspace_size() bytes; may be NULL when
 * that size is 0): the library then allocates nothing.  Same arguments and
 * return codes otherwise. */
RDNA_API int32_t rdna_attention_forward_ws(
    const void* q, const void* k, const void* v, void* output,
    const void* rot_cos, const void* rot_sin,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, int32_t causal, int32_t has_rope, int32_t window_size,
    void* workspace, uint64_t workspace_bytes, void* stream);

/* FP16 forward that allocates nothing, even with RoPE.  No counterpart in
 * the reference library.
 *
 * Who needs it: callers that cannot allocate device memory — a plugin
 * running inside a host framework that owns the device allocator and
 * forbids allocations behind its back, a process under a hard device-memory
 * budget where an allocation may fail at any time, or a device without
 * stream-ordered memory pools (where rdna_attention_forward's cudaMallocAsync
 * is unavailable).  Same arguments and return codes as
 * rdna_attention_forward.
 *
 * The RoPE workspace (rdna_attention_forward_workspace_size bytes) lives in
 * a fixed 32 MiB array inside the library, which every GPU that loads the
 * library keeps reserved until the process exits; a problem whose workspace
 * exceeds it (for example 8 KV heads, head_dim 128: up to 16384 keys in
 * total over the batch fit, 20480 do not) returns -3 with a message naming
 * the limit.  Without RoPE no workspace is used.  The first call on a
 * device looks up the array's device address on that device; make that
 * first call before any stream capture; the address is kept for the life
 * of the process, so calls after cudaDeviceReset are unsupported.  All
 * calls share the one array: calls that overlap on the GPU (different
 * streams or threads) race on it, so serialise them. */
RDNA_API int32_t rdna_attention_forward_noalloc(
    const void* q, const void* k, const void* v, void* output,
    const void* rot_cos, const void* rot_sin,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, int32_t causal, int32_t has_rope, int32_t window_size,
    void* stream);

/* rdna_attention_forward_int8qk plus a per-channel V scale: v_channel, when
 * non-NULL, is fp32 (batch, num_kv_heads, head_dim) and multiplies output
 * column d of every row before the single fp16 rounding (the reference
 * applies the same factor afterwards, on the fp16 result, in its Python
 * helper flash_attn_int8qk_quantized, rdnattention/__init__.py:346-357).
 * Other arguments and return codes as rdna_attention_forward_int8qk. */
RDNA_API int32_t rdna_attention_forward_int8qk_vch(
    const void* q, const void* k, const void* v, void* output,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, float q_scale, float k_scale, float v_scale,
    const void* q_scale_vec, const void* k_scale_vec, const void* v_channel,
    int32_t causal, int32_t window_size, void* stream);

/* fp16 Q/K/V (strided, element strides, head_dim contiguous) -> int8 operands
 * for the INT8 path, on `stream`: q_scale (B, H, S) and k_scale (B, Hkv, KS)
 * = per-row max|x| / 127 (0 -> 1), v_channel (B, Hkv, D) = per-column max
 * over the key sequence of |v| / 127 (0 -> 1); int8 = round-half-even(x /
 * scale) clamped to [-127, 127], written contiguous [B, H(kv), S, D].  Bit-
 * identical to the reference's helpers quantize_int8_qk_pertoken (Q, K) and
 * quantize_int8_perchannel_v (V) (rdnattention/__init__.py:303-343) run as
 * torch ops on CUDA tensors (where max / 127 is a multiplication by the fp32
 * reciprocal of 127).  head_dim 64 or 128.  Returns 0, or -3 with
 * rdna_get_error() set ("Attention (int8qk) failed: ..."). */
RDNA_API int32_t rdna_int8_quantize_qkv(
    const void* q, const void* k, const void* v,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    void* q_int8, void* k_int8, void* v_int8,
    void* q_scale, void* k_scale, void* v_channel, void* stream);

/* Debug (extension, no counterpart in the reference): rdna_attention_forward_int8qk
 * that also writes the raw int32 Q K^T of every key block the kernel computes to
 * `scores`, int32 (batch, num_heads, seq_len, key_seq_len) contiguous; entries of
 * blocks the masks skip are left untouched.  The tensor cores accumulate int8
 * products exactly, so these equal the integer dot products.  Other arguments
 * and return codes as rdna_attention_forward_int8qk. */
RDNA_API int32_t rdna_debug_int8qk_scores(
    const void* q, const void* k, const void* v, void* output,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, float q_scale, float k_scale, float v_scale,
    const void* q_scale_vec, const void* k_scale_vec,
    int32_t causal, int32_t window_size, void* scores, void* stream);

/* Reads and clears the device status word of the current device: out[0] =
 * first error code a kernel recorded (a bounded wait that expired), out[1] =
 * number of such events.  Synchronises the current device.  Returns 0, or
 * -3 with rdna_get_error() set. */
RDNA_API int32_t rdna_debug_read_status(int32_t* out2);

/* Debug (extension, no counterpart in the reference): a test hook for the
 * bounded waits.  Until it is called again with withhold_block < 0, prefill
 * calls made by the calling thread launch with CTA 0 never loading the K tile
 * of its withhold_block-th key block and with CTA 0's waits limited to
 * wait_limit_ns: the wait for that tile expires, the CTA records the wait's
 * site in the status word (rdna_debug_read_status), unwinds (copies in flight
 * land, issued MMAs drain, TMEM is released) and skips its output store, so
 * that CTA's rows of O are left unwritten.  rdna_peer_barrier calls made by
 * the thread meanwhile wait at most wait_limit_ns.  Nothing faults or hangs,
 * and the next call without the hook is unaffected.  Always returns 0. */
RDNA_API int32_t rdna_debug_set_wait_test(int32_t withhold_block, uint64_t wait_limit_ns);

/* Debug (extension): a timing hook.  Until it is called again with NULLs,
 * forward calls made by the calling thread record start_event (a cudaEvent_t)
 * on their stream right before launching their attention kernel (prefill or
 * decode) and stop_event right after it, so the caller can time that kernel
 * alone, without the RoPE pre-pass; the event between the two serialises them
 * (no programmatic overlap of the pre-pass tail).  Always returns 0. */
RDNA_API int32_t rdna_debug_set_kernel_events(void* start_event, void* stop_event);

/* ---- Multi-GPU (extension, no counterpart in the single-device reference) ----
 *
 * The all-gather of the output across the GPUs of one node, fused into the
 * kernels: a *_peers call also writes every output element to each of the
 * n_peers (0..7) buffers in peer_outputs, the other GPUs' counterparts of
 * `output` (same strides, mapped into this process with rdna_ipc_open,
 * 16-byte aligned): the epilogue of each output tile stores it by TMA into
 * every peer's buffer over NVLink (the decode kernel with 16-byte stores), so
 * the transfer overlaps the tiles still being computed.  The
 * peers may read the values once this call's kernels have completed (order
 * their reads after it, e.g. with a collective on the same stream). */

/* rdna_attention_forward_ws with output replicas on other GPUs. */
RDNA_API int32_t rdna_attention_forward_ws_peers(
    const void* q, const void* k, const void* v, void* output,
    const void* rot_cos, const void* rot_sin,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, int32_t causal, int32_t has_rope, int32_t window_size,
    void* workspace, uint64_t workspace_bytes, int32_t n_peers, void* const* peer_outputs, void* stream);

/* rdna_attention_forward_int8qk_vch with output replicas on other GPUs. */
RDNA_API int32_t rdna_attention_forward_int8qk_vch_peers(
    const void* q, const void* k, const void* v, void* output,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, float q_scale, float k_scale, float v_scale,
    const void* q_scale_vec, const void* k_scale_vec, const void* v_channel,
    int32_t causal, int32_t window_size,
    int32_t n_peers, void* const* peer_outputs, void* stream);

/* Device memory other processes can map (CUDA IPC): allocates `bytes` on the
 * current device and writes its 64-byte handle to `handle`. */
RDNA_API int32_t rdna_ipc_alloc(uint64_t bytes, void** ptr, void* handle);
/* Maps another process's rdna_ipc_alloc memory (its 64-byte handle) into this
 * process with peer access enabled. */
RDNA_API int32_t rdna_ipc_open(const void* handle, void** ptr);
/* Unmaps memory mapped by rdna_ipc_open. */
RDNA_API int32_t rdna_ipc_close(void* ptr);
/* Frees rdna_ipc_alloc memory; every process that mapped it must have closed
 * it first. */
RDNA_API int32_t rdna_ipc_free(void* ptr);

/* Cross-GPU barrier ordering the peer stores of a *_peers call, enqueued on
 * `stream` after it: writes `epoch` into word `rank` of each other rank's flag
 * array (peer_flags: the world - 1 other arrays, in rank order without this
 * rank, mapped into this process; 4-byte aligned) and waits until every other
 * rank's word of my_flags (this rank's array, `world` words, zeroed before
 * first use) has reached `epoch` (modulo 2^32).  Work queued after it sees
 * every rank's stores.  Each wait is bounded (60 s); one that expires records
 * code 0x401 in the status word (rdna_debug_read_status) and returns. */
RDNA_API int32_t rdna_peer_barrier(int32_t world, int32_t rank, void* const* peer_flags, void* my_flags,
                                   uint32_t epoch, void* stream);

#endif /* RDNATTENTION_H_ */
