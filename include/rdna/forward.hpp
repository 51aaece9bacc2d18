// C++ entry points behind the C ABI, with the reference's namespace API
// (src/rdna/fa2_forward_f16.hpp:10-44, src/rdna/fa2_forward_int8qk.hpp:10-46)
// so code written against rdna::forwardF16 / rdna::forwardInt8QK links
// against librdnattention.so unchanged.
#pragma once

#include <cstddef>
#include <cstdint>

namespace rdna {

/// Q/K/V/output point at fp16, head_dim contiguous; strides in elements.
/// rot_cos/rot_sin (if hasRope): fp32 [max(seqLen, keySeqLen), headDim/2].
struct ForwardParams {
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    void* o = nullptr;
    const void* rot_cos = nullptr;
    const void* rot_sin = nullptr;
    int64_t qStrideB = 0, qStrideH = 0, qStrideS = 0;
    int64_t kStrideB = 0, kStrideH = 0, kStrideS = 0;
    int64_t vStrideB = 0, vStrideH = 0, vStrideS = 0;
    int64_t oStrideB = 0, oStrideH = 0, oStrideS = 0;
    uint32_t batchSize = 0;
    uint32_t numHeads = 0;
    uint32_t numKvHeads = 0;
    uint32_t seqLen = 0;
    uint32_t keySeqLen = 0;
    uint32_t headDim = 0;  // multiple of 32 in [32, 512]
    float scale = 1.0f;
    uint32_t causal = 0;
    uint32_t hasRope = 0;
    int32_t windowSize = -1;  // <= 0: full attention
};

/// Q/K/V int8, head_dim contiguous; output fp16.
struct ForwardParamsInt8QK {
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    void* o = nullptr;
    int64_t qStrideB = 0, qStrideH = 0, qStrideS = 0;
    int64_t kStrideB = 0, kStrideH = 0, kStrideS = 0;
    int64_t vStrideB = 0, vStrideH = 0, vStrideS = 0;
    int64_t oStrideB = 0, oStrideH = 0, oStrideS = 0;
    uint32_t batchSize = 0;
    uint32_t numHeads = 0;
    uint32_t numKvHeads = 0;
    uint32_t seqLen = 0;
    uint32_t keySeqLen = 0;
    uint32_t headDim = 0;  // 64 or 128
    float scale = 1.0f;
    float qScale = 1.0f;
    float kScale = 1.0f;
    float vScale = 1.0f;
    uint32_t causal = 0;
    int32_t windowSize = -1;
    const void* qScaleVec = nullptr;  // const float*, (batch, heads, seq)
    const void* kScaleVec = nullptr;  // const float*, (batch, kv_heads, key_seq)
    // Extension (no counterpart in the reference): const float*, (batch,
    // kv_heads, head_dim); when set, output column d of every row is
    // multiplied by it before the fp16 rounding (per-channel V dequantisation).
    const void* vChannel = nullptr;
};

/// fp16 Q/K/V -> the operands of the INT8 path with per-token Q/K scales and a
/// per-channel V scale (extension; no counterpart in the reference library,
/// whose Python helpers do this on the host side with torch ops).
struct QuantizeInt8Params {
    const void* q = nullptr;  // fp16 [B, H, S, D], head_dim contiguous, strides in elements
    const void* k = nullptr;  // fp16 [B, Hkv, KS, D]
    const void* v = nullptr;  // fp16 [B, Hkv, KS, D]
    int64_t qStrideB = 0, qStrideH = 0, qStrideS = 0;
    int64_t kStrideB = 0, kStrideH = 0, kStrideS = 0;
    int64_t vStrideB = 0, vStrideH = 0, vStrideS = 0;
    uint32_t batchSize = 0, numHeads = 0, numKvHeads = 0, seqLen = 0, keySeqLen = 0;
    uint32_t headDim = 0;     // 64 or 128
    void* qInt8 = nullptr;    // int8 [B, H, S, D] contiguous
    void* kInt8 = nullptr;    // int8 [B, Hkv, KS, D] contiguous
    void* vInt8 = nullptr;    // int8 [B, Hkv, KS, D] contiguous
    void* qScale = nullptr;   // float [B, H, S]
    void* kScale = nullptr;   // float [B, Hkv, KS]
    void* vChannel = nullptr; // float [B, Hkv, D]
};

/// Enqueues the FP16 forward on `stream` (a cudaStream_t). Non-blocking. 0 on success.
/// With RoPE it takes a stream-ordered workspace (cudaMallocAsync / cudaFreeAsync).
int forwardF16(const ForwardParams& params, void* stream);
/// Device workspace forwardF16Ws() needs for these parameters (0 without RoPE).
size_t workspaceBytesF16(const ForwardParams& params);
/// forwardF16 with a caller-provided workspace (256-byte aligned, at least
/// workspaceBytesF16() bytes; may be null when that is 0).  Allocates nothing.
int forwardF16Ws(const ForwardParams& params, void* workspace, size_t workspace_bytes, void* stream);
/// forwardF16 taking its RoPE workspace from a fixed 32 MiB device array
/// inside the library instead of allocating (see rdna_attention_forward_noalloc).
int forwardF16NoAlloc(const ForwardParams& params, void* stream);
/// Size of that fixed array in bytes.
size_t noAllocWorkspaceLimit();
/// Reason the most recent forwardF16() call on this thread failed, or nullptr.
const char* lastError();
/// Enqueues the INT8 forward on `stream`. Non-blocking. 0 on success.
int forwardInt8QK(const ForwardParamsInt8QK& params, void* stream);
/// Debug (extension): forwardInt8QK that also writes the raw int32 Q K^T of every
/// key block it computes to `scores`, int32 [batch, heads, seq, key_seq]
/// contiguous (entries of skipped blocks are left as they were).
int debugInt8QKScores(const ForwardParamsInt8QK& params, void* scores, void* stream);
/// Reason the most recent forwardInt8QK() / quantizeInt8QKV() call on this thread failed, or nullptr.
const char* lastErrorInt8QK();
/// Enqueues the quantisation on `stream`. Non-blocking. 0 on success.
int quantizeInt8QKV(const QuantizeInt8Params& params, void* stream);
/// Whether a CUDA device is visible.
bool hasDevice();

/// Multi-GPU extensions.  forwardF16Ws / forwardInt8QK that also write the output
/// to `n_peers` (<= 7) other GPUs' counterparts of params.o: same strides,
/// mapped into this process (ipcOpen), 16-byte aligned.  The all-gather of the
/// output is fused into the kernels' epilogues as TMA stores to the peers; the peers
/// may read them once this call's kernels have completed.
int forwardF16WsPeers(const ForwardParams& params, void* workspace, size_t workspace_bytes, int n_peers,
                      void* const* peers, void* stream);
int forwardInt8QKPeers(const ForwardParamsInt8QK& params, int n_peers, void* const* peers, void* stream);
/// Device memory another process can map: cudaMalloc plus its 64-byte IPC handle.
int ipcAlloc(size_t bytes, void** ptr, void* handle);
/// Maps another process's ipcAlloc memory into this one (peer access enabled).
int ipcOpen(const void* handle, void** ptr);
/// Unmaps ipcOpen memory.
int ipcClose(void* ptr);
/// Frees ipcAlloc memory (after every process that mapped it has closed it).
int ipcFree(void* ptr);
/// Enqueues the cross-GPU barrier of the fused all-gather on `stream`: writes
/// `epoch` into slot `rank` of each other rank's flag array (peer_flags: the
/// world - 1 other arrays in rank order, mapped here) and waits (bounded) until
/// every other rank's slot of my_flags has reached it.
int peerBarrier(int world, int rank, void* const* peer_flags, void* my_flags, unsigned int epoch, void* stream);

}  // namespace rdna
