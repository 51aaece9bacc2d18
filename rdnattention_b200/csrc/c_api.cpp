// extern "C" exports of librdnattention.so (include/rdnattention.h).  Same
// marshalling and error contract as the reference (src/c_api.cpp:1-195):
// arguments are copied into the rdna:: parameter structs, a failure returns
// -3 and leaves a thread-local message that is never cleared on success.
// RDNA_API is on the definitions as well as the declarations, so a
// definition whose signature drifts from the header fails to compile.
#include "rdnattention.h"

#include <array>
#include <cstdio>

#include "rdna/forward.hpp"

namespace rdna {
int debugReadStatus(int32_t* out2, const char** why);
void debugSetWaitTest(int32_t withhold_block, uint64_t wait_limit_ns);
void debugSetKernelEvents(void* start, void* stop);
}

namespace {

thread_local std::array<char, 512> g_error{};

void set_error(const char* fmt, const char* detail) {
    std::snprintf(g_error.data(), g_error.size(), fmt, detail != nullptr ? detail : "unknown error");
}

}  // namespace

RDNA_API int32_t rdna_has_device(void) { return rdna::hasDevice() ? 1 : 0; }

RDNA_API const char* rdna_get_error(void) { return g_error.data(); }

namespace {

rdna::ForwardParams f16_params(
    const void* q, const void* k, const void* v, void* output,
    const void* rot_cos, const void* rot_sin,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, int32_t causal, int32_t has_rope, int32_t window_size) {
    rdna::ForwardParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = output;
    p.rot_cos = rot_cos;
    p.rot_sin = rot_sin;
    p.qStrideB = q_stride_b;
    p.qStrideH = q_stride_h;
    p.qStrideS = q_stride_s;
    p.kStrideB = k_stride_b;
    p.kStrideH = k_stride_h;
    p.kStrideS = k_stride_s;
    p.vStrideB = v_stride_b;
    p.vStrideH = v_stride_h;
    p.vStrideS = v_stride_s;
    p.oStrideB = o_stride_b;
    p.oStrideH = o_stride_h;
    p.oStrideS = o_stride_s;
    p.batchSize = batch_size;
    p.numHeads = num_heads;
    p.numKvHeads = num_kv_heads;
    p.seqLen = seq_len;
    p.keySeqLen = key_seq_len;
    p.headDim = head_dim;
    p.scale = scale;
    p.causal = causal != 0 ? 1u : 0u;
    p.hasRope = has_rope != 0 ? 1u : 0u;
    p.windowSize = window_size;
    return p;
}

}  // namespace

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
    void* stream) {
    const rdna::ForwardParams p = f16_params(q, k, v, output, rot_cos, rot_sin, q_stride_b, q_stride_h, q_stride_s,
                                             k_stride_b, k_stride_h, k_stride_s, v_stride_b, v_stride_h, v_stride_s,
                                             o_stride_b, o_stride_h, o_stride_s, batch_size, num_heads, num_kv_heads,
                                             seq_len, key_seq_len, head_dim, scale, causal, has_rope, window_size);
    if (rdna::forwardF16(p, stream) != 0) {
        set_error("Attention (fp16) failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API uint64_t rdna_attention_forward_workspace_size(
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim, int32_t has_rope) {
    rdna::ForwardParams p{};
    p.batchSize = batch_size;
    p.numHeads = num_heads;
    p.numKvHeads = num_kv_heads;
    p.seqLen = seq_len;
    p.keySeqLen = key_seq_len;
    p.headDim = head_dim;
    p.hasRope = has_rope != 0 ? 1u : 0u;
    return rdna::workspaceBytesF16(p);
}

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
    void* workspace, uint64_t workspace_bytes, void* stream) {
    const rdna::ForwardParams p = f16_params(q, k, v, output, rot_cos, rot_sin, q_stride_b, q_stride_h, q_stride_s,
                                             k_stride_b, k_stride_h, k_stride_s, v_stride_b, v_stride_h, v_stride_s,
                                             o_stride_b, o_stride_h, o_stride_s, batch_size, num_heads, num_kv_heads,
                                             seq_len, key_seq_len, head_dim, scale, causal, has_rope, window_size);
    if (rdna::forwardF16Ws(p, workspace, workspace_bytes, stream) != 0) {
        set_error("Attention (fp16) failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

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
    void* workspace, uint64_t workspace_bytes, int32_t n_peers, void* const* peer_outputs, void* stream) {
    const rdna::ForwardParams p = f16_params(q, k, v, output, rot_cos, rot_sin, q_stride_b, q_stride_h, q_stride_s,
                                             k_stride_b, k_stride_h, k_stride_s, v_stride_b, v_stride_h, v_stride_s,
                                             o_stride_b, o_stride_h, o_stride_s, batch_size, num_heads, num_kv_heads,
                                             seq_len, key_seq_len, head_dim, scale, causal, has_rope, window_size);
    if (rdna::forwardF16WsPeers(p, workspace, workspace_bytes, n_peers, peer_outputs, stream) != 0) {
        set_error("Attention (fp16) failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_ipc_alloc(uint64_t bytes, void** ptr, void* handle) {
    if (rdna::ipcAlloc(bytes, ptr, handle) != 0) {
        set_error("IPC allocation failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_ipc_open(const void* handle, void** ptr) {
    if (rdna::ipcOpen(handle, ptr) != 0) {
        set_error("IPC open failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_ipc_close(void* ptr) {
    if (rdna::ipcClose(ptr) != 0) {
        set_error("IPC close failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_peer_barrier(int32_t world, int32_t rank, void* const* peer_flags, void* my_flags,
                                   uint32_t epoch, void* stream) {
    if (rdna::peerBarrier(world, rank, peer_flags, my_flags, epoch, stream) != 0) {
        set_error("Peer barrier failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_ipc_free(void* ptr) {
    if (rdna::ipcFree(ptr) != 0) {
        set_error("IPC free failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

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
    int32_t causal, int32_t window_size, void* stream) {
    rdna::ForwardParamsInt8QK p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = output;
    p.qStrideB = q_stride_b;
    p.qStrideH = q_stride_h;
    p.qStrideS = q_stride_s;
    p.kStrideB = k_stride_b;
    p.kStrideH = k_stride_h;
    p.kStrideS = k_stride_s;
    p.vStrideB = v_stride_b;
    p.vStrideH = v_stride_h;
    p.vStrideS = v_stride_s;
    p.oStrideB = o_stride_b;
    p.oStrideH = o_stride_h;
    p.oStrideS = o_stride_s;
    p.batchSize = batch_size;
    p.numHeads = num_heads;
    p.numKvHeads = num_kv_heads;
    p.seqLen = seq_len;
    p.keySeqLen = key_seq_len;
    p.headDim = head_dim;
    p.scale = scale;
    p.qScale = q_scale;
    p.kScale = k_scale;
    p.vScale = v_scale;
    p.causal = causal != 0 ? 1u : 0u;
    p.windowSize = window_size;
    p.qScaleVec = q_scale_vec;
    p.kScaleVec = k_scale_vec;
    if (rdna::forwardInt8QK(p, stream) != 0) {
        set_error("Attention (int8qk) failed: %s", rdna::lastErrorInt8QK());
        return -3;
    }
    return 0;
}

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
    int32_t causal, int32_t window_size, void* scores, void* stream) {
    rdna::ForwardParamsInt8QK p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = output;
    p.qStrideB = q_stride_b;
    p.qStrideH = q_stride_h;
    p.qStrideS = q_stride_s;
    p.kStrideB = k_stride_b;
    p.kStrideH = k_stride_h;
    p.kStrideS = k_stride_s;
    p.vStrideB = v_stride_b;
    p.vStrideH = v_stride_h;
    p.vStrideS = v_stride_s;
    p.oStrideB = o_stride_b;
    p.oStrideH = o_stride_h;
    p.oStrideS = o_stride_s;
    p.batchSize = batch_size;
    p.numHeads = num_heads;
    p.numKvHeads = num_kv_heads;
    p.seqLen = seq_len;
    p.keySeqLen = key_seq_len;
    p.headDim = head_dim;
    p.scale = scale;
    p.qScale = q_scale;
    p.kScale = k_scale;
    p.vScale = v_scale;
    p.causal = causal != 0 ? 1u : 0u;
    p.windowSize = window_size;
    p.qScaleVec = q_scale_vec;
    p.kScaleVec = k_scale_vec;
    if (rdna::debugInt8QKScores(p, scores, stream) != 0) {
        set_error("Attention (int8qk) failed: %s", rdna::lastErrorInt8QK());
        return -3;
    }
    return 0;
}

// ForwardParamsInt8QK of the _vch entry points.
static rdna::ForwardParamsInt8QK i8_params(
    const void* q, const void* k, const void* v, void* output,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    float scale, float q_scale, float k_scale, float v_scale,
    const void* q_scale_vec, const void* k_scale_vec, const void* v_channel,
    int32_t causal, int32_t window_size) {
    rdna::ForwardParamsInt8QK p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = output;
    p.qStrideB = q_stride_b;
    p.qStrideH = q_stride_h;
    p.qStrideS = q_stride_s;
    p.kStrideB = k_stride_b;
    p.kStrideH = k_stride_h;
    p.kStrideS = k_stride_s;
    p.vStrideB = v_stride_b;
    p.vStrideH = v_stride_h;
    p.vStrideS = v_stride_s;
    p.oStrideB = o_stride_b;
    p.oStrideH = o_stride_h;
    p.oStrideS = o_stride_s;
    p.batchSize = batch_size;
    p.numHeads = num_heads;
    p.numKvHeads = num_kv_heads;
    p.seqLen = seq_len;
    p.keySeqLen = key_seq_len;
    p.headDim = head_dim;
    p.scale = scale;
    p.qScale = q_scale;
    p.kScale = k_scale;
    p.vScale = v_scale;
    p.causal = causal != 0 ? 1u : 0u;
    p.windowSize = window_size;
    p.qScaleVec = q_scale_vec;
    p.kScaleVec = k_scale_vec;
    p.vChannel = v_channel;
    return p;
}

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
    int32_t causal, int32_t window_size, void* stream) {
    const rdna::ForwardParamsInt8QK p =
        i8_params(q, k, v, output, q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h, k_stride_s,
                  v_stride_b, v_stride_h, v_stride_s, o_stride_b, o_stride_h, o_stride_s, batch_size, num_heads,
                  num_kv_heads, seq_len, key_seq_len, head_dim, scale, q_scale, k_scale, v_scale, q_scale_vec,
                  k_scale_vec, v_channel, causal, window_size);
    if (rdna::forwardInt8QK(p, stream) != 0) {
        set_error("Attention (int8qk) failed: %s", rdna::lastErrorInt8QK());
        return -3;
    }
    return 0;
}

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
    int32_t n_peers, void* const* peer_outputs, void* stream) {
    const rdna::ForwardParamsInt8QK p =
        i8_params(q, k, v, output, q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h, k_stride_s,
                  v_stride_b, v_stride_h, v_stride_s, o_stride_b, o_stride_h, o_stride_s, batch_size, num_heads,
                  num_kv_heads, seq_len, key_seq_len, head_dim, scale, q_scale, k_scale, v_scale, q_scale_vec,
                  k_scale_vec, v_channel, causal, window_size);
    if (rdna::forwardInt8QKPeers(p, n_peers, peer_outputs, stream) != 0) {
        set_error("Attention (int8qk) failed: %s", rdna::lastErrorInt8QK());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_int8_quantize_qkv(
    const void* q, const void* k, const void* v,
    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    uint32_t batch_size, uint32_t num_heads, uint32_t num_kv_heads,
    uint32_t seq_len, uint32_t key_seq_len, uint32_t head_dim,
    void* q_int8, void* k_int8, void* v_int8,
    void* q_scale, void* k_scale, void* v_channel, void* stream) {
    rdna::QuantizeInt8Params p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.qStrideB = q_stride_b;
    p.qStrideH = q_stride_h;
    p.qStrideS = q_stride_s;
    p.kStrideB = k_stride_b;
    p.kStrideH = k_stride_h;
    p.kStrideS = k_stride_s;
    p.vStrideB = v_stride_b;
    p.vStrideH = v_stride_h;
    p.vStrideS = v_stride_s;
    p.batchSize = batch_size;
    p.numHeads = num_heads;
    p.numKvHeads = num_kv_heads;
    p.seqLen = seq_len;
    p.keySeqLen = key_seq_len;
    p.headDim = head_dim;
    p.qInt8 = q_int8;
    p.kInt8 = k_int8;
    p.vInt8 = v_int8;
    p.qScale = q_scale;
    p.kScale = k_scale;
    p.vChannel = v_channel;
    if (rdna::quantizeInt8QKV(p, stream) != 0) {
        set_error("Attention (int8qk) failed: %s", rdna::lastErrorInt8QK());
        return -3;
    }
    return 0;
}

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
    void* stream) {
    const rdna::ForwardParams p = f16_params(q, k, v, output, rot_cos, rot_sin, q_stride_b, q_stride_h, q_stride_s,
                                             k_stride_b, k_stride_h, k_stride_s, v_stride_b, v_stride_h, v_stride_s,
                                             o_stride_b, o_stride_h, o_stride_s, batch_size, num_heads, num_kv_heads,
                                             seq_len, key_seq_len, head_dim, scale, causal, has_rope, window_size);
    if (rdna::forwardF16NoAlloc(p, stream) != 0) {
        set_error("Attention (fp16) failed: %s", rdna::lastError());
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_debug_read_status(int32_t* out2) {
    const char* why = nullptr;
    if (out2 == nullptr) {
        set_error("Debug status failed: %s", "null output pointer");
        return -3;
    }
    if (rdna::debugReadStatus(out2, &why) != 0) {
        set_error("Debug status failed: %s", why);
        return -3;
    }
    return 0;
}

RDNA_API int32_t rdna_debug_set_wait_test(int32_t withhold_block, uint64_t wait_limit_ns) {
    rdna::debugSetWaitTest(withhold_block, wait_limit_ns);
    return 0;
}

RDNA_API int32_t rdna_debug_set_kernel_events(void* start_event, void* stop_event) {
    rdna::debugSetKernelEvents(start_event, stop_event);
    return 0;
}
