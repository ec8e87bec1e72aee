// qmm_handles.h -- definitions of the opaque C-ABI handles, shared by the
// translation units that implement include/rce_qmm.h.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <thread>
#include <unordered_map>

#include "qmm_layout.cuh"

struct RceScratch {
    void *gemm_ws = nullptr;  // prefill GEMM workspace (fp16 activations, token scales)
    size_t gemm_ws_bytes = 0;
    void *moe_ws = nullptr;   // MoE FFN workspace (routes, rows, activations per row)
    size_t moe_ws_bytes = 0;
    int32_t *moe_host = nullptr;  // pinned copy of the per-expert row offsets
    size_t moe_host_n = 0;
};

struct RceThreadState {
    cudaStream_t stream = nullptr;
    float *d_in = nullptr;
    size_t d_in_cap = 0;
    float *d_out = nullptr;
    size_t d_out_cap = 0;
    void *h_pin = nullptr;
    size_t h_cap = 0;
    // Host-buffer decode calls replayed as CUDA graphs (copy in, matmul, copy
    // out: one launch instead of three API calls), keyed by weight serial and
    // batch; valid while the staging buffers above stay where they are.
    std::unordered_map<uint64_t, cudaGraphExec_t> graphs;
};

struct rce_qmm_ctx {
    int device = 0;
    int sm_count = 148;
    // Error word the kernels write when a bounded wait expires: mapped,
    // pinned host memory, so the host reads it without a copy.
    int *err_host = nullptr;
    int *err_dev = nullptr;
    // mm_batched runs the tensor-core prefill GEMM from this many tokens on
    // (0: never; every token then takes the exact decode path).
    int prefill_min_tokens = 16;
    std::mutex mu;
    std::unordered_map<cudaStream_t, RceScratch> scratch;
    std::unordered_map<std::thread::id, RceThreadState> threads;
};

struct rce_qmm_weight {
    rce_qmm_ctx *ctx = nullptr;
    uint64_t serial = 0;  // unique per handle (a freed handle's address may be reused; its serial is not)
    int dtype = 0;
    rce::Geometry g;
    uint8_t *dev = nullptr;
    bool owner = false;
};

// Records `msg` as the calling thread's rce_qmm_last_error() and returns code.
int rce_qmm_set_error(int code, const char *msg);
