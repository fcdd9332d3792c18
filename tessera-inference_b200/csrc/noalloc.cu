// An allocation-free entry point: the GEMM + residual + LayerNorm op of
// tcb_op_gemm_ln, for callers that must not allocate device memory.
//
// Who cannot allocate: a host program that hands this library a fixed device
// memory budget at start-up (for example an inference-server plugin whose
// framework owns all device memory and forbids allocation while it enqueues
// work), or any caller on a hot path where cudaMalloc is off limits because
// it can fail under a full budget and implicitly synchronises the device.
// Such a caller passes only its inputs and outputs; the intermediate this op
// needs (the bf16 pre-LayerNorm rows y, M x 640) and its status word live in
// one file-scope __device__ array of fixed size, created when the library's
// code is loaded on a GPU and held by every GPU that loads the library until
// the process exits.
//
// The op runs as two launches of the existing kernels: the single-CTA tcgen05
// GEMM writes y = bf16(A W^T + bias + residual) into the array, then the
// LayerNorm kernel writes out = bf16(LN(y) * g + b).
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm_sm100.h"
#include "kernels.h"
#include "tessera_b200_ops.h"

namespace tcb {
namespace {

constexpr int NOALLOC_MAX_ROWS = 8192;                 // largest M one call accepts
constexpr size_t NOALLOC_Y_OFFSET = 256;               // [0, 256): status word
constexpr size_t NOALLOC_BYTES = NOALLOC_Y_OFFSET + (size_t)NOALLOC_MAX_ROWS * D * sizeof(bf16);  // 10 MiB + 256 B

// Device scratch shared by every call on a device. In host code this name is
// only a stand-in: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

std::mutex g_mu;
void *g_scratch_addr[64] = {};  // per device ordinal

// Device address of the scratch array on the current device, looked up once
// per device (the first call on a device does this set-up).
void *scratch_on_current_device() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) throw std::runtime_error("device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            throw std::runtime_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    return g_scratch_addr[dev];
}

}  // namespace
}  // namespace tcb

using namespace tcb;

extern "C" int tcb_op_gemm_ln_noalloc(const void *A, int lda, const void *W, const float *bias, const void *res,
                                      int ldr, const float *ln_g, const float *ln_b, void *out, int M, int K,
                                      void *stream) {
    try {
        if (M < 0 || M > NOALLOC_MAX_ROWS)
            throw std::runtime_error("M = " + std::to_string(M) + " is outside [0, " +
                                     std::to_string(NOALLOC_MAX_ROWS) + "], the size of the static scratch");
        if (!A || !W || !ln_g || !ln_b || !out) throw std::runtime_error("null pointer");
        if (M == 0) return 0;
        uint8_t *base = static_cast<uint8_t *>(scratch_on_current_device());
        int *status = reinterpret_cast<int *>(base);
        bf16 *y = reinterpret_cast<bf16 *>(base + NOALLOC_Y_OFFSET);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        // the array keeps the previous call's contents: the status word must start at zero
        cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
        if (e != cudaSuccess) throw std::runtime_error(std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
        GemmArgs p;
        p.M = M;
        p.N = D;
        p.K = K;
        p.bias = bias;
        p.res = static_cast<const bf16 *>(res);
        p.ldr = ldr;
        p.out = y;
        p.ldo = D;
        p.status = status;
        launch_gemm(p, static_cast<const bf16 *>(A), lda, static_cast<const bf16 *>(W), st, 0, 0, 1);
        launch_layernorm640(y, M, ln_g, ln_b, static_cast<bf16 *>(out), st);
        // the status word is read back on the caller's stream, behind the two
        // kernels, and one wait on that stream covers all three: no other
        // stream of the device is waited for
        int s = 0;
        e = cudaMemcpyAsync(&s, status, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) throw std::runtime_error(std::string("status read: ") + cudaGetErrorString(e));
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) throw std::runtime_error(std::string("stream: ") + cudaGetErrorString(e));
        if (s != 0) throw std::runtime_error("device status " + std::to_string(s));
        return 0;
    } catch (const std::exception &ex) {
        std::fprintf(stderr, "tcb_op_gemm_ln_noalloc: %s\n", ex.what());
        return -1;
    }
}
