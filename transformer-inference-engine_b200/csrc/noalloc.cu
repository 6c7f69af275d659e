// noalloc.cu -- the greedy head (tied-embedding GEMV + argmax) for callers that
// cannot allocate device memory.
//
// Who needs it: code that runs the head inside a host program whose device
// memory is owned by someone else -- a serving framework whose caching
// allocator has reserved the GPU's memory up front, a plugin loaded into a
// runtime that forbids allocations outside its own allocator, or a latency-
// bound loop that cannot afford cudaMalloc's implicit device synchronisation.
// The regular path keeps its per-block partial maxima in a buffer the model
// allocates; this entry point keeps them in a fixed array compiled into the
// library instead, so a call allocates nothing.
//
// The array lives in every GPU that loads this library, for the life of the
// process (512 KiB). Its address is looked up on the first call made with a
// device current (cudaGetSymbolAddress, which also makes the device's primary
// context current if it is not yet); that first call on a device should come
// before any stream capture. The address is kept together with the context it belongs to and
// looked up again when a call finds another context current (after
// cudaDeviceReset, for instance). All calls share the one array: two calls
// that overlap on the GPU (different streams, or different host threads on one
// device) race on it. Nothing in it needs to start at zero -- every partial the
// final reduction reads is written earlier by the same call.
#include <cuda.h>

#include "../../include/tie_b200.h"
#include "common.cuh"

#include <mutex>

namespace {

constexpr int kMaxRows = 16;          // hidden-state rows per call
constexpr int kMaxVocab = 65536;      // vocabulary rows of the head
constexpr int kMaxBlocks = kMaxVocab / tie::kGemvArgmaxRowsPerBlock;
constexpr size_t kScratchBytes = (size_t)kMaxBlocks * kMaxRows * (sizeof(float) + sizeof(int));

// per-block partial maxima: kMaxBlocks x kMaxRows values, then as many indices
static __device__ __align__(256) unsigned char g_head_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct ScratchAddr {
    CUcontext ctx = nullptr;
    void* ptr = nullptr;
};
ScratchAddr g_scratch[kMaxDevices];

// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link the driver library directly, so it loads on machines without one)
CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        fn = reinterpret_cast<Fn>(p);
    }
    CUcontext ctx = nullptr;
    return fn(&ctx) == CUDA_SUCCESS ? ctx : nullptr;
}

// The device address of g_head_scratch in the current device's context.
cudaError_t scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lock(g_mu);
    ScratchAddr& s = g_scratch[dev];
    if (!s.ptr || !ctx || ctx != s.ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_head_scratch);
        if (e != cudaSuccess) return e;
        ctx = current_context();
        s.ptr = p;
        s.ctx = ctx;
    }
    *out = s.ptr;
    return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" model_status tie_head_argmax_noalloc(const float* x, int ldx, const float* w, int ldw,
                                                int rows, int vocab, int k, float* logits, int ldl,
                                                int32_t* next, void* stream) {
    if (!x || !w || !next || rows <= 0 || vocab <= 0 || k <= 0) return MODEL_ERR_ARG;
    if ((k & 3) || (ldx & 3) || (ldw & 3) || ldx < k || ldw < k || !aligned16(x) || !aligned16(w))
        return MODEL_ERR_ARG;
    if (logits && ldl < vocab) return MODEL_ERR_ARG;
    if (rows > kMaxRows || vocab > kMaxVocab) return MODEL_ERR_CAPACITY;
    // the head kernel writes one partial per (block, row): never past the array
    const int blocks = tie::gemv_argmax_blocks(vocab);
    if (blocks > kMaxBlocks) return MODEL_ERR_CAPACITY;
    void* scratch = nullptr;
    if (scratch_for_current_device(&scratch) != cudaSuccess) { cudaGetLastError(); return MODEL_ERR_DEVICE; }
    float* part_val = static_cast<float*>(scratch);
    int* part_idx = reinterpret_cast<int*>(static_cast<unsigned char*>(scratch) +
                                           (size_t)kMaxBlocks * kMaxRows * sizeof(float));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (tie::launch_gemv_argmax(x, ldx, w, ldw, logits, ldl, rows, vocab, k, part_val, part_idx, st) !=
            cudaSuccess ||
        tie::launch_argmax_finalize(part_val, part_idx, blocks, rows, next, st) != cudaSuccess) {
        cudaGetLastError();
        return MODEL_ERR_DEVICE;
    }
    return MODEL_OK;
}
