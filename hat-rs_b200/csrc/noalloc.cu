// hat_b200_linear_noalloc: the kernel-level linear with every piece of scratch in one
// fixed, statically allocated device array, so that the call allocates no device memory.
//
// Who needs it: callers that must not allocate on this path. Examples are a process whose
// device memory is already reserved by another allocator (a framework's caching pool
// holding everything, where a cudaMalloc of a few MB fails), a latency-critical loop where
// an allocation and the synchronisation a cudaFree can bring are not acceptable, and a
// caller that must know the call's device-memory use before it runs.
//
// Scratch layout (floats, each region starting on a 256-byte boundary):
//   [0, 64)    the tensor-core kernels' error word (an int); zeroed by every call before
//              the first launch, because a nonzero value means "a wait gave up"
//   weights    n*k (CUDA-core copy) + 2*n_pad*k_pad (tf32 hi/lo tensor-core blocks)
//   operand    2*m*k (x split into tf32 hi/lo; fp32-parity mode only)
// Everything except the error word is fully rewritten by each call before it is read, so
// nothing else needs to start at zero.
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/hat_b200.h"
#include "umma.cuh"

namespace hat {

// 8 MiB: the largest scratch one call may use (HAT_B200_NOALLOC_SCRATCH_BYTES).
constexpr size_t NOALLOC_FLOATS = HAT_B200_NOALLOC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_FLOATS];

namespace {

size_t round64(size_t n) { return (n + 63) / 64 * 64; }

// The scratch array's address on the current device. In host code `g_noalloc_scratch`
// names a host-side stand-in, not device memory, so the device address is looked up with
// that device current. The lookup is repeated on every call rather than cached: a
// cudaDeviceReset or another context on the same ordinal loads the module again, and the
// array can then sit at a different address.
float* scratch_on_current_device() {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
        throw Error(3, std::string("hat_b200_linear_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    return static_cast<float*>(p);
}

void set_msg(char* err, size_t errlen, const std::string& m) {
    if (!err || errlen == 0) return;
    const size_t n = m.size() < errlen - 1 ? m.size() : errlen - 1;
    memcpy(err, m.data(), n);
    err[n] = 0;
}

}  // namespace
}  // namespace hat

using namespace hat;

extern "C" int hat_b200_linear_noalloc(int mode, const float* x, const float* w, const float* b, float* y, int m,
                                       int n, int k, void* stream, char* err, size_t errlen) {
    try {
        if (!x || !w || !y || m <= 0 || n <= 0 || k <= 0)
            throw Error(1, "hat_b200_linear_noalloc: null buffer or non-positive size");
        if (mode != HAT_B200_MODE_PARITY && mode != HAT_B200_MODE_FAST && mode != HAT_B200_MODE_SIMT)
            throw Error(1, "hat_b200_linear_noalloc: unknown mode " + std::to_string(mode));
        GemmW g;
        plan_gemm_w(g, n, k, false, 0);
        const bool split = mode == HAT_B200_MODE_PARITY;
        const size_t w_simt = round64((size_t)n * k);
        const size_t w_tc = g.umma ? round64((size_t)g.n_pad * g.k_pad) : 0;
        const size_t x_split = split ? round64((size_t)m * k) : 0;
        const size_t need = 64 + w_simt + 2 * w_tc + 2 * x_split;
        if (need > NOALLOC_FLOATS) {
            char buf[256];
            snprintf(buf, sizeof buf,
                     "hat_b200_linear_noalloc: m=%d n=%d k=%d needs %zu bytes of scratch; the limit is %zu bytes "
                     "(use hat_b200_linear, which allocates)",
                     m, n, k, need * sizeof(float), (size_t)HAT_B200_NOALLOC_SCRATCH_BYTES);
            throw Error(1, buf);
        }
        cudaStream_t st = (cudaStream_t)stream;
        float* s = scratch_on_current_device();
        int* derr = reinterpret_cast<int*>(s);
        float* simt = s + 64;
        float* hi = simt + w_simt;
        float* lo = hi + w_tc;
        float* xs = lo + w_tc;
        HAT_CUDA(cudaMemsetAsync(derr, 0, sizeof(int), st));
        launch_prep_gemm_w(w, simt, g.umma ? hi : nullptr, g.umma ? lo : nullptr, g, st);
        g.simt = simt;
        g.hi = hi;
        g.lo = lo;
        Opnd xo{x, nullptr};
        if (split) {
            launch_split(x, xs, xs + x_split, (long)m * k, st);
            xo = Opnd{xs, xs + x_split};
        }
        Epi e;
        e.bias = b;
        GemmCtx c{mode == HAT_B200_MODE_SIMT ? 0 : mode, mode == HAT_B200_MODE_SIMT, derr};
        gemm_linear(c, xo, g, Dst{y, nullptr}, m, e, st);
        int v = 0;
        HAT_CUDA(cudaMemcpyAsync(&v, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
        HAT_CUDA(cudaStreamSynchronize(st));
        if (v)
            throw Error(3, "hat_b200_linear_noalloc: tensor-core kernel gave up waiting on its pipeline (code " +
                               std::to_string(v) + ")");
        set_msg(err, errlen, "");
        return HAT_B200_OK;
    } catch (const Error& e) {
        set_msg(err, errlen, e.what());
        return e.code ? e.code : HAT_B200_EINVAL;
    } catch (const std::exception& e) {
        set_msg(err, errlen, e.what());
        return HAT_B200_EINVAL;
    }
}
