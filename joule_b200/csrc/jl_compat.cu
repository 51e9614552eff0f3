// The reference's own Q4 GEMV / GEMM symbols, with its exact signatures.
//
// The reference's Python binds two functions by name through its single
// loader, get_dll(name) (src/jouleai/native/backend.py:32-42):
//   get_dll("quant_gemv").q4_gemv_f32(out, x, packed, scales, m, d, group)
//     (kernel.py:15-41, ScalarBackend backend.py:72-91; quant_gemv.c:35-57)
//   get_dll("expert_ffn").q4_gemm_f32(out, X, T, packed, scales, m, d, group)
//     (kernel.py:43-62, AVX2Backend backend.py:94-116; expert_ffn.c:200-215)
// Both take HOST pointers, return void and finish before returning. These
// exports keep that contract on the GPU: the inputs are copied to device
// buffers that this file caches per device (grown on demand), the kernel runs
// on a library-owned stream, and the result is copied back before return.
//
// Arithmetic: q4_gemv_f32 follows quant_gemv.c's scalar loop (per byte
// gacc += lo*x0 + hi*x1, then acc += gacc*s per group), so it equals
// ScalarBackend bit for bit; q4_gemm_f32 follows expert_ffn.c's AVX2 row dot,
// as jl_q4_gemm_f32 does (that kernel is reused here).
//
// Errors: the reference's functions return void, so a failed call (bad
// argument, no device, CUDA error) fills `out` with NaN, which no caller can
// mistake for a result, and records the status for jl_compat_status().
#include <cmath>
#include <cstring>
#include <limits>
#include <mutex>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace {

constexpr int kCompatDevices = 128;

struct compat_dev {
    cudaStream_t st = nullptr;
    void* buf = nullptr;
    size_t bytes = 0;
};

std::mutex g_compat_mu;
compat_dev g_compat[kCompatDevices];
thread_local int t_compat_status = JL_OK;

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

// quant_gemv.c:35-57, one warp per row. Lane j computes group g0 + j's
// sequential byte chain; lane 0 then adds the group products in group order.
__global__ void k_q4_gemv_scalar(float* __restrict__ out, const float* __restrict__ x,
                                 const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                                 int m, int d) {
    const int row = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= m) return;
    const int nb = d / 2, ng = d / jl::kGroup;
    const uint8_t* r = packed + (size_t)row * nb;
    const uint16_t* sc = scales + (size_t)row * ng;
    float acc = 0.0f;
    for (int g0 = 0; g0 < ng; g0 += 32) {
        const int g = g0 + lane;
        float p = 0.0f;
        if (g < ng) {
            float gacc = 0.0f;
            for (int b = g * 32; b < g * 32 + 32; b++) {
                const uint32_t byte = r[b];
                const float t1 = __fmul_rn((float)((int)(byte & 15u) - 8), x[2 * b]);
                const float t2 = __fmul_rn((float)((int)(byte >> 4) - 8), x[2 * b + 1]);
                gacc = __fadd_rn(gacc, __fadd_rn(t1, t2));
            }
            p = __fmul_rn(gacc, jl::fp16_to_f32(sc[g]));
        }
        const int n = min(32, ng - g0);
        for (int j = 0; j < n; j++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, p, j));
    }
    if (lane == 0) out[row] = acc;
}

void fill_nan(float* out, size_t n) {
    if (!out) return;
    const float q = std::numeric_limits<float>::quiet_NaN();
    for (size_t i = 0; i < n; i++) out[i] = q;
}

// Device buffers of at least `need` bytes and the stream of the current
// device. Called with g_compat_mu held.
int compat_buffers(size_t need, compat_dev** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return jl_note_cuda(e);
    if (dev < 0 || dev >= kCompatDevices) return JL_ERR_INVALID;
    compat_dev& c = g_compat[dev];
    if (!c.st) {
        e = cudaStreamCreateWithFlags(&c.st, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            c.st = nullptr;
            return jl_note_cuda(e);
        }
    }
    if (c.bytes < need) {
        if (c.buf) cudaFree(c.buf);
        c.buf = nullptr;
        c.bytes = 0;
        e = cudaMalloc(&c.buf, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return JL_ERR_OOM;
        }
        c.bytes = need;
    }
    *out = &c;
    return JL_OK;
}

// Shared body: T = 0 selects the scalar GEMV (x is one row), T >= 1 the GEMM.
int compat_run(float* out, const float* X, int T, const unsigned char* packed,
               const unsigned short* scales, int m, int d, int group) {
    const bool gemv = T == 0;
    const int rows = gemv ? 1 : T;
    if (!out || !X || !packed || !scales || m <= 0 || d <= 0 || rows <= 0) return JL_ERR_INVALID;
    if (group != jl::kGroup || d % jl::kGroup) return JL_ERR_INVALID;
    const size_t pkb = (size_t)m * d / 2, scb = (size_t)m * (d / jl::kGroup) * 2;
    const size_t xb = (size_t)rows * d * 4, ob = (size_t)rows * m * 4;
    const size_t o_pk = 0, o_sc = up256(pkb), o_x = o_sc + up256(scb), o_o = o_x + up256(xb);
    std::lock_guard<std::mutex> lk(g_compat_mu);
    compat_dev* c = nullptr;
    int rc = compat_buffers(o_o + up256(ob), &c);
    if (rc) return rc;
    uint8_t* b = static_cast<uint8_t*>(c->buf);
    JL_CUDA(cudaMemcpyAsync(b + o_pk, packed, pkb, cudaMemcpyHostToDevice, c->st));
    JL_CUDA(cudaMemcpyAsync(b + o_sc, scales, scb, cudaMemcpyHostToDevice, c->st));
    JL_CUDA(cudaMemcpyAsync(b + o_x, X, xb, cudaMemcpyHostToDevice, c->st));
    float* od = reinterpret_cast<float*>(b + o_o);
    if (gemv) {
        const int tpb = 256;
        const size_t threads = (size_t)m * 32;
        k_q4_gemv_scalar<<<(unsigned)((threads + tpb - 1) / tpb), tpb, 0, c->st>>>(
            od, reinterpret_cast<const float*>(b + o_x), b + o_pk,
            reinterpret_cast<const uint16_t*>(b + o_sc), m, d);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return jl_note_cuda(e);
    } else {
        rc = jl_q4_gemm_f32(od, reinterpret_cast<const float*>(b + o_x), T, b + o_pk,
                            reinterpret_cast<const unsigned short*>(b + o_sc), m, d, group, c->st);
        if (rc) return rc;
    }
    JL_CUDA(cudaMemcpyAsync(out, od, ob, cudaMemcpyDeviceToHost, c->st));
    JL_CUDA(cudaStreamSynchronize(c->st));
    return JL_OK;
}

}  // namespace

extern "C" void q4_gemv_f32(float* out, const float* x, const unsigned char* packed,
                            const unsigned short* scales, int m, int d, int group) {
    t_compat_status = compat_run(out, x, 0, packed, scales, m, d, group);
    if (t_compat_status != JL_OK && m > 0) fill_nan(out, (size_t)m);
}

extern "C" void q4_gemm_f32(float* out, const float* X, int T, const unsigned char* packed,
                            const unsigned short* scales, int m, int d, int group) {
    if (T == 0) {  // the reference's loop runs zero times
        t_compat_status = JL_OK;
        return;
    }
    t_compat_status = T < 0 ? JL_ERR_INVALID : compat_run(out, X, T, packed, scales, m, d, group);
    if (t_compat_status != JL_OK && m > 0 && T > 0) fill_nan(out, (size_t)T * m);
}

extern "C" int jl_compat_status(void) { return t_compat_status; }
