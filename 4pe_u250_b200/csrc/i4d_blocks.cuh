// i4d_blocks.cuh -- small kernels of the token schedule and the op-level API.
//
// RMSNorm reciprocal, normalise+quantise, G32 quantiser, SwiGLU+quantise and
// the element-wise expf hook.  The fused path runs the same device functions
// inside the GEMV prologues / epilogues (i4d_linear.cuh); these kernels serve
// the first norm of a token and the per-stage entry points.
#pragma once

#include "i4d_device.cuh"
#include "i4d_expf.cuh"

namespace i4d {

// r = RMS reciprocal of x[4096] (emulator:427-447).  One warp.
__global__ void __launch_bounds__(32) k_rms_recip(const float* x, float* out) {
    pdl_trigger();
    pdl_wait();
    const float r = rms_recip_warp(x);
    if (threadIdx.x == 0) *out = r;
}

// q = quantize(fl(fl(x * r) * gamma)) over 4096 (emulator:448-453).
__global__ void __launch_bounds__(128) k_norm_quant(const float* x, const float* gamma, const float* recip,
                                                     int16_t* q, uint8_t* e) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const float v = __fmul_rn(__fmul_rn(x[i], *recip), gamma[i]);
    uint32_t e8;
    q[i] = static_cast<int16_t>(quantize_g32_lane(v, &e8));
    if ((i & 31) == 0) e[i >> 5] = static_cast<uint8_t>(e8);
}

// G32 quantiser over n values (n % 32 == 0, grid covers n exactly).
__global__ void __launch_bounds__(128) k_quant_g32(const float* x, int n, int16_t* q, uint8_t* e) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if ((i & ~31) >= n) return;
    uint32_t e8;
    q[i] = static_cast<int16_t>(quantize_g32_lane(x[i], &e8));
    if ((i & 31) == 0) e[i >> 5] = static_cast<uint8_t>(e8);
}

// SwiGLU then G32 quantiser (emulator:716-722, 769-770).
__global__ void __launch_bounds__(128) k_swiglu_quant(const float* gate, const float* up, int n, ExpfFix fx,
                                                       int16_t* q, uint8_t* e) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if ((i & ~31) >= n) return;
    uint32_t e8;
    q[i] = static_cast<int16_t>(quantize_g32_lane(swiglu1(gate[i], up[i], fx), &e8));
    if ((i & 31) == 0) e[i >> 5] = static_cast<uint8_t>(e8);
}

// Writes the decode position into device memory (kernel argument, so an
// enqueued step never reads host memory that the caller may reuse).
__global__ void k_set_pos(int* dst, int pos) { *dst = pos; }

__global__ void k_expf(const float* x, float* y, size_t n, ExpfFix fx) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) y[i] = expf_libc(x[i], fx);
}

}  // namespace i4d
