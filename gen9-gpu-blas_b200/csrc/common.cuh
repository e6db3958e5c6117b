// common.cuh -- device helpers shared by the kernels: element types, 16-byte vector access, conversions.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace g9 {

// Compute type R of a storage type T: FP16 and FP32 compute in FP32, FP64 in FP64 (as the reference's level12.cl:6-65).
template <typename T> struct Compute { using R = T; };
template <> struct Compute<__half> { using R = float; };

template <typename T> __device__ __forceinline__ typename Compute<T>::R to_r(T v) { return v; }
template <> __device__ __forceinline__ float to_r<__half>(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_r(typename Compute<T>::R v) { return v; }
template <> __device__ __forceinline__ __half from_r<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float fma_r(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_r(double a, double b, double c) { return __fma_rn(a, b, c); }

// 16-byte vector of T: W elements.
template <typename T> struct V16;
template <> struct V16<float> { static constexpr int W = 4; };
template <> struct V16<double> { static constexpr int W = 2; };
template <> struct V16<__half> { static constexpr int W = 8; };

// Loads 16 bytes (aligned) through the read-only path and widens to R.
template <typename T> __device__ __forceinline__ void load16(const T *p, typename Compute<T>::R *out);
template <> __device__ __forceinline__ void load16<float>(const float *p, float *o) {
    float4 v = __ldg(reinterpret_cast<const float4 *>(p));
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
template <> __device__ __forceinline__ void load16<double>(const double *p, double *o) {
    double2 v = __ldg(reinterpret_cast<const double2 *>(p));
    o[0] = v.x; o[1] = v.y;
}
template <> __device__ __forceinline__ void load16<__half>(const __half *p, float *o) {
    uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __half22float2(h[i]);
        o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
}
// Plain (coherent) 16-byte load, for data the same kernel may also write.
template <typename T> __device__ __forceinline__ void load16_rw(const T *p, typename Compute<T>::R *out);
template <> __device__ __forceinline__ void load16_rw<float>(const float *p, float *o) {
    float4 v = *reinterpret_cast<const float4 *>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
template <> __device__ __forceinline__ void load16_rw<double>(const double *p, double *o) {
    double2 v = *reinterpret_cast<const double2 *>(p);
    o[0] = v.x; o[1] = v.y;
}
template <> __device__ __forceinline__ void load16_rw<__half>(const __half *p, float *o) {
    uint4 v = *reinterpret_cast<const uint4 *>(p);
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __half22float2(h[i]);
        o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
}
// Narrows W values of R to T (round to nearest even) and stores 16 bytes (aligned).
template <typename T> __device__ __forceinline__ void store16(T *p, const typename Compute<T>::R *v);
template <> __device__ __forceinline__ void store16<float>(float *p, const float *v) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <> __device__ __forceinline__ void store16<double>(double *p, const double *v) {
    *reinterpret_cast<double2 *>(p) = make_double2(v[0], v[1]);
}
template <> __device__ __forceinline__ void store16<__half>(__half *p, const float *v) {
    uint4 u;
    __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = u;
}

__device__ __forceinline__ bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// ggml GELU, tanh form, with the FP16 rounding of ggml-cpu's table (x <= -10: 0, x >= 10: x, else
// fp16(gelu(fp16(x)))); written with explicit roundings so that no multiply-add is contracted. Shared by the
// elementwise op and the fused GEMM epilogue, so that both give the same bits.
__device__ __forceinline__ float gelu_ggml(float v) {
    if (v <= -10.0f) return 0.0f;
    if (v >= 10.0f) return v;
    const float h = __half2float(__float2half_rn(v));
    const float hh = __fmul_rn(h, h);
    const float inner = __fmul_rn(__fmul_rn(0.79788456080286535588f, h), __fadd_rn(1.0f, __fmul_rn(0.044715f, hh)));
    const float g = __fmul_rn(__fmul_rn(0.5f, h), __fadd_rn(1.0f, tanhf(inner)));
    return __half2float(__float2half_rn(g));
}

}  // namespace g9
