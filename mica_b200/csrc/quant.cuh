// quant.cuh -- per-token int8 activation quantiser and the fused RMSNorm + quantiser.
//
// One CTA per token row; each thread keeps up to QV vectors of 8 elements in registers,
// so the row is read from HBM once (the reference kernel, v0.5/serving/kernel_src/
// kernels.py:15-38, reads it twice: one pass for the absmax, one for the codes).
// Memory-bound: per row 2K (bf16 in) + K (int8 out) + 4 bytes, plus y/sum when requested.
#pragma once

#include "common.cuh"

namespace mica {

constexpr int QV = 4;  // 8-element vectors cached per thread (K <= 1024 * 32)

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (std::is_same<T, __half>::value) {
                const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
                f[2 * i] = __low2float(h);
                f[2 * i + 1] = __high2float(h);
            } else {
                f[2 * i] = __uint_as_float(w[i] << 16);
                f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
            }
        }
    }
}

template <typename T>
__device__ __forceinline__ float round_to(float x) {
    if constexpr (std::is_same<T, __half>::value) return __half2float(__float2half_rn(x));
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(x));
    else return x;
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
    if constexpr (sizeof(T) == 4) {
        reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (std::is_same<T, __half>::value) {
                __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            } else {
                __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Block-wide reduction; every thread gets the result. `red` holds 32 floats.
template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int nw = (blockDim.x + 31) >> 5;
    v = MAX ? warp_max(v) : warp_sum(v);
    __syncthreads();                 // `red` may still be read from the previous reduction
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = l < nw ? red[l] : (MAX ? 0.f : 0.f);
    r = MAX ? warp_max(r) : warp_sum(r);
    return r;
}

struct QuantArgs {
    const void* x; long ldx;
    const void* residual; long ldr;
    const void* gamma; int norm_style; float eps;
    const float* inv;
    void* y_out; long ldy;
    void* sum_out; long ldsum;
    int8_t* q; long ldq;
    float* s;
    int M, K, round_mode;
};

template <int MODE>
__device__ __forceinline__ void store_codes(const float (&v)[QV][8], int nvec, float scale, float rscale, int8_t* qr) {
#pragma unroll
    for (int i = 0; i < QV; ++i) {
        const int idx = threadIdx.x + i * blockDim.x;
        if (idx < nvec) *reinterpret_cast<uint2*>(qr + idx * 8) = quant8<MODE>(v[i], scale, rscale);
    }
}

// Element-wise |.| max of eight packed 16-bit floats into `m` (exact: the max of bf16/fp16
// values is one of them, so converting the final max to fp32 equals the fp32 max).
template <typename T>
__device__ __forceinline__ void absmax8(const uint4& w, uint32_t& m) {
    using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
    T2 acc = *reinterpret_cast<const T2*>(&m);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = __hmax2(acc, __habs2(*reinterpret_cast<const T2*>(&ws[j])));
    m = *reinterpret_cast<const uint32_t*>(&acc);
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<T, __half>::value) {
            const __half2 h = *reinterpret_cast<const __half2*>(&ws[i]);
            f[2 * i] = __low2float(h);
            f[2 * i + 1] = __high2float(h);
        } else {
            f[2 * i] = __uint_as_float(ws[i] << 16);
            f[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
        }
    }
}

// mica_act_quant on 16-bit input without a smoothing vector (quant_rows_packed_kernel): the
// row stays packed in registers (half the registers of an fp32 copy) and the absmax runs on
// packed pairs.
template <typename T, int MODE, int QV = mica::QV>
__device__ __forceinline__ void quant_row_packed(const QuantArgs& a, float* red) {
    const int row = blockIdx.x;
    const int nvec = a.K >> 3;
    const T* xr = static_cast<const T*>(a.x) + static_cast<long>(row) * a.ldx;
    uint4 w[QV];
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < QV; ++i) {
        const int idx = threadIdx.x + i * blockDim.x;
        w[i] = idx < nvec ? __ldg(reinterpret_cast<const uint4*>(xr + idx * 8)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < QV; ++i) absmax8<T>(w[i], m);
    float am;
    if constexpr (std::is_same<T, __half>::value) {
        const __half2 h = *reinterpret_cast<const __half2*>(&m);
        am = fmaxf(__low2float(h), __high2float(h));
    } else {
        am = fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
    }
    am = block_reduce<true>(am, red);
    const float scale = __fdiv_rn(fmaxf(am, 1e-8f), 127.0f);
    const float rscale = __frcp_rn(scale);
    int8_t* qr = a.q + static_cast<long>(row) * a.ldq;
#pragma unroll
    for (int i = 0; i < QV; ++i) {
        const int idx = threadIdx.x + i * blockDim.x;
        if (idx < nvec) {
            float f[8];
            unpack8<T>(w[i], f);
            *reinterpret_cast<uint2*>(qr + idx * 8) = quant8<MODE>(f, scale, rscale);
        }
    }
    if (threadIdx.x == 0) a.s[row] = scale;
}

// What a row goes through before the quantiser.
enum QuantKind {
    QK_PLAIN = 0,    // mica_act_quant: x as is
    QK_NORM = 1,     // mica_rmsnorm_quant: residual add, RMSNorm
    QK_SWIGLU = 2,   // mica_swiglu_quant: h = RN(RN(silu(g)) * u) with g = x, u = residual
};

// MAXT bounds the block size (512 for rows up to 16384 elements, 1024 beyond), which bounds
// registers per thread.
template <typename T, int KIND, int MAXT = 512>
__global__ void __launch_bounds__(MAXT) quant_rows_kernel(const QuantArgs a) {
    constexpr bool NORM = KIND == QK_NORM;
    __shared__ float red[32];
    const int row = blockIdx.x;
    const int nvec = a.K >> 3;
    const T* xr = static_cast<const T*>(a.x) + static_cast<long>(row) * a.ldx;
    float v[QV][8];
#pragma unroll
    for (int i = 0; i < QV; ++i) {
        const int idx = threadIdx.x + i * blockDim.x;
        if (idx < nvec) {
            load8(xr + idx * 8, v[i]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
        }
    }

    if constexpr (NORM) {
        if (a.residual != nullptr) {
            const T* rr = static_cast<const T*>(a.residual) + static_cast<long>(row) * a.ldr;
#pragma unroll
            for (int i = 0; i < QV; ++i) {
                const int idx = threadIdx.x + i * blockDim.x;
                if (idx < nvec) {
                    float r[8];
                    load8(rr + idx * 8, r);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[i][e] = round_to<T>(__fadd_rn(v[i][e], r[e]));
                    if (a.sum_out != nullptr)
                        store8(static_cast<T*>(a.sum_out) + static_cast<long>(row) * a.ldsum + idx * 8, v[i]);
                }
            }
        }
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < QV; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(v[i][e], v[i][e]));
        ss = block_reduce<false>(ss, red);
        const float rs = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.K)), a.eps));
        const T* gp = static_cast<const T*>(a.gamma);
#pragma unroll
        for (int i = 0; i < QV; ++i) {
            const int idx = threadIdx.x + i * blockDim.x;
            if (idx < nvec) {
                float w[8];
                load8(gp + idx * 8, w);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float n = __fmul_rn(v[i][e], rs);
                    v[i][e] = a.norm_style == MICA_NORM_OFFSET ? round_to<T>(__fmul_rn(n, __fadd_rn(1.0f, w[e])))
                                                               : round_to<T>(__fmul_rn(w[e], round_to<T>(n)));
                }
                if (a.y_out != nullptr)
                    store8(static_cast<T*>(a.y_out) + static_cast<long>(row) * a.ldy + idx * 8, v[i]);
            }
        }
    }

    if constexpr (KIND == QK_SWIGLU) {
        // fused_kernels.swiglu (lib/fused_kernels.py:37-44): silu in fp32 rounded to the
        // activation dtype, times u, rounded again; silu as in the fused GEMM epilogue.
        const T* ur = static_cast<const T*>(a.residual) + static_cast<long>(row) * a.ldr;
#pragma unroll
        for (int i = 0; i < QV; ++i) {
            const int idx = threadIdx.x + i * blockDim.x;
            if (idx < nvec) {
                float u[8];
                load8(ur + idx * 8, u);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float g = v[i][e];
                    const float act = round_to<T>(__fdividef(g, 1.0f + __expf(-g)));
                    v[i][e] = round_to<T>(__fmul_rn(act, u[e]));
                }
                if (a.y_out != nullptr)
                    store8(static_cast<T*>(a.y_out) + static_cast<long>(row) * a.ldy + idx * 8, v[i]);
            }
        }
    }

    if (KIND != QK_PLAIN && a.q == nullptr) return;  // norm-only / swiglu-only call
    if (a.inv != nullptr) {
#pragma unroll
        for (int i = 0; i < QV; ++i) {
            const int idx = threadIdx.x + i * blockDim.x;
            if (idx < nvec) {
                const float4 i0 = __ldg(reinterpret_cast<const float4*>(a.inv + idx * 8));
                const float4 i1 = __ldg(reinterpret_cast<const float4*>(a.inv + idx * 8) + 1);
                const float iv[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) v[i][e] = __fmul_rn(v[i][e], iv[e]);
            }
        }
    }
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < QV; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(v[i][e]));
    am = block_reduce<true>(am, red);
    const float scale = __fdiv_rn(fmaxf(am, 1e-8f), 127.0f);
    const float rscale = __frcp_rn(scale);
    int8_t* qr = a.q + static_cast<long>(row) * a.ldq;
    if (a.round_mode == MICA_ROUND_HALF_EVEN) store_codes<MICA_ROUND_HALF_EVEN>(v, nvec, scale, rscale, qr);
    else store_codes<MICA_ROUND_HALF_AWAY>(v, nvec, scale, rscale, qr);
    if (threadIdx.x == 0) a.s[row] = scale;
}

// mica_act_quant on 16-bit rows without a smoothing vector, QVP vectors of 8 elements per
// thread (quant_row_packed): wide rows take 8 per thread, so a row needs half the threads,
// its two reductions are shallower and more rows fit on an SM.
template <typename T, int QVP>
__global__ void __launch_bounds__(512) quant_rows_packed_kernel(const QuantArgs a) {
    __shared__ float red[32];
    if (a.round_mode == MICA_ROUND_HALF_EVEN) quant_row_packed<T, MICA_ROUND_HALF_EVEN, QVP>(a, red);
    else quant_row_packed<T, MICA_ROUND_HALF_AWAY, QVP>(a, red);
}

// ---- residual add + RMSNorm + quantiser, one warp per row ----------------------------------
// For rows up to 32 x 8 x MAXV elements (the 4B model's hidden 2560 needs MAXV = 10). No block
// barriers: the row (after the residual add, rounded to T) stays packed in registers, a
// 128-thread block holds four rows, and rows up to 2560 wide are held to 96 registers so that
// five blocks (20 rows) fit on an SM, against ~11 rows for the block-per-row form. Same
// arithmetic per element as quant_rows_kernel<T, QK_NORM>; the sum of squares runs per lane,
// then over a warp tree (a different order than the block form).
template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<T, __half>::value) {
            __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        } else {
            __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T, int MAXV, int MODE>
__device__ __forceinline__ void norm_row_warp(const QuantArgs& a, long row, int lane) {
    const int nvec = a.K >> 3;
    // distinct buffers: restrict lets the compiler issue later vectors' loads ahead of
    // earlier vectors' stores
    const T* __restrict__ xr = static_cast<const T*>(a.x) + row * a.ldx;
    T* __restrict__ sum_row = a.sum_out ? static_cast<T*>(a.sum_out) + row * a.ldsum : nullptr;
    T* __restrict__ y_row = a.y_out ? static_cast<T*>(a.y_out) + row * a.ldy : nullptr;
    const T* __restrict__ gp = static_cast<const T*>(a.gamma);
    const float* __restrict__ inv = a.inv;
    uint4 v[MAXV];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + 32 * i;
        v[i] = idx < nvec ? __ldg(reinterpret_cast<const uint4*>(xr + idx * 8)) : make_uint4(0u, 0u, 0u, 0u);
    }
    if (a.residual != nullptr) {
        const T* __restrict__ rr = static_cast<const T*>(a.residual) + row * a.ldr;
        uint4 rv[MAXV];
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + 32 * i;
            rv[i] = idx < nvec ? __ldg(reinterpret_cast<const uint4*>(rr + idx * 8)) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + 32 * i;
            if (idx < nvec) {
                float f[8], r[8];
                unpack8<T>(v[i], f);
                unpack8<T>(rv[i], r);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = __fadd_rn(f[e], r[e]);   // rounded to T by the pack
                v[i] = pack8<T>(f);
                if (sum_row != nullptr) *reinterpret_cast<uint4*>(sum_row + idx * 8) = v[i];
            }
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        if (lane + 32 * i < nvec) {
            float f[8];
            unpack8<T>(v[i], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(f[e], f[e]));
        }
    }
    ss = warp_sum(ss);
    const float rs = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.K)), a.eps));
    float am = 0.f;
    if (a.norm_style == MICA_NORM_WEIGHT && inv == nullptr) {
        // y = T(w * T(x * rs)) on packed pairs: the fp32 products x * rs go to T as one packed
        // pair (cvt.rn), and w * h is a packed T multiply -- the single rounding of the exact
        // product of two T values, which is what the fp32 multiply and cast give. The absmax
        // runs on the packed pairs too (exact: the max is one of the values).
        using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
        uint32_t am2 = 0u;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + 32 * i;
            if (idx < nvec) {
                float f[8];
                unpack8<T>(v[i], f);
                const uint4 wv = __ldg(reinterpret_cast<const uint4*>(gp + idx * 8));
                const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
                uint32_t ys[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    T2 h;
                    if constexpr (std::is_same<T, __half>::value)
                        h = __floats2half2_rn(__fmul_rn(f[2 * j], rs), __fmul_rn(f[2 * j + 1], rs));
                    else
                        h = __floats2bfloat162_rn(__fmul_rn(f[2 * j], rs), __fmul_rn(f[2 * j + 1], rs));
                    const T2 y = __hmul2_rn(*reinterpret_cast<const T2*>(&ws[j]), h);
                    ys[j] = *reinterpret_cast<const uint32_t*>(&y);
                }
                v[i] = make_uint4(ys[0], ys[1], ys[2], ys[3]);
                if (y_row != nullptr) *reinterpret_cast<uint4*>(y_row + idx * 8) = v[i];
                absmax8<T>(v[i], am2);
            }
        }
        const T2 m2 = *reinterpret_cast<const T2*>(&am2);
        am = fmaxf(__low2float(m2), __high2float(m2));
    } else {
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + 32 * i;
            if (idx < nvec) {
                float f[8], w[8];
                unpack8<T>(v[i], f);
                unpack8<T>(__ldg(reinterpret_cast<const uint4*>(gp + idx * 8)), w);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float n = __fmul_rn(f[e], rs);
                    f[e] = a.norm_style == MICA_NORM_OFFSET ? round_to<T>(__fmul_rn(n, __fadd_rn(1.0f, w[e])))
                                                            : round_to<T>(__fmul_rn(w[e], round_to<T>(n)));
                }
                v[i] = pack8<T>(f);
                if (y_row != nullptr) *reinterpret_cast<uint4*>(y_row + idx * 8) = v[i];
                if (inv != nullptr) {
                    const float4 i0 = __ldg(reinterpret_cast<const float4*>(inv + idx * 8));
                    const float4 i1 = __ldg(reinterpret_cast<const float4*>(inv + idx * 8) + 1);
                    const float iv[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __fmul_rn(f[e], iv[e]);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(f[e]));
            }
        }
    }
    if (a.q == nullptr) return;          // norm-only call
    am = warp_max(am);
    const float scale = __fdiv_rn(fmaxf(am, 1e-8f), 127.0f);
    const float rscale = __frcp_rn(scale);
    int8_t* qr = a.q + row * a.ldq;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + 32 * i;
        if (idx < nvec) {
            float f[8];
            unpack8<T>(v[i], f);
            if (inv != nullptr) {
                const float4 i0 = __ldg(reinterpret_cast<const float4*>(inv + idx * 8));
                const float4 i1 = __ldg(reinterpret_cast<const float4*>(inv + idx * 8) + 1);
                const float iv[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = __fmul_rn(f[e], iv[e]);
            }
            *reinterpret_cast<uint2*>(qr + idx * 8) = quant8<MODE>(f, scale, rscale);
        }
    }
    if (lane == 0) a.s[row] = scale;
}

template <typename T, int MAXV>
__global__ void __launch_bounds__(128, MAXV <= 10 ? 5 : 3) norm_rows_warp_kernel(const QuantArgs a) {
    const long row = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= a.M) return;
    if (a.round_mode == MICA_ROUND_HALF_EVEN) norm_row_warp<T, MAXV, MICA_ROUND_HALF_EVEN>(a, row, lane);
    else norm_row_warp<T, MAXV, MICA_ROUND_HALF_AWAY>(a, row, lane);
}

}  // namespace mica
