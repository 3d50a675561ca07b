// readout.cuh -- last-position option-logit scorer.
//
// logits[b, r] = sum_d float(hn[b, d]) * rows[r, d]   (fp32; rows = gathered lm_head rows)
// probs[b, lo_b:hi_b] = softmax(logits[b, lo_b:hi_b])
//
// Reference: the readout closure v0.5/serving/lib/release_runtime.py:302-306 (fp32
// linear over the gathered label rows of lm_head, after the final norm) and the slice +
// softmax v0.5/serving/lib/release_runtime.py:430-431, :509-522.
//
// Kernel 1: one warp per gathered row; the row (D fp32) is held in registers and dotted
// with every request's normalised hidden state, which the CTA builds in shared memory
// one request at a time. HBM traffic: the rows once (n_rows * D * 4 bytes) plus B * D * 2.
// Kernel 2: one warp per request for the sliced softmax.
#pragma once

#include "quant.cuh"

namespace mica {

struct ReadoutArgs {
    const void* h; long ldh;
    const void* gamma; int norm_style; float eps;
    const float* rows; int n_rows; int D;
    const int* lo; const int* hi;
    float* logits; float* probs;
    int B;
};

constexpr int RO_WARPS = 8;

template <typename T, int DV>  // DV = float4 per lane (D <= DV * 128)
__global__ void __launch_bounds__(RO_WARPS * 32) option_logits_kernel(const ReadoutArgs a) {
    extern __shared__ float hn[];      // [D] normalised hidden state of the current request
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * RO_WARPS + warp;
    const int D = a.D;
    float4 wrow[DV];
#pragma unroll
    for (int i = 0; i < DV; ++i) {
        const int d = (i * 32 + lane) * 4;
        wrow[i] = (r < a.n_rows && d < D) ? __ldg(reinterpret_cast<const float4*>(a.rows + static_cast<long>(r) * D + d))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int nvec = D >> 3;
    for (int b = 0; b < a.B; ++b) {
        const T* hr = static_cast<const T*>(a.h) + static_cast<long>(b) * a.ldh;
        // ---- build hn[b] in shared memory (optional RMSNorm, rounded to T) ----
        float ss = 0.f;
        for (int idx = threadIdx.x; idx < nvec; idx += blockDim.x) {
            float v[8];
            load8(hr + idx * 8, v);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(v[e], v[e]));
        }
        float rs = 1.f;
        if (a.gamma != nullptr) {
            ss = block_reduce<false>(ss, red);
            rs = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), a.eps));
        }
        __syncthreads();  // previous request's dot products are done with hn
        for (int idx = threadIdx.x; idx < nvec; idx += blockDim.x) {
            float v[8];
            load8(hr + idx * 8, v);
            if (a.gamma != nullptr) {
                float w[8];
                load8(static_cast<const T*>(a.gamma) + idx * 8, w);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float n = __fmul_rn(v[e], rs);
                    v[e] = a.norm_style == MICA_NORM_OFFSET ? round_to<T>(__fmul_rn(n, __fadd_rn(1.0f, w[e])))
                                                            : round_to<T>(__fmul_rn(w[e], round_to<T>(n)));
                }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) hn[idx * 8 + e] = v[e];
        }
        __syncthreads();
        if (r < a.n_rows) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < DV; ++i) {
                const int d = (i * 32 + lane) * 4;
                if (d < D) {
                    const float4 hv = *reinterpret_cast<const float4*>(hn + d);
                    acc = fmaf(wrow[i].x, hv.x, acc);
                    acc = fmaf(wrow[i].y, hv.y, acc);
                    acc = fmaf(wrow[i].z, hv.z, acc);
                    acc = fmaf(wrow[i].w, hv.w, acc);
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) a.logits[static_cast<long>(b) * a.n_rows + r] = acc;
        }
    }
}

__global__ void option_softmax_kernel(const ReadoutArgs a) {
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= a.B) return;
    const float* z = a.logits + static_cast<long>(b) * a.n_rows;
    float* p = a.probs + static_cast<long>(b) * a.n_rows;
    int lo = a.lo ? a.lo[b] : 0, hi = a.hi ? a.hi[b] : a.n_rows;
    lo = max(0, min(lo, a.n_rows));
    hi = max(lo, min(hi, a.n_rows));
    float m = -INFINITY;
    for (int i = lo + lane; i < hi; i += 32) m = fmaxf(m, z[i]);
    m = warp_max(m);
    float sum = 0.f;
    for (int i = lo + lane; i < hi; i += 32) sum += expf(z[i] - m);
    sum = warp_sum(sum);
    for (int i = lane; i < a.n_rows; i += 32) p[i] = (i >= lo && i < hi) ? expf(z[i] - m) / sum : 0.f;
}

}  // namespace mica
