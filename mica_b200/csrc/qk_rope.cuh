// qk_rope.cuh -- per-head RMSNorm of q and k plus rotary embedding, in place on the QKV
// GEMM output, reproducing the bf16 op sequence of HF Qwen3 attention:
//   n   = bf16( x * rsqrt(mean(x^2) + eps) )   (fp32 math)      Qwen3RMSNorm(q_norm/k_norm)
//   y   = bf16( w * n )
//   out = bf16( bf16(y * cos) + bf16(rotate_half(y) * sin) )      apply_rotary_pos_emb
// with rotate_half(y)[d] = -y[d + D/2] for d < D/2 and y[d - D/2] otherwise.
// One warp per (token, head); D = 128 gives 4 elements per lane. HBM-bound: it reads and
// writes the q and k columns of each token once (v is untouched).
#pragma once

#include "quant.cuh"

namespace mica {

struct QkRopeArgs {
    __nv_bfloat16* qkv;            // [S, ld] rows: q (H*D) | k (KV*D) | v
    long ld;
    const __nv_bfloat16* q_w;      // [D]
    const __nv_bfloat16* k_w;      // [D]
    const __nv_bfloat16* cos;      // [*, D] row = position
    const __nv_bfloat16* sin;
    const long* pos;               // [S] positions or nullptr (= row index + pos0)
    long pos0;
    int S, H, KV;
    float eps;
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int D>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const QkRopeArgs a) {
    constexpr int E = D / 32;                 // elements per lane
    static_assert(E % 2 == 0 && E <= 8, "head dim");
    const long warp_global = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int heads = a.H + a.KV;
    if (warp_global >= static_cast<long>(a.S) * heads) return;
    const int s = static_cast<int>(warp_global / heads);
    const int h = static_cast<int>(warp_global % heads);
    const bool is_q = h < a.H;
    __nv_bfloat16* x = a.qkv + static_cast<long>(s) * a.ld + static_cast<long>(h) * D;
    const __nv_bfloat16* w = is_q ? a.q_w : a.k_w;
    const long p = a.pos ? a.pos[s] : a.pos0 + s;
    const __nv_bfloat16* cr = a.cos + p * D;
    const __nv_bfloat16* sr = a.sin + p * D;
    // lane holds elements d = lane*E/2 + i (i < E/2) of the first half and their partners
    // d + D/2 of the second half, so rotate_half pairs stay inside the lane.
    constexpr int HALF = E / 2;
    const int d0 = lane * HALF;
    float lo[HALF], hi[HALF];
    if constexpr (HALF % 2 == 0) {
#pragma unroll
        for (int i = 0; i < HALF; i += 2) {       // 4-byte pair loads (coalesced 128 B per half)
            const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(x + d0 + i);
            const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(x + D / 2 + d0 + i);
            lo[i] = __low2float(a); lo[i + 1] = __high2float(a);
            hi[i] = __low2float(b); hi[i + 1] = __high2float(b);
        }
    } else {
#pragma unroll
        for (int i = 0; i < HALF; ++i) {
            lo[i] = __bfloat162float(x[d0 + i]);
            hi[i] = __bfloat162float(x[D / 2 + d0 + i]);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < HALF; ++i) ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(lo[i], lo[i]), __fmul_rn(hi[i], hi[i])));
    ss = warp_sum(ss);
    const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), a.eps));
    float ol[HALF], oh[HALF];
#pragma unroll
    for (int i = 0; i < HALF; ++i) {
        const int dl = d0 + i, dh = D / 2 + d0 + i;
        const float yl = bf(__fmul_rn(__bfloat162float(w[dl]), bf(__fmul_rn(lo[i], r))));
        const float yh = bf(__fmul_rn(__bfloat162float(w[dh]), bf(__fmul_rn(hi[i], r))));
        const float cl = __bfloat162float(cr[dl]), ch = __bfloat162float(cr[dh]);
        const float sl = __bfloat162float(sr[dl]), sh = __bfloat162float(sr[dh]);
        ol[i] = bf(__fadd_rn(bf(__fmul_rn(yl, cl)), bf(__fmul_rn(-yh, sl))));
        oh[i] = bf(__fadd_rn(bf(__fmul_rn(yh, ch)), bf(__fmul_rn(yl, sh))));
    }
    if constexpr (HALF % 2 == 0) {
#pragma unroll
        for (int i = 0; i < HALF; i += 2) {
            *reinterpret_cast<__nv_bfloat162*>(x + d0 + i) = __floats2bfloat162_rn(ol[i], ol[i + 1]);
            *reinterpret_cast<__nv_bfloat162*>(x + D / 2 + d0 + i) = __floats2bfloat162_rn(oh[i], oh[i + 1]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < HALF; ++i) {
            x[d0 + i] = __float2bfloat16_rn(ol[i]);
            x[D / 2 + d0 + i] = __float2bfloat16_rn(oh[i]);
        }
    }
}

// One warp per token for D = 128: lane l owns dims (2l, 2l+1) and their rotation partners
// (64+2l, 64+2l+1). cos/sin of the token and both norm weights stay in registers across the
// token's H + KV heads; each head costs two 4-byte loads and stores per lane. Every step is
// fp32 arithmetic followed by an explicit bf16 rounding, the HF op sequence.
__global__ void __launch_bounds__(256) qk_norm_rope_token_kernel(const QkRopeArgs a) {
    constexpr int D = 128;
    const long s = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (s >= a.S) return;
    const long p = a.pos ? a.pos[s] : a.pos0 + s;
    const int d = 2 * lane;
    const __nv_bfloat162 c_lo = *reinterpret_cast<const __nv_bfloat162*>(a.cos + p * D + d);
    const __nv_bfloat162 c_hi = *reinterpret_cast<const __nv_bfloat162*>(a.cos + p * D + D / 2 + d);
    const __nv_bfloat162 s_lo = *reinterpret_cast<const __nv_bfloat162*>(a.sin + p * D + d);
    const __nv_bfloat162 s_hi = *reinterpret_cast<const __nv_bfloat162*>(a.sin + p * D + D / 2 + d);
    __nv_bfloat162 wq_lo = __float2bfloat162_rn(0.f), wq_hi = wq_lo, wk_lo = wq_lo, wk_hi = wq_lo;
    if (a.H > 0) {
        wq_lo = *reinterpret_cast<const __nv_bfloat162*>(a.q_w + d);
        wq_hi = *reinterpret_cast<const __nv_bfloat162*>(a.q_w + D / 2 + d);
    }
    if (a.KV > 0) {
        wk_lo = *reinterpret_cast<const __nv_bfloat162*>(a.k_w + d);
        wk_hi = *reinterpret_cast<const __nv_bfloat162*>(a.k_w + D / 2 + d);
    }
    __nv_bfloat16* row = a.qkv + s * a.ld;
    const int heads = a.H + a.KV;
    // Eight heads are loaded before any is rewritten: the stores could alias later heads'
    // loads, so without this the compiler keeps every load behind the previous head's store
    // and the warp has one 256-byte request in flight.
    constexpr int G = 8;
    for (int h0 = 0; h0 < heads; h0 += G) {
        __nv_bfloat162 xls[G], xhs[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (h0 + g < heads) {
                const __nv_bfloat16* x = row + static_cast<long>(h0 + g) * D;
                xls[g] = *reinterpret_cast<const __nv_bfloat162*>(x + d);
                xhs[g] = *reinterpret_cast<const __nv_bfloat162*>(x + D / 2 + d);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int h = h0 + g;
            if (h >= heads) break;                 // uniform across the warp
            __nv_bfloat16* x = row + static_cast<long>(h) * D;
            const float2 fl = __bfloat1622float2(xls[g]), fh = __bfloat1622float2(xhs[g]);
            float ss = __fadd_rn(__fadd_rn(__fmul_rn(fl.x, fl.x), __fmul_rn(fl.y, fl.y)),
                                 __fadd_rn(__fmul_rn(fh.x, fh.x), __fmul_rn(fh.y, fh.y)));
            ss = warp_sum(ss);
            const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), a.eps));
            const bool is_q = h < a.H;
            const float2 wl = __bfloat1622float2(is_q ? wq_lo : wk_lo), wh = __bfloat1622float2(is_q ? wq_hi : wk_hi);
            const float2 cl = __bfloat1622float2(c_lo), ch = __bfloat1622float2(c_hi);
            const float2 sl = __bfloat1622float2(s_lo), sh = __bfloat1622float2(s_hi);
            const float yl0 = bf(__fmul_rn(wl.x, bf(__fmul_rn(fl.x, r)))), yl1 = bf(__fmul_rn(wl.y, bf(__fmul_rn(fl.y, r))));
            const float yh0 = bf(__fmul_rn(wh.x, bf(__fmul_rn(fh.x, r)))), yh1 = bf(__fmul_rn(wh.y, bf(__fmul_rn(fh.y, r))));
            const float ol0 = __fadd_rn(bf(__fmul_rn(yl0, cl.x)), bf(__fmul_rn(-yh0, sl.x)));
            const float ol1 = __fadd_rn(bf(__fmul_rn(yl1, cl.y)), bf(__fmul_rn(-yh1, sl.y)));
            const float oh0 = __fadd_rn(bf(__fmul_rn(yh0, ch.x)), bf(__fmul_rn(yl0, sh.x)));
            const float oh1 = __fadd_rn(bf(__fmul_rn(yh1, ch.y)), bf(__fmul_rn(yl1, sh.y)));
            *reinterpret_cast<__nv_bfloat162*>(x + d) = __floats2bfloat162_rn(ol0, ol1);
            *reinterpret_cast<__nv_bfloat162*>(x + D / 2 + d) = __floats2bfloat162_rn(oh0, oh1);
        }
    }
}

}  // namespace mica
