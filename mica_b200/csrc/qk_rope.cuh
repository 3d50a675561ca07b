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

// One warp per token for D = 128, two heads at a time: half-warp p (lanes 16p..16p+15) takes
// head h0 + p, and its lane j owns dims [4j, 4j+4) and their rotation partners [64+4j, 64+4j+4).
// cos/sin of the token and both norm weights stay in registers across the token's H + KV
// heads; each head costs a lane two 8-byte loads and stores, and one 4-step shuffle sequence
// reduces both heads' sums of squares. Eight heads are loaded before any is rewritten (a store
// could alias a later head's load, which would otherwise serialise them).
// Arithmetic follows the HF op sequence: the sum of squares and x * rsqrt(...) in fp32, the
// cast to bf16 (one packed cvt.rn per pair), then bf16 ops on packed pairs -- w * h, q * cos,
// rotate_half(q) * sin and their sum. A packed bf16 multiply is the single rounding of the
// exact product, which is what the fp32 multiply and cast give; a packed add of two bf16
// values equals the fp32 add and cast too (their fp32 sum is exact unless the exponents differ
// by more than 15, and then the smaller term is far below half an ulp of the result either way).
// The _rn forms keep the compiler from contracting a multiply and the add into one fma, which
// would round once where the HF sequence rounds twice.
__device__ __forceinline__ void unpack4_bf16(const uint2 w, float (&f)[4]) {
    f[0] = __uint_as_float(w.x << 16);
    f[1] = __uint_as_float(w.x & 0xFFFF0000u);
    f[2] = __uint_as_float(w.y << 16);
    f[3] = __uint_as_float(w.y & 0xFFFF0000u);
}
__device__ __forceinline__ __nv_bfloat162 bf2(uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); }
__device__ __forceinline__ uint32_t bits2(__nv_bfloat162 v) { return *reinterpret_cast<const uint32_t*>(&v); }

// Five 256-thread blocks per SM (48 registers): 40 warps in flight instead of 32; the few
// values that no longer fit (the token's cos/sin words) reload from L1, which measured faster.
__global__ void __launch_bounds__(256, 5) qk_norm_rope_token_kernel(const QkRopeArgs a) {
    constexpr int D = 128;
    const long s = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (s >= a.S) return;
    const int half = lane >> 4;
    const int d = 4 * (lane & 15);
    const long p = a.pos ? a.pos[s] : a.pos0 + s;
    // packed bf16 pairs: cos/sin of dims [d, d+4) (l) and [64+d, 64+d+4) (h); -sin for the
    // rotated low half (rotate_half negates q's high half: (-y_h) * sin_l = y_h * (-sin_l))
    const uint2 cl = *reinterpret_cast<const uint2*>(a.cos + p * D + d);
    const uint2 ch = *reinterpret_cast<const uint2*>(a.cos + p * D + D / 2 + d);
    const uint2 sl = *reinterpret_cast<const uint2*>(a.sin + p * D + d);
    const uint2 sh = *reinterpret_cast<const uint2*>(a.sin + p * D + D / 2 + d);
    const uint32_t cl2[2] = {cl.x, cl.y}, ch2[2] = {ch.x, ch.y}, sh2[2] = {sh.x, sh.y};
    const uint32_t nsl2[2] = {sl.x ^ 0x80008000u, sl.y ^ 0x80008000u};
    uint2 wql = make_uint2(0u, 0u), wqh = wql, wkl = wql, wkh = wql;
    if (a.H > 0) {
        wql = *reinterpret_cast<const uint2*>(a.q_w + d);
        wqh = *reinterpret_cast<const uint2*>(a.q_w + D / 2 + d);
    }
    if (a.KV > 0) {
        wkl = *reinterpret_cast<const uint2*>(a.k_w + d);
        wkh = *reinterpret_cast<const uint2*>(a.k_w + D / 2 + d);
    }
    __nv_bfloat16* row = a.qkv + s * a.ld;
    const int heads = a.H + a.KV;
    constexpr int G = 4;                          // head pairs loaded ahead
    for (int h0 = 0; h0 < heads; h0 += 2 * G) {
        uint2 xl[G], xh[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int h = h0 + 2 * g + half;
            if (h < heads) {
                const __nv_bfloat16* x = row + static_cast<long>(h) * D;
                xl[g] = *reinterpret_cast<const uint2*>(x + d);
                xh[g] = *reinterpret_cast<const uint2*>(x + D / 2 + d);
            } else {
                xl[g] = xh[g] = make_uint2(0u, 0u);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (h0 + 2 * g >= heads) break;       // uniform across the warp
            const int h = h0 + 2 * g + half;
            float fl[4], fh[4];
            unpack4_bf16(xl[g], fl);
            unpack4_bf16(xh[g], fh);
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(fl[e], fl[e]), __fmul_rn(fh[e], fh[e])));
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            if (h >= heads) continue;
            const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), a.eps));
            const bool is_q = h < a.H;
            const uint2 wl = is_q ? wql : wkl, wh = is_q ? wqh : wkh;
            const uint32_t wl2[2] = {wl.x, wl.y}, wh2[2] = {wh.x, wh.y};
            uint32_t ol[2], oh[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const __nv_bfloat162 yl = __hmul2_rn(
                    bf2(wl2[k]), __floats2bfloat162_rn(__fmul_rn(fl[2 * k], r), __fmul_rn(fl[2 * k + 1], r)));
                const __nv_bfloat162 yh = __hmul2_rn(
                    bf2(wh2[k]), __floats2bfloat162_rn(__fmul_rn(fh[2 * k], r), __fmul_rn(fh[2 * k + 1], r)));
                ol[k] = bits2(__hadd2_rn(__hmul2_rn(yl, bf2(cl2[k])), __hmul2_rn(yh, bf2(nsl2[k]))));
                oh[k] = bits2(__hadd2_rn(__hmul2_rn(yh, bf2(ch2[k])), __hmul2_rn(yl, bf2(sh2[k]))));
            }
            __nv_bfloat16* x = row + static_cast<long>(h) * D;
            *reinterpret_cast<uint2*>(x + d) = make_uint2(ol[0], ol[1]);
            *reinterpret_cast<uint2*>(x + D / 2 + d) = make_uint2(oh[0], oh[1]);
        }
    }
}

}  // namespace mica
