// attention.cuh -- causal grouped-query attention forward for the prefill, on tcgen05 (sm_100a).
//
//   O[t, h, :] = sum_{s <= t} softmax_s(scale * Q[t, h, :] . K[s, h / G, :]) V[s, h / G, :]
//
// bf16 Q, K, V read in place from the QKV projection's output ([rows, (H + 2 KV) D], q | k | v
// columns), D = 128, G = H / KV query heads per key/value head; each request of a [B, L] batch
// attends within its own L rows. fp32 scores and accumulator, bf16 output [rows, H D].
//
// One CTA per (request, block of 128 query rows, query head), heaviest blocks first. Warps:
//   warp 0      TMA producer: the Q tile once (two 64-column boxes, 128-byte swizzle), then
//               K and V tiles of 128 keys in two rings of KV_STAGES stages;
//   warp 1      one lane issues the MMAs: S_j = Q K_j^T (kind::f16, M 128, N 128, K 16 steps,
//               both operands K-major in shared memory) into one of two TMEM score buffers,
//               then O += P_{j-1} V_{j-1} with P read from tensor memory (the TS form) and V
//               MN-major in shared memory, so scoring tile j overlaps the softmax of tile j-1;
//   warps 2..5  softmax, one query row per thread: scores from TMEM, causal mask on the
//               diagonal tile, running max in the exp2 domain, p = 2^(s c - m), row sum, P to
//               TMEM as bf16 pairs. O is rescaled (read, scaled, written back in TMEM) only when
//               the running max grows by more than 8 (a factor of 256): otherwise the stale max
//               is kept, p stays below 2^8 and nothing is lost in fp32. At the end each thread
//               divides its O row by its sum and stores it.
// Tensor memory (512 columns): S0 [0,128) S1 [128,256) O [256,384) P0 [384,448) P1 [448,512).
// Every wait is bounded (common.cuh); a wait that runs out unwinds the CTA.
//
// Reference semantics: the reference's prefill runs attention through torch SDPA
// (v0.5/serving/lib/prefill_engine.py:308-324, lib/fast_runtime.py:189-220); its Triton kernel
// v0.5/serving/kernel_src/kernels.py:72-124 computes the same causal GQA softmax with exp2.
#pragma once

#include "common.cuh"

namespace mica {

struct AttnArgs {
    const __nv_bfloat16* qkv;   // [B * L, (H + 2 KV) * D]
    long ld_qkv;                // elements
    __nv_bfloat16* out;         // [B * L, H * D]
    long ld_out;                // elements
    int B, L, H, KV;
    float scale_log2;           // softmax scale * log2(e)
};

constexpr int ATT_D = 128;
constexpr int ATT_BM = 128;                 // query rows per CTA
constexpr int ATT_BN = 128;                 // keys per tile
constexpr int ATT_HALF_BYTES = 128 * 128;   // one 128-row x 64-column bf16 box (128-byte rows)
constexpr int ATT_TILE_BYTES = 2 * ATT_HALF_BYTES;
constexpr int ATT_KV_STAGES = 3;
constexpr int ATT_SMEM_BYTES = 1024 + ATT_TILE_BYTES * (1 + 2 * ATT_KV_STAGES) + 256;
constexpr int ATT_THREADS = 192;
constexpr float ATT_RESCALE_LOG2 = 8.0f;

// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, M 128, N 128; B K-major
// (scores) or MN-major (the value tile, d contiguous).
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Shared-memory descriptor of a 128-byte-swizzled tile: start address, leading and stride byte
// offsets (>> 4), version 1, swizzle mode 2. K-major tiles use LBO 16 (unused) and SBO 1024
// (8-row groups); an MN-major tile uses LBO = the distance between 64-element column blocks
// and SBO = the distance between 8-row groups along K.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// A from tensor memory (rows in lanes, two bf16 of K per 32-bit column).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Number of key tiles query block `qb` needs (keys 0 .. min(L, q0 + 128) - 1).
__host__ __device__ __forceinline__ int att_key_tiles(int qb, int L) {
    const int last = min(L, (qb + 1) * ATT_BM) - 1;
    return last / ATT_BN + 1;
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
attention_fwd_kernel(const __grid_constant__ CUtensorMap tmap_qkv, const AttnArgs args) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q_blocks = (args.L + ATT_BM - 1) / ATT_BM;
    // heaviest (latest) query blocks first; within a block index, requests then heads
    const int per_qb = args.B * args.H;
    const int qb = q_blocks - 1 - static_cast<int>(blockIdx.x) / per_qb;
    const int rem = static_cast<int>(blockIdx.x) % per_qb;
    const int b = rem / args.H;
    const int h = rem % args.H;
    const int kvh = h / (args.H / args.KV);
    const int q0 = qb * ATT_BM;
    const int row0 = b * args.L;              // first row of this request
    const int nkv = att_key_tiles(qb, args.L);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sq = smem;
    uint8_t* sk = smem + ATT_TILE_BYTES;
    uint8_t* sv = sk + ATT_KV_STAGES * ATT_TILE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sv + ATT_KV_STAGES * ATT_TILE_BYTES);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + ATT_KV_STAGES;
    uint64_t* v_full = k_empty + ATT_KV_STAGES;
    uint64_t* v_empty = v_full + ATT_KV_STAGES;
    uint64_t* s_full = v_empty + ATT_KV_STAGES;     // [2] MMA -> softmax: scores ready
    uint64_t* s_read = s_full + 2;                  // [2] softmax -> MMA: scores read
    uint64_t* p_full = s_read + 2;                  // [2] softmax -> MMA: P (and O rescale) written
    uint64_t* p_done = p_full + 2;                  // [2] MMA -> softmax: P.V of that buffer finished
    uint64_t* drain = p_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < ATT_KV_STAGES; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_read[i], 4);
            mbar_init(&p_full[i], 4);
            mbar_init(&p_done[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_qkv);
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_s = tmem, t_o = tmem + 256, t_p = tmem + 384;

    const int qcol = h * ATT_D;
    const int kcol = (args.H + kvh) * ATT_D;
    const int vcol = (args.H + args.KV + kvh) * ATT_D;

    if (warp == 0) {
        // ---------------------------------- producer ----------------------------------
        if (lane == 0) {
            const uint64_t pol_kv = policy_evict_last();     // re-read by the G query heads and later blocks
            mbar_arrive_expect_tx(q_full, ATT_TILE_BYTES);
            tma_load_2d(sq, &tmap_qkv, q_full, qcol, row0 + q0);
            tma_load_2d(sq + ATT_HALF_BYTES, &tmap_qkv, q_full, qcol + 64, row0 + q0);
            bool ok = true;
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j % ATT_KV_STAGES;
                const uint32_t ph = (j / ATT_KV_STAGES) & 1u;
                const int k0 = row0 + j * ATT_BN;
                if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
                mbar_arrive_expect_tx(&k_full[st], ATT_TILE_BYTES);
                uint8_t* kd = sk + st * ATT_TILE_BYTES;
                tma_load_2d_hint(kd, &tmap_qkv, &k_full[st], kcol, k0, pol_kv);
                tma_load_2d_hint(kd + ATT_HALF_BYTES, &tmap_qkv, &k_full[st], kcol + 64, k0, pol_kv);
                if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
                mbar_arrive_expect_tx(&v_full[st], ATT_TILE_BYTES);
                uint8_t* vd = sv + st * ATT_TILE_BYTES;
                tma_load_2d_hint(vd, &tmap_qkv, &v_full[st], vcol, k0, pol_kv);
                tma_load_2d_hint(vd + ATT_HALF_BYTES, &tmap_qkv, &v_full[st], vcol + 64, k0, pol_kv);
            }
            // the last loads of each ring land before shared memory is released
            mbar_wait(q_full, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
            const int first = nkv > ATT_KV_STAGES ? nkv - ATT_KV_STAGES : 0;
            for (int j = first; j < nkv && ok; ++j) {
                mbar_wait(&k_full[j % ATT_KV_STAGES], (j / ATT_KV_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
                mbar_wait(&v_full[j % ATT_KV_STAGES], (j / ATT_KV_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------- MMA issuer --------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_bf16(ATT_BM, ATT_BN, false);
            constexpr uint32_t idesc_pv = idesc_bf16(ATT_BM, ATT_D, true);
            const uint32_t q_addr = smem_u32(sq);
            bool ok = mbar_wait(q_full, 0, abort_flag, MICA_DEV_TIMEOUT_MMA);
            // issue order: S0, S1, PV0, S2, PV1, ... so the scores of tile j+1 are computed
            // while the softmax works on tile j
            for (int step = 0; step <= nkv && ok; ++step) {
                if (step < nkv) {
                    const int j = step;
                    const int sb = j & 1;
                    const int st = j % ATT_KV_STAGES;
                    if (!mbar_wait(&k_full[st], (j / ATT_KV_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) break;
                    // the softmax has read this score buffer's previous tile (j - 2)
                    if (j >= 2 && !mbar_wait(&s_read[sb], ((j - 2) >> 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA))
                        break;
                    tc_fence_after();
                    const uint32_t k_addr = smem_u32(sk + st * ATT_TILE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < ATT_D / 16; ++kk) {
                        const uint32_t off = (kk >> 2) * ATT_HALF_BYTES + (kk & 3) * 32;
                        mma_bf16_ss(t_s + sb * 128, smem_desc_sw128(q_addr + off, 16, 1024),
                                    smem_desc_sw128(k_addr + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(&k_empty[st]);
                    mma_commit(&s_full[sb]);
                }
                if (step >= 1) {
                    const int j = step - 1;
                    const int pb = j & 1;
                    const int st = j % ATT_KV_STAGES;
                    if (!mbar_wait(&p_full[pb], (j >> 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) break;
                    if (!mbar_wait(&v_full[st], (j / ATT_KV_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) break;
                    tc_fence_after();
                    const uint32_t v_addr = smem_u32(sv + st * ATT_TILE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < ATT_BN / 16; ++kk) {
                        // 16 keys: 8 columns of P (bf16 pairs); V rows kk*16.. as the K of the MMA
                        mma_bf16_ts(t_o, t_p + pb * 64 + kk * 8, smem_desc_sw128(v_addr + kk * 16 * 128, ATT_HALF_BYTES, 1024),
                                    idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&v_empty[st]);
                    mma_commit(&p_done[pb]);
                }
            }
            mma_commit(drain);
            mbar_wait(drain, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else {
        // ---------------------------------- softmax ----------------------------------
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;                     // row in the tile
        const int qi = q0 + r;                            // query index in the request
        const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
        const float c = args.scale_log2;
        float m_use = -1e30f;                             // running max (exp2 domain) in use
        float l = 0.f;                                    // running sum of p
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            const int sb = j & 1;
            bool w = true;
            if (lane == 0) w = mbar_wait(&s_full[sb], (j >> 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
            tc_fence_after();
            uint32_t sr[128];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t (&part)[32] = *reinterpret_cast<uint32_t (*)[32]>(&sr[cc * 32]);
                tmem_ld_32x32b_x32(t_s + sb * 128 + lane_off + cc * 32, part);
            }
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_read[sb]);
            // causal and length mask on the tile that reaches the diagonal or the end
            const int k0 = j * ATT_BN;
            const bool masked = k0 + ATT_BN - 1 > q0 || k0 + ATT_BN > args.L;
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 128; ++i) {
                float s = __uint_as_float(sr[i]) * c;
                if (masked && (k0 + i > qi || k0 + i >= args.L)) s = -INFINITY;
                sr[i] = __float_as_uint(s);
                mx = fmaxf(mx, s);
            }
            float alpha = 1.f;
            const bool rescale = mx > m_use + ATT_RESCALE_LOG2;
            if (rescale) {
                alpha = fast_exp2(m_use - mx);
                m_use = mx;
            }
            float sum = 0.f;
            uint32_t pk[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                const float p0 = fast_exp2(__uint_as_float(sr[2 * i]) - m_use);
                const float p1 = fast_exp2(__uint_as_float(sr[2 * i + 1]) - m_use);
                sum += p0 + p1;
                pk[i] = pack_bf16(p0, p1);
            }
            l = l * alpha + sum;
            // O must hold P_{j-1} V_{j-1} before it is rescaled, and P_{j-2} V_{j-2} must be done
            // with this P buffer before it is overwritten
            if (j >= 1 && rescale) {
                if (lane == 0) w = mbar_wait(&p_done[(j - 1) & 1], ((j - 1) >> 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
                if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(t_o + lane_off + cc * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st_32x32b_x32(t_o + lane_off + cc * 32, o);
                }
            }
            if (j >= 2) {
                if (lane == 0) w = mbar_wait(&p_done[sb], ((j - 2) >> 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
                if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
                tc_fence_after();
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t (&part)[32] = *reinterpret_cast<uint32_t (*)[32]>(&pk[half * 32]);
                tmem_st_32x32b_x32(t_p + sb * 64 + lane_off + half * 32, part);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[sb]);
        }
        if (ok) {
            // the last P.V is done: normalise and store this thread's output row
            const int jl = nkv - 1;
            bool w = true;
            if (lane == 0) w = mbar_wait(&p_done[jl & 1], (jl >> 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (__shfl_sync(0xffffffffu, w, 0)) {
                tc_fence_after();
                const float inv = 1.f / l;
                __nv_bfloat16* orow = args.out + static_cast<long>(row0 + qi) * args.ld_out + h * ATT_D;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(t_o + lane_off + cc * 32, o);
                    tmem_ld_wait();
                    if (qi < args.L) {
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint4 pkt;
                            pkt.x = pack_bf16(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
                            pkt.y = pack_bf16(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
                            pkt.z = pack_bf16(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
                            pkt.w = pack_bf16(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
                            *reinterpret_cast<uint4*>(orow + cc * 32 + v * 8) = pkt;
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_free(tmem, 512);
    }
}

}  // namespace mica
