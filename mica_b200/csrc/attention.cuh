// attention.cuh -- causal grouped-query attention forward for the prefill, on tcgen05 (sm_100a).
//
//   O[t, h, :] = sum_{s <= t} softmax_s(scale * Q[t, h, :] . K[s, h / G, :]) V[s, h / G, :]
//
// bf16 Q, K, V read in place from the QKV projection's output ([rows, (H + 2 KV) D], q | k | v
// columns), D = 128, G = H / KV query heads per key/value head; each request of a [B, L] batch
// attends within its own L rows. fp32 scores and accumulator, bf16 output [rows, H D].
//
// One CTA per (request, block of 256 query rows, query head), heaviest blocks first: two query
// tiles A and B of 128 rows share every K and V tile. Warps:
//   warp 0      TMA producer: both Q tiles once (64-column boxes, 128-byte swizzle), then K and
//               V tiles of 128 keys in rings of 3 and 2 stages;
//   warp 1      one lane issues the MMAs: S = Q_X K_j^T (kind::f16, M 128, N 128, K 16 steps,
//               both operands K-major in shared memory) and O_X += P_X V_j with P read from tensor
//               memory (the TS form) and V MN-major in shared memory;
//   warps 2..5  softmax of tile A, warps 6..9 of tile B, one query row per thread: scores from
//               TMEM, causal mask on the diagonal tile, running max in the exp2 domain,
//               p = 2^(s c - m), row sum, P to TMEM as bf16 pairs. O is rescaled in TMEM only when
//               the running max grows by more than 8 (a factor of 256): otherwise the stale max is
//               kept, p stays below 2^8 and nothing is lost in fp32. At the end each thread divides
//               its O row by its sum and stores it.
// Tensor memory (512 columns): S [0,128) P_A [128,192) P_B [192,256) O_A [256,384) O_B [384,512).
// The one score buffer is taken in turn, S_A(0) S_B(0) S_A(1) S_B(1) ...: a tile's softmax frees it
// as soon as it has the scores in registers, so the tensor core computes the other tile's scores
// (and a P.V) while that softmax runs; the next P.V of a tile is issued when its P is written. MMA
// order per key tile j: S_A(j+1), O_A += P_A(j) V_j, S_B(j+1), O_B += P_B(j) V_j.
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
constexpr int ATT_BM = 128;                 // query rows per tile (two tiles per CTA)
constexpr int ATT_BN = 128;                 // keys per tile
constexpr int ATT_HALF_BYTES = 128 * 128;   // one 128-row x 64-column bf16 box (128-byte rows)
constexpr int ATT_TILE_BYTES = 2 * ATT_HALF_BYTES;
// K is needed one step ahead of V (the next scores are issued right after this step's P.V), so its
// ring is a stage deeper: with two stages the TMA round trip of K_{j+1} sat on the critical path.
constexpr int ATT_K_STAGES = 3;
constexpr int ATT_V_STAGES = 2;
constexpr int ATT_SMEM_BYTES = 1024 + ATT_TILE_BYTES * (2 + ATT_K_STAGES + ATT_V_STAGES) + 256;
constexpr int ATT_THREADS = 320;
constexpr float ATT_RESCALE_LOG2 = 8.0f;

// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, M 128, N 128; B K-major
// (scores) or MN-major (the value tile, d contiguous).
// Bounded polling wait (no sleep hint) for the waits on the per-step critical path: the MMA
// issuer's, and the softmax's wait for its scores and for its previous P.V. With mbar_wait's
// sleep hint each of them took a few hundred cycles to resume after the phase completed.
__device__ __forceinline__ bool mma_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1u;
            atomicExch(&g_dev_error, code);
            return false;
        }
    }
}

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

__device__ __forceinline__ float fmax3(float a, float b, float d) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(d));
    return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long d) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(d));
    return r;
}

// 2^x on the MUFU unit. Measured on B200: ex2.approx.f16x2 runs at half the rate of the f32 form
// (the same exponentials per cycle) and its f16 pack costs as much again, so the f32 form is used.
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
    const int pairs = (args.L + 2 * ATT_BM - 1) / (2 * ATT_BM);
    // heaviest (latest) blocks first; within a block index, requests then heads
    const int per_cb = args.B * args.H;
    const int cb = pairs - 1 - static_cast<int>(blockIdx.x) / per_cb;
    const int rem = static_cast<int>(blockIdx.x) % per_cb;
    const int b = rem / args.H;
    const int h = rem % args.H;
    const int kvh = h / (args.H / args.KV);
    const int q0 = cb * 2 * ATT_BM;           // tile A rows q0.., tile B rows q0 + 128..
    const int row0 = b * args.L;              // first row of this request
    const int nkv_a = att_key_tiles(2 * cb, args.L);
    const int nkv_b = att_key_tiles(2 * cb + 1, args.L);   // >= nkv_a: the key tiles loaded

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sq = smem;                                       // Q_A, Q_B
    uint8_t* sk = smem + 2 * ATT_TILE_BYTES;
    uint8_t* sv = sk + ATT_K_STAGES * ATT_TILE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sv + ATT_V_STAGES * ATT_TILE_BYTES);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + ATT_K_STAGES;
    uint64_t* v_full = k_empty + ATT_K_STAGES;
    uint64_t* v_empty = v_full + ATT_V_STAGES;
    uint64_t* s_full = v_empty + ATT_V_STAGES;      // [2] per tile, MMA -> softmax: its scores are in S
    uint64_t* s_free = s_full + 2;                  // softmax -> MMA: S read into registers (4 warps)
    uint64_t* p_full = s_free + 1;                  // [2] softmax -> MMA: P (and any O rescale) written
    uint64_t* pv_done = p_full + 2;                 // [2] MMA -> softmax: the tile's P.V finished
    uint64_t* drain = pv_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < ATT_K_STAGES; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < ATT_V_STAGES; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&pv_done[i], 1);
        }
        mbar_init(s_free, 4);
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

    const int qcol = h * ATT_D;
    const int kcol = (args.H + kvh) * ATT_D;
    const int vcol = (args.H + args.KV + kvh) * ATT_D;

    if (warp == 0) {
        // ---------------------------------- producer ----------------------------------
        if (lane == 0) {
            const uint64_t pol_kv = policy_evict_last();     // re-read by the G query heads and later blocks
            mbar_arrive_expect_tx(q_full, 2 * ATT_TILE_BYTES);
            for (int t = 0; t < 2; ++t) {
                tma_load_2d(sq + t * ATT_TILE_BYTES, &tmap_qkv, q_full, qcol, row0 + q0 + t * ATT_BM);
                tma_load_2d(sq + t * ATT_TILE_BYTES + ATT_HALF_BYTES, &tmap_qkv, q_full, qcol + 64,
                            row0 + q0 + t * ATT_BM);
            }
            bool ok = true;
            // K runs up to ATT_K_STAGES tiles ahead, V up to ATT_V_STAGES: load K_j, then V_{j-d}
            // where d = ATT_K_STAGES - ATT_V_STAGES, so a full V ring never holds back K
            constexpr int d = ATT_K_STAGES - ATT_V_STAGES;
            auto load_k = [&](int j) {
                const int st = j % ATT_K_STAGES;
                if (!mbar_wait(&k_empty[st], ((j / ATT_K_STAGES) & 1u) ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER))
                    return false;
                mbar_arrive_expect_tx(&k_full[st], ATT_TILE_BYTES);
                uint8_t* kd = sk + st * ATT_TILE_BYTES;
                tma_load_2d_hint(kd, &tmap_qkv, &k_full[st], kcol, row0 + j * ATT_BN, pol_kv);
                tma_load_2d_hint(kd + ATT_HALF_BYTES, &tmap_qkv, &k_full[st], kcol + 64, row0 + j * ATT_BN, pol_kv);
                return true;
            };
            auto load_v = [&](int j) {
                const int st = j % ATT_V_STAGES;
                if (!mbar_wait(&v_empty[st], ((j / ATT_V_STAGES) & 1u) ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER))
                    return false;
                mbar_arrive_expect_tx(&v_full[st], ATT_TILE_BYTES);
                uint8_t* vd = sv + st * ATT_TILE_BYTES;
                tma_load_2d_hint(vd, &tmap_qkv, &v_full[st], vcol, row0 + j * ATT_BN, pol_kv);
                tma_load_2d_hint(vd + ATT_HALF_BYTES, &tmap_qkv, &v_full[st], vcol + 64, row0 + j * ATT_BN, pol_kv);
                return true;
            };
            for (int j = 0; j < nkv_b + d && ok; ++j) {
                if (j < nkv_b && !load_k(j)) ok = false;
                if (ok && j >= d && !load_v(j - d)) ok = false;
            }
            // the last loads of each ring land before shared memory is released
            mbar_wait(q_full, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
            for (int j = nkv_b > ATT_K_STAGES ? nkv_b - ATT_K_STAGES : 0; j < nkv_b && ok; ++j)
                mbar_wait(&k_full[j % ATT_K_STAGES], (j / ATT_K_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
            for (int j = nkv_b > ATT_V_STAGES ? nkv_b - ATT_V_STAGES : 0; j < nkv_b && ok; ++j)
                mbar_wait(&v_full[j % ATT_V_STAGES], (j / ATT_V_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------- MMA issuer --------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_bf16(ATT_BM, ATT_BN, false);
            constexpr uint32_t idesc_pv = idesc_bf16(ATT_BM, ATT_D, true);
            const int nkv[2] = {nkv_a, nkv_b};
            bool ok = mma_wait(q_full, 0, abort_flag, MICA_DEV_TIMEOUT_MMA);
            // S = Q_X K_j^T; the fills of S alternate between the tiles and each waits until the
            // previous one has been read (s_free completes once per fill)
            int fills = 0;
            // descriptors of the stage bases; a byte offset within a tile adds (offset >> 4)
            const uint64_t q_desc0 = smem_desc_sw128(smem_u32(sq), 16, 1024);
            const uint64_t k_desc0 = smem_desc_sw128(smem_u32(sk), 16, 1024);
            const uint64_t v_desc0 = smem_desc_sw128(smem_u32(sv), ATT_HALF_BYTES, 1024);
            constexpr uint64_t kTileStep = ATT_TILE_BYTES >> 4;
            auto scores = [&](int x, int j) {
                if (fills > 0 && !mma_wait(s_free, (fills - 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) return false;
                tc_fence_after();
                const uint64_t qd = q_desc0 + static_cast<uint64_t>(x) * kTileStep;
                const uint64_t kd = k_desc0 + static_cast<uint64_t>(j % ATT_K_STAGES) * kTileStep;
#pragma unroll
                for (int kk = 0; kk < ATT_D / 16; ++kk) {
                    const uint64_t off = static_cast<uint64_t>(((kk >> 2) * ATT_HALF_BYTES + (kk & 3) * 32) >> 4);
                    mma_bf16_ss(tmem, qd + off, kd + off, idesc_qk, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[x]);
                ++fills;
                return true;
            };
            // O_X += P_X V_j once tile X's softmax has written P_X(j)
            auto values = [&](int x, int j) {
                if (!mma_wait(&p_full[x], j & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) return false;
                tc_fence_after();
                const uint64_t vd = v_desc0 + static_cast<uint64_t>(j % ATT_V_STAGES) * kTileStep;
                const uint32_t d_o = tmem + 256 + x * 128, a_p = tmem + 128 + x * 64;
                mma_bf16_ts(d_o, a_p, vd, idesc_pv, j > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 1; kk < ATT_BN / 16; ++kk)
                    mma_bf16_ts(d_o, a_p + kk * 8, vd + ((kk * 16 * 128) >> 4), idesc_pv, 1u);
                mma_commit(&pv_done[x]);
                return true;
            };
            auto k_ready = [&](int j) {
                return mma_wait(&k_full[j % ATT_K_STAGES], (j / ATT_K_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA);
            };
            ok = ok && k_ready(0) && (nkv[0] == 0 || scores(0, 0)) && scores(1, 0);
            if (ok) mma_commit(&k_empty[0]);
            for (int j = 0; j < nkv_b && ok; ++j) {
                const bool next = j + 1 < nkv_b;
                if (next && !k_ready(j + 1)) { ok = false; break; }
                if (j + 1 < nkv[0] && !scores(0, j + 1)) { ok = false; break; }
                if (!mma_wait(&v_full[j % ATT_V_STAGES], (j / ATT_V_STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) {
                    ok = false;
                    break;
                }
                if (j < nkv[0] && !values(0, j)) { ok = false; break; }
                if (next) {
                    if (!scores(1, j + 1)) { ok = false; break; }
                    mma_commit(&k_empty[(j + 1) % ATT_K_STAGES]);   // both tiles' scores of K_{j+1} issued
                }
                if (!values(1, j)) { ok = false; break; }
                mma_commit(&v_empty[j % ATT_V_STAGES]);             // both tiles' P.V of V_j issued
            }
            mma_commit(drain);
            mbar_wait(drain, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else {
        // ---------------------------------- softmax ----------------------------------
        const int x = (warp - 2) >> 2;                    // query tile of this warpgroup
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;                     // row in the tile
        const int qt0 = q0 + x * ATT_BM;                  // first query of the tile
        const int qi = qt0 + r;                           // query index in the request
        const int nkv = x == 0 ? nkv_a : nkv_b;
        const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
        const uint32_t t_s = tmem + lane_off, t_p = tmem + 128 + x * 64 + lane_off;
        const uint32_t t_o = tmem + 256 + x * 128 + lane_off;
        const float c = args.scale_log2;
        float m_use = -1e30f;                             // running max (exp2 domain) in use
        float l = 0.f;                                    // running sum of p
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            bool w = true;
            if (lane == 0) w = mma_wait(&s_full[x], j & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
            tc_fence_after();
            uint32_t sr[128];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t (&part)[32] = *reinterpret_cast<uint32_t (*)[32]>(&sr[cc * 32]);
                tmem_ld_32x32b_x32(t_s + cc * 32, part);
            }
            tmem_ld_wait();
            // S goes back to the MMA issuer for the other tile's scores
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            // causal and length mask on the tile that reaches the diagonal or the end
            const int k0 = j * ATT_BN;
            if (k0 + ATT_BN - 1 > qt0 || k0 + ATT_BN > args.L) {
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    if (k0 + i > qi || k0 + i >= args.L) sr[i] = __float_as_uint(-INFINITY);
            }
            // row max: eight independent chains of three-input max
            float mp[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mp[e] = fmax3(__uint_as_float(sr[e]), __uint_as_float(sr[8 + e]),
                                                    __uint_as_float(sr[16 + e]));
#pragma unroll
            for (int i = 24; i < 128; i += 16) {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    mp[e] = fmax3(mp[e], __uint_as_float(sr[i + e]), __uint_as_float(sr[i + 8 + e]));
            }
            const float mx = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7])) * c;
            float alpha = 1.f;
            const bool rescale = mx > m_use + ATT_RESCALE_LOG2;
            if (rescale) {
                alpha = fast_exp2(m_use - mx);
                m_use = mx;
            }
            // p = 2^(s c - m): one f32x2 fma per two scores, two exp2, one f32x2 add into four
            // partial sums, one bf16x2 pack
            const unsigned long long c2 = f2_pack(c, c);
            const unsigned long long nm2 = f2_pack(-m_use, -m_use);
            unsigned long long sp[4] = {0ull, 0ull, 0ull, 0ull};
            uint32_t pk[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                const unsigned long long x2 = f2_fma(f2_pack(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])),
                                                     c2, nm2);
                float x0, x1;
                f2_unpack(x2, x0, x1);
                const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
                sp[i & 3] = f2_add(sp[i & 3], f2_pack(p0, p1));
                pk[i] = pack_bf16(p0, p1);
            }
            float a0, a1, b0, b1, d0, d1, e0, e1;
            f2_unpack(sp[0], a0, a1);
            f2_unpack(sp[1], b0, b1);
            f2_unpack(sp[2], d0, d1);
            f2_unpack(sp[3], e0, e1);
            l = l * alpha + (((a0 + a1) + (b0 + b1)) + ((d0 + d1) + (e0 + e1)));
            // P_X and O_X are free again once the previous P.V is done
            if (j >= 1) {
                if (lane == 0) w = mma_wait(&pv_done[x], (j - 1) & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
                if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
                tc_fence_after();
            }
            if (j >= 1 && rescale) {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(t_o + cc * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st_32x32b_x32(t_o + cc * 32, o);
                }
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t (&part)[32] = *reinterpret_cast<uint32_t (*)[32]>(&pk[half * 32]);
                tmem_st_32x32b_x32(t_p + half * 32, part);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[x]);
        }
        if (ok && nkv > 0) {
            // the tile's last P.V is done: normalise and store this thread's output row
            const int jl = nkv - 1;
            bool w = true;
            if (lane == 0) w = mbar_wait(&pv_done[x], jl & 1u, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (__shfl_sync(0xffffffffu, w, 0)) {
                tc_fence_after();
                const float inv = 1.f / l;
                __nv_bfloat16* orow = args.out + static_cast<long>(row0 + qi) * args.ld_out + h * ATT_D;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(t_o + cc * 32, o);
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
