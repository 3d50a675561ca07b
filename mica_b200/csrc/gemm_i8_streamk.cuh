// gemm_i8_streamk.cuh -- stream-K W8A8 GEMM for sm_100a: the last partial wave spread evenly.
//
// When a grid of 128 x BN tiles is a little more than a multiple of the SM count (M 2048 x
// N 3072 = 192 tiles of 128 x 256 on 148 SMs, too many for one wave even at 128 x 320), the
// data-parallel kernel's critical path is whole extra tiles. Here the G persistent CTAs (one per SM, co-resident: cooperative
// launch) share the tiles x k-blocks units equally: CTA c takes units
// [c * U / G, (c + 1) * U / G), U = tiles * num_kb, in tile-major order. With tiles >= G every
// CTA's run spans at least one tile's k-blocks, so a tile is cut at most once, between two
// neighbouring CTAs:
//   - CTA c + 1 starts in the middle of the tile (k-blocks [j, num_kb)): its first segment is
//     a STORE: the int32 accumulator goes to workspace slot c + 1, then four per-warp flags
//     are released;
//   - CTA c ends in it (k-blocks [0, j)): its last segment is a FINISH: while that segment's
//     MMAs run, each epilogue warp waits for its flag (acquire, bounded) and copies the stored
//     partial into the other (idle) TMEM accumulator buffer; the epilogue then adds the two
//     buffers and runs the usual dequant. Integer addition keeps the result bit-exact.
// A STORE never waits, and a FINISH waits only for a STORE that its neighbour issues first
// thing, so there is no cycle. Warp roles, the stage ring, the double-buffered TMEM
// accumulator and the TMA store epilogue are those of gemm_i8_kernel (gemm_i8.cuh).
//
// Workspace (caller's, 16-byte aligned): [0, 4096) flags, u32 [G][4], zeroed before the
// launch; from byte 4096, G slots of 128 x BN int32 in the order [quarter][chunk][16-byte
// group][lane] so that a warp's 16-byte stores or loads cover 512 contiguous bytes.
#pragma once

#include "gemm_i8.cuh"

namespace mica {

constexpr int SK_FLAG_BYTES = 4096;

__device__ __forceinline__ void st_global_cg_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.global.cg.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_global_cg_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One CTA's run of units as segments (tile, kb0, kb1).
struct SkRun {
    long u, end;
    int num_kb;
    __device__ SkRun(long total, int G, int c, int nkb)
        : u(total * c / G), end(total * (c + 1) / G), num_kb(nkb) {}
    __device__ bool next(int& tile, int& kb0, int& kb1) {
        if (u >= end) return false;
        tile = static_cast<int>(u / num_kb);
        kb0 = static_cast<int>(u % num_kb);
        const long left = end - u;
        kb1 = left < static_cast<long>(num_kb - kb0) ? kb0 + static_cast<int>(left) : num_kb;
        u += kb1 - kb0;
        return true;
    }
};

template <int BN, typename OutT>
__global__ void __launch_bounds__(64 + 32 * 4, 1)
gemm_i8_streamk_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       const __grid_constant__ CUtensorMap tmap_c, const GemmArgs args, uint8_t* workspace) {
    using S = GemmShape<BN, 4>;
    constexpr int STAGES = S::STAGES;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + STAGES * S::A_BYTES;
    uint8_t* smem_epi = smem_b + STAGES * S::B_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + S::EPI_BYTES);
    uint64_t* full_bar = bars;
    uint64_t* empty_bar = bars + STAGES;
    uint64_t* tfull_bar = bars + 2 * STAGES;
    uint64_t* tempty_bar = bars + 2 * STAGES + 2;
    uint64_t* drain_bar = bars + 2 * STAGES + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int M = args.M, N = args.N, K = args.K;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = ((M + S::BM - 1) / S::BM) * num_n;
    const int num_kb = (K + S::BK - 1) / S::BK;
    const long total = static_cast<long>(num_tiles) * num_kb;
    const int G = gridDim.x;
    const int cta = blockIdx.x;
    uint32_t* flags = reinterpret_cast<uint32_t*>(workspace);
    int32_t* slots = reinterpret_cast<int32_t*>(workspace + SK_FLAG_BYTES);
    constexpr long SLOT_INTS = 128L * BN;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull_bar[i], 1);
            mbar_init(&tempty_bar[i], S::EPI_WARPS * 32);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        tma_prefetch_desc(&tmap_c);
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------- TMA producer -------------------------------
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            const uint64_t pol_b = policy_evict_last();
            SkRun run(total, G, cta, num_kb);
            int tile, kb0, kb1;
            while (ok && run.next(tile, kb0, kb1)) {
                const int m0 = (tile / num_n) * S::BM;
                const int n0 = (tile % num_n) * BN;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int st = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    if (!mbar_wait(&empty_bar[st], ph ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_bar[st], S::STAGE_BYTES);
                    tma_load_2d(smem_a + st * S::A_BYTES, &tmap_a, &full_bar[st], kb * S::BK, m0);
                    tma_load_2d_hint(smem_b + st * S::B_BYTES, &tmap_b, &full_bar[st], kb * S::BK, n0, pol_b);
                }
            }
            const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
            for (uint32_t j = first; j < it; ++j) {
                mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------- MMA issuer ---------------------------------
        constexpr uint32_t idesc = idesc_i8(S::BM, BN);
        const uint32_t a_base = smem_u32(smem_a);
        const uint32_t b_base = smem_u32(smem_b);
        uint32_t it = 0;
        int local = 0;
        bool ok = true;
        SkRun run(total, G, cta, num_kb);
        int tile, kb0, kb1;
        while (ok && run.next(tile, kb0, kb1)) {
            const int acc = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            ++local;
            bool w = true;
            if (lane == 0) w = mbar_wait(&tempty_bar[acc], acc_ph ^ 1u, abort_flag, MICA_DEV_TIMEOUT_MMA);
            if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * S::ACC_COLS;
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int st = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1u;
                if (lane == 0) w = mbar_wait(&full_bar[st], ph, abort_flag, MICA_DEV_TIMEOUT_MMA);
                if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_addr = a_base + st * S::A_BYTES;
                    const uint32_t b_addr = b_base + st * S::B_BYTES;
#pragma unroll
                    for (int k = 0; k < S::BK / S::UMMA_K; ++k) {
                        mma_i8(d_tmem, smem_desc_k128(a_addr + k * S::UMMA_K), smem_desc_k128(b_addr + k * S::UMMA_K),
                               idesc, (kb != kb0 || k != 0) ? 1u : 0u);
                    }
                    mma_commit(&empty_bar[st]);
                    if (kb == kb1 - 1) mma_commit(&tfull_bar[acc]);
                }
                __syncwarp();
            }
        }
        if (lane == 0) {
            mma_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else {
        // ------------------------------- epilogue -----------------------------------
        const int q4 = warp & 3;
        const int row_local = q4 * 32 + lane;
        const int ew = warp - 2;
        uint8_t* my_boxes = smem_epi + ew * S::BOX_BUFS * S::BOX_BYTES;
        int box_count = 0;
        int local = 0;
        const uint64_t pol_c = policy_evict_first();
        constexpr int CHUNKS = BN / 32;
        SkRun run(total, G, cta, num_kb);
        int tile, kb0, kb1;
        while (run.next(tile, kb0, kb1)) {
            const int m0 = (tile / num_n) * S::BM;
            const int n0 = (tile % num_n) * BN;
            const int acc = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            ++local;
            // row scale and column-vector lines fetched before any wait (gemm_i8.cuh)
            if (m0 + row_local < M) prefetch_l1(args.sa + m0 + row_local);
            if (lane * 32 < BN && n0 + lane * 32 < N) {
                prefetch_l1(args.sb + n0 + lane * 32);
                if (args.bias != nullptr) prefetch_l1(args.bias + n0 + lane * 32);
            }
            const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q4 * 32) << 16);
            const uint32_t t_row = lane_base + acc * S::ACC_COLS;
            // FINISH (kb0 == 0, kb1 < num_kb): the rest of this tile is CTA cta + 1's STORE. It is
            // this CTA's last segment, so the other accumulator buffer is free: the partial is
            // copied there while this segment's MMAs still run, and the epilogue adds the two.
            const bool finish = kb0 == 0 && kb1 < num_kb;
            const uint32_t p_row = lane_base + (acc ^ 1) * S::ACC_COLS;
            if (finish) {
                bool ok = true;
                if (lane == 0) {
                    const uint32_t* f = flags + (cta + 1) * 4 + q4;
                    const unsigned long long t0 = global_ns();
                    for (uint32_t it = 0; ld_acquire_gpu_u32(f) == 0u; ++it) {
                        if (*abort_flag) { ok = false; break; }
                        if ((it & 15u) == 15u && global_ns() - t0 > kWaitLimitNs) {
                            *abort_flag = 1u;
                            atomicExch(&g_dev_error, MICA_DEV_TIMEOUT_STREAMK);
                            ok = false;
                            break;
                        }
                        __nanosleep(32);
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) break;
                (void)ld_acquire_gpu_u32(flags + (cta + 1) * 4 + q4);   // acquire on every lane
                const int32_t* part = slots + (cta + 1) * SLOT_INTS + q4 * (CHUNKS * 8 * 32 * 4);
#pragma unroll 2
                for (int cc = 0; cc < CHUNKS; ++cc) {
                    uint32_t v[32];
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const uint4 p = ld_global_cg_v4(part + ((cc * 8 + g) * 32 + lane) * 4);
                        v[4 * g] = p.x;
                        v[4 * g + 1] = p.y;
                        v[4 * g + 2] = p.z;
                        v[4 * g + 3] = p.w;
                    }
                    tmem_st_32x32b_x32(p_row + cc * 32, v);
                }
                tmem_st_wait();
            }
            bool w = true;
            if (lane == 0) w = mbar_wait(&tfull_bar[acc], acc_ph, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (!__shfl_sync(0xffffffffu, w, 0)) break;
            tc_fence_after();

            if (kb0 > 0) {
                // STORE: this warp's 32 rows of the partial accumulator into slot `cta`.
                int32_t* slot = slots + cta * SLOT_INTS + q4 * (CHUNKS * 8 * 32 * 4);
#pragma unroll 1
                for (int cc = 0; cc < CHUNKS; ++cc) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + cc * 32, r);
                    tmem_ld_wait();
                    reg_pin32(r);
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        st_global_cg_v4(slot + ((cc * 8 + g) * 32 + lane) * 4, r[4 * g], r[4 * g + 1], r[4 * g + 2],
                                        r[4 * g + 3]);
                    }
                }
                tc_fence_before();
                mbar_arrive(&tempty_bar[acc]);
                __threadfence();
                __syncwarp();
                if (lane == 0) st_release_gpu_u32(flags + cta * 4 + q4, 1u);
                continue;
            }

            const int grow = m0 + row_local;
            const float sa_v = grow < M ? args.sa[grow] : 0.f;
            constexpr int COLS_PER_BOX = 128 / static_cast<int>(sizeof(OutT));
            constexpr int CHUNKS_PER_BOX = COLS_PER_BOX / 32;
            constexpr int BOXES = BN / COLS_PER_BOX;
            // lane j's scale and bias of column j of the next chunk are loaded one chunk ahead
            // (gemm_i8.cuh load_sb4): loaded at the chunk's start they cost an L2 round trip each
            float sb_n = n0 + lane < N ? args.sb[n0 + lane] : 0.f;
            float bias_n = (args.bias != nullptr && n0 + lane < N) ? args.bias[n0 + lane] : 0.f;
#pragma unroll 1
            for (int bx = 0; bx < BOXES; ++bx, ++box_count) {
                uint8_t* box = my_boxes + (box_count % S::BOX_BUFS) * S::BOX_BYTES;
                if (lane == 0) tma_store_wait_read<1>();
                __syncwarp();
                const uint32_t box_row = smem_u32(box) + lane * 128;
#pragma unroll
                for (int cc = 0; cc < CHUNKS_PER_BOX; ++cc) {
                    const int col0 = bx * COLS_PER_BOX + cc * 32;
                    const float sb_l = sb_n, bias_l = bias_n;
                    const int ncol = n0 + col0 + 32 + lane;
                    if (col0 + 32 < BN) {
                        sb_n = ncol < N ? args.sb[ncol] : 0.f;
                        bias_n = (args.bias != nullptr && ncol < N) ? args.bias[ncol] : 0.f;
                    }
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + col0, r);
                    if (finish) {
                        uint32_t p[32];
                        tmem_ld_32x32b_x32(p_row + col0, p);
                        tmem_ld_wait();
                        reg_pin32(r);
                        reg_pin32(p);
#pragma unroll
                        for (int j = 0; j < 32; ++j) r[j] += p[j];
                    } else {
                        tmem_ld_wait();
                        reg_pin32(r);
                    }
                    dequant_chunk_to_box<OutT>(r, sa_v, sb_l, bias_l, args.bias != nullptr, box_row, cc);
                }
                if (bx + 1 == BOXES) {
                    tc_fence_before();
                    mbar_arrive(&tempty_bar[acc]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int x = n0 + bx * COLS_PER_BOX, y = m0 + q4 * 32;
                    if (x < N && y < M) tma_store_2d_hint(&tmap_c, box, x, y, pol_c);
                    tma_store_commit();
                }
            }
        }
        if (lane == 0) tma_store_wait_all<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_free(tmem_base, S::TMEM_COLS);
    }
}

}  // namespace mica
