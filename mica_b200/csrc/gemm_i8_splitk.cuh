// gemm_i8_splitk.cuh -- W8A8 GEMM with each output tile's K loop split across a cluster.
//
// For grids that would leave most SMs idle (few 128 x BN tiles: decode-sized and other small
// M), one output tile is computed by a cluster of S CTAs (2 <= S <= 8). CTA rank r runs the
// TMA + tcgen05 main loop of gemm_i8_kernel over k-blocks [r*ceil(kb/S), ...) into its own
// TMEM accumulator. A single CTA streams a tile's K at a bounded rate (one 128-byte k-block
// costs it about 0.4 us of TMA + MMA latency on B200), so splitting K over S SMs divides a
// small grid's main loop by about S.
//
// Reduction, in distributed shared memory, exact (int32 adds commute):
//   ranks 1..S-1  copy their int32 partial from TMEM into their own stage buffers (idle once
//                 the main loop has drained) as [16-byte column chunk][row], so that a warp's
//                 32 rows of one chunk are 512 contiguous bytes, then arrive (release.cluster)
//                 on the leader's `ready` barrier;
//   rank 0        waits on `ready` (acquire.cluster, bounded), adds the peers' partials to its
//                 own accumulator with ld.shared::cluster (one contiguous 512-byte read per
//                 warp and chunk; scattered 16-byte reads ran at ~25 GB/s per SM on B200), and
//                 runs the dequant epilogue of gemm_i8_kernel (same arithmetic and stores).
// Every CTA ends at a cluster barrier, so no CTA leaves while the leader may still read its
// shared memory. Every other wait is bounded (common.cuh); no global workspace is used.
#pragma once

#include "gemm_i8.cuh"

namespace mica {

__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint4 ld_shared_cluster_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
// Bounded wait whose completion also acquires, at cluster scope, what the arriving threads of
// other CTAs released (their shared-memory writes).
__device__ __forceinline__ bool mbar_wait_cluster_acquire(uint64_t* bar, uint32_t parity,
                                                          volatile uint32_t* abort_flag, int code) {
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (*abort_flag) return false;
        if ((it & 15u) == 15u && global_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1u;
            atomicExch(&g_dev_error, code);
            return false;
        }
    }
}

template <int BN, typename OutT>
__global__ void __launch_bounds__(192, 1)
gemm_i8_splitk_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_c, const GemmArgs args) {
    using S = GemmShape<BN, 4>;
    constexpr int STAGES = S::STAGES;
    static_assert(128 * BN * 4 <= STAGES * S::STAGE_BYTES, "the partial must fit in the stage buffers");
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t nsplit = cluster_nctarank();
    const bool leader = rank == 0;

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
    uint64_t* ready_bar = bars + 2 * STAGES + 1;
    uint64_t* drain_bar = bars + 2 * STAGES + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 3);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int M = args.M, N = args.N, K = args.K;
    const int num_n = (N + BN - 1) / BN;
    const int num_kb = (K + S::BK - 1) / S::BK;
    const int tile = static_cast<int>(blockIdx.x / nsplit);
    const int m0 = (tile / num_n) * S::BM;
    const int n0 = (tile % num_n) * BN;
    const int kb_per = (num_kb + static_cast<int>(nsplit) - 1) / static_cast<int>(nsplit);
    const int kb0 = static_cast<int>(rank) * kb_per;
    const int kb1 = min(num_kb, kb0 + kb_per);   // the host keeps kb0 < kb1 for every rank

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(tfull_bar, 1);
        mbar_init(ready_bar, (nsplit - 1) * S::EPI_WARPS * 32);
        mbar_init(drain_bar, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        tma_prefetch_desc(&tmap_c);
    }
    if (warp == 1) tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    cluster_sync();            // every CTA's barriers initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------- TMA producer -------------------------------
        if (lane == 0) {
            const uint64_t pol_b = policy_evict_last();
            uint32_t it = 0;
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int st = it % STAGES;
                if (!mbar_wait(&empty_bar[st], ((it / STAGES) & 1u) ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER)) break;
                mbar_arrive_expect_tx(&full_bar[st], S::STAGE_BYTES);
                tma_load_2d(smem_a + st * S::A_BYTES, &tmap_a, &full_bar[st], kb * S::BK, m0);
                tma_load_2d_hint(smem_b + st * S::B_BYTES, &tmap_b, &full_bar[st], kb * S::BK, n0, pol_b);
            }
            const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
            for (uint32_t j = first; j < it; ++j)
                mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------- MMA issuer ---------------------------------
        constexpr uint32_t idesc = idesc_i8(S::BM, BN);
        const uint32_t a_base = smem_u32(smem_a);
        const uint32_t b_base = smem_u32(smem_b);
        uint32_t it = 0;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int st = it % STAGES;
            bool w = true;
            if (lane == 0) w = mbar_wait(&full_bar[st], (it / STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA);
            if (!__shfl_sync(0xffffffffu, w, 0)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a_addr = a_base + st * S::A_BYTES;
                const uint32_t b_addr = b_base + st * S::B_BYTES;
#pragma unroll
                for (int k = 0; k < S::BK / S::UMMA_K; ++k)
                    mma_i8(tmem_base, smem_desc_k128(a_addr + k * S::UMMA_K), smem_desc_k128(b_addr + k * S::UMMA_K),
                           idesc, (kb != kb0 || k != 0) ? 1u : 0u);
                mma_commit(&empty_bar[st]);
                if (kb == kb1 - 1) mma_commit(tfull_bar);
            }
            __syncwarp();
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
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q4 * 32) << 16);
        // this row's int32 partial in the stage buffers: 16-byte chunk c of row r at
        // (c * 128 + r) * 16, so one warp's 32 rows of a chunk are contiguous
        const uint32_t part_row = smem_u32(smem) + static_cast<uint32_t>(row_local) * 16u;
        // row scale and column-vector lines fetched before the accumulator wait (gemm_i8.cuh)
        if (m0 + row_local < M) prefetch_l1(args.sa + m0 + row_local);
        if (lane * 32 < BN && n0 + lane * 32 < N) {
            prefetch_l1(args.sb + n0 + lane * 32);
            if (args.bias != nullptr) prefetch_l1(args.bias + n0 + lane * 32);
        }
        bool w = true;
        if (lane == 0) w = mbar_wait(tfull_bar, 0, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
        w = __shfl_sync(0xffffffffu, w, 0);
        tc_fence_after();
        if (!leader) {
            if (w) {
#pragma unroll 1
                for (int col0 = 0; col0 < BN; col0 += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + col0, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t c = static_cast<uint32_t>(col0 / 4 + j);
                        st_shared_v4(part_row + c * 2048u, r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
                    }
                }
            }
            // arrive even after a failed wait: the leader then finds its own abort or times out
            mbar_arrive_cluster(map_to_rank(smem_u32(ready_bar), 0));
        } else {
            bool ok = w;
            if (lane == 0 && ok && nsplit > 1)
                ok = mbar_wait_cluster_acquire(ready_bar, 0, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok) {
                const int ew = warp - 2;
                uint8_t* my_boxes = smem_epi + ew * S::BOX_BUFS * S::BOX_BYTES;
                const uint64_t pol_c = policy_evict_first();
                const int grow = m0 + row_local;
                const float sa_v = grow < M ? args.sa[grow] : 0.f;
                constexpr int COLS_PER_BOX = 128 / static_cast<int>(sizeof(OutT));
                constexpr int CHUNKS_PER_BOX = COLS_PER_BOX / 32;
                constexpr int BOXES = BN / COLS_PER_BOX;
#pragma unroll 1
                for (int bx = 0; bx < BOXES; ++bx) {
                    uint8_t* box = my_boxes + (bx % S::BOX_BUFS) * S::BOX_BYTES;
                    if (lane == 0) tma_store_wait_read<S::BOX_BUFS - 1>();
                    __syncwarp();
                    const uint32_t box_row = smem_u32(box) + lane * 128;
#pragma unroll
                    for (int cc = 0; cc < CHUNKS_PER_BOX; ++cc) {
                        const int col0 = bx * COLS_PER_BOX + cc * 32;
                        const int gcol = n0 + col0 + lane;
                        const float sb_l = gcol < N ? args.sb[gcol] : 0.f;
                        const float bias_l = (args.bias != nullptr && gcol < N) ? args.bias[gcol] : 0.f;
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(t_row + col0, r);
                        tmem_ld_wait();
                        // peers' 32 columns of this row: the next peer's eight loads are issued
                        // before the current peer's adds, so remote latencies overlap
                        const uint32_t c_addr = part_row + static_cast<uint32_t>(col0 / 4) * 2048u;
                        uint4 cur[8], nxt[8];
                        if (nsplit > 1) {      // always: the host launches 2 <= S <= 8
#pragma unroll
                            for (int j = 0; j < 8; ++j) cur[j] = ld_shared_cluster_v4(map_to_rank(c_addr + j * 2048u, 1));
                        }
                        for (uint32_t p = 1; p < nsplit; ++p) {
                            if (p + 1 < nsplit) {
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    nxt[j] = ld_shared_cluster_v4(map_to_rank(c_addr + j * 2048u, p + 1));
                            }
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                r[4 * j] += cur[j].x;
                                r[4 * j + 1] += cur[j].y;
                                r[4 * j + 2] += cur[j].z;
                                r[4 * j + 3] += cur[j].w;
                                cur[j] = nxt[j];
                            }
                        }
                        float y[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float sbj = __shfl_sync(0xffffffffu, sb_l, j);
                            y[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), sa_v), sbj);
                        }
                        if (args.bias != nullptr) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) y[j] = __fadd_rn(y[j], __shfl_sync(0xffffffffu, bias_l, j));
                        }
                        if constexpr (sizeof(OutT) == 2) {
                            uint32_t pk[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                if constexpr (std::is_same<OutT, __half>::value) pk[j] = pack_f16(y[2 * j], y[2 * j + 1]);
                                else pk[j] = pack_bf16(y[2 * j], y[2 * j + 1]);
                            }
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                const int chunk = cc * 4 + c;
                                st_shared_v4(box_row + ((chunk ^ (lane & 7)) << 4), pk[4 * c], pk[4 * c + 1],
                                             pk[4 * c + 2], pk[4 * c + 3]);
                            }
                        } else {
#pragma unroll
                            for (int c = 0; c < 8; ++c) {
                                st_shared_v4(box_row + ((c ^ (lane & 7)) << 4), __float_as_uint(y[4 * c]),
                                             __float_as_uint(y[4 * c + 1]), __float_as_uint(y[4 * c + 2]),
                                             __float_as_uint(y[4 * c + 3]));
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int x = n0 + bx * COLS_PER_BOX, yy = m0 + q4 * 32;
                        if (x < N && yy < M) tma_store_2d_hint(&tmap_c, box, x, yy, pol_c);
                        tma_store_commit();
                    }
                }
                if (lane == 0) tma_store_wait_all<0>();
                __syncwarp();
            }
        }
    }

    // No CTA leaves while the leader may still read its partial.
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_free(tmem_base, BN);
    }
}

}  // namespace mica
