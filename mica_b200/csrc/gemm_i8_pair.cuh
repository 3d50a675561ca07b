// gemm_i8_pair.cuh -- W8A8 GEMM on CTA pairs (tcgen05 cta_group::2), 256 x BN output tiles.
//
// A cluster of two CTAs on two SMs computes one 256 x BN tile with a single stream of
// tcgen05.mma.cta_group::2.kind::i8 instructions (256 x BN x 32 each) issued by the even
// CTA. Each CTA holds 128 rows of A and BN/2 rows of B per stage in its own shared memory
// (at identical offsets), so per SM the MMA reads 16 KB of A and 16 KB of B per 128-byte K
// step instead of 16 + 32 KB in the single-CTA kernel. A 128 x 256 single-CTA MMA asks the
// shared memory for 96 bytes per clock of operands while TMA writes the next stages at the
// same rate, more than its bandwidth; on pairs both halve, which is what lets this tile keep
// the tensor pipe busy.
//
// Loads: each CTA's producer issues its own two loads per stage (its A rows and its half of
// B) into its own shared memory, and both complete their bytes on the EVEN CTA's full
// barrier, which the even producer arms with the pair's byte count (.cta_group::2 TMA; a
// byte count may land before the arming, the transaction count is signed). So every SM's
// TMA unit moves 32 KB per stage, and the MMA issuer waits on one local barrier.
// The MMA commit of a stage arrives on both CTAs' empty barriers (two commits), so each
// producer refills its own stages as soon as the pair's MMAs are done with them.
//
// Synchronisation (all waits bounded, as in gemm_i8.cuh):
//   full[s]    even CTA: the pair's four TMA loads of the stage complete their bytes on it;
//   empty[s]   per CTA: the even CTA's MMA commit of the stage arrives on both copies;
//   tfull[a]   per CTA: the even CTA's last commit of a tile arrives on both copies;
//   tempty[a]  even CTA only: one arrival per epilogue warp of the pair (8).
// Epilogue and semantics are those of gemm_i8_kernel (dequant, no FMA, TMA store).
#pragma once

#include "gemm_i8.cuh"

namespace mica {

template <int BN_>
struct PairShape {
    static constexpr int BN = BN_;
    static constexpr int BM = 256;                      // rows per pair tile (128 per CTA)
    static constexpr int BK = 128;
    static constexpr int UMMA_K = 32;
    static constexpr int A_BYTES = 128 * BK;            // this CTA's 128 rows
    static constexpr int B_BYTES = (BN / 2) * BK;       // this CTA's half of B's rows
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_WARPS = 4;
    static constexpr int BOX_BYTES = 32 * 128;
    static constexpr int EPI_BYTES = EPI_WARPS * 2 * BOX_BYTES;
    static constexpr int AUX_BYTES = 256;
    static constexpr int SMEM_OPTIN = 232448;
    static constexpr int STAGES_RAW = (SMEM_OPTIN - 1024 - EPI_BYTES - AUX_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + AUX_BYTES;
    static constexpr int ACC_COLS = BN;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int THREADS = 192;
    static_assert(BN == 128 || BN == 256, "pair tile width");
    static_assert(SMEM_BYTES <= SMEM_OPTIN, "smem");
};

template <int BN, typename OutT>
__global__ void __launch_bounds__(192, 1)
gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_c, const GemmArgs args) {
    using S = PairShape<BN>;
    constexpr int STAGES = S::STAGES;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();      // 0 = the CTA that issues the MMAs
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
    uint64_t* tempty_bar = bars + 2 * STAGES + 2;
    uint64_t* drain_bar = bars + 2 * STAGES + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int M = args.M, N = args.N, K = args.K;
    const int num_m = (M + S::BM - 1) / S::BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + S::BK - 1) / S::BK;
    const int cluster_id = blockIdx.x >> 1;
    const int num_clusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull_bar[i], 1);
            mbar_init(&tempty_bar[i], 2 * S::EPI_WARPS);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        tma_prefetch_desc(&tmap_c);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    cluster_sync();            // barriers of both CTAs initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------- TMA producers (both CTAs) -------------------
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            const uint64_t pol_b = policy_evict_last();
            const uint64_t pol_a = policy_evict_normal();  // activations: re-read by every N tile
            for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters) {
                int mt, nt;
                tile_origin(tile, num_m, num_n, args.panel, mt, nt);
                const int m0 = mt * S::BM;
                const int n0 = nt * BN;
                for (int kb = 0; kb < num_kb; ++kb, ++it) {
                    const int st = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    if (!mbar_wait(&empty_bar[st], ph ^ 1u, abort_flag, MICA_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = map_to_rank(smem_u32(&full_bar[st]), 0);
                    if (leader) mbar_arrive_expect_tx(&full_bar[st], 2 * S::STAGE_BYTES);
                    tma_load_2d_pair(map_to_rank(smem_u32(smem_a + st * S::A_BYTES), rank), &tmap_a, full,
                                     kb * S::BK, m0 + static_cast<int>(rank) * 128, pol_a);
                    tma_load_2d_pair(map_to_rank(smem_u32(smem_b + st * S::B_BYTES), rank), &tmap_b, full,
                                     kb * S::BK, n0 + static_cast<int>(rank) * (BN / 2), pol_b);
                }
            }
            // Drain: every stage this CTA loaded has been consumed by the pair's MMAs (so its
            // bytes have landed) before the CTA reaches the closing cluster barrier.
            const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
            for (uint32_t j = first; j < it && ok; ++j)
                mbar_wait(&empty_bar[j % STAGES], (j / STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------- MMA issuer (even CTA) -----------------------
        // One lane runs the loop (see gemm_i8_kernel): a wait per stage, the k-step MMAs, a
        // commit to both CTAs' empty barriers; a tcgen05 fence only per accumulator hand-back.
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_i8(S::BM, BN);
            const uint64_t a_desc0 = smem_desc_k128(smem_u32(smem_a));
            const uint64_t b_desc0 = smem_desc_k128(smem_u32(smem_b));
            uint32_t it = 0;
            int local = 0;
            bool ok = true;
            for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters, ++local) {
                const int acc = local & 1;
                const uint32_t acc_ph = (local >> 1) & 1;
                if (!mbar_wait(&tempty_bar[acc], acc_ph ^ 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * S::ACC_COLS;
                for (int kb = 0; kb < num_kb; ++kb, ++it) {
                    const int st = it % STAGES;
                    if (!mbar_wait(&full_bar[st], (it / STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    const uint64_t a_st = a_desc0 + static_cast<uint64_t>((st * S::A_BYTES) >> 4);
                    const uint64_t b_st = b_desc0 + static_cast<uint64_t>((st * S::B_BYTES) >> 4);
#pragma unroll
                    for (int k = 0; k < S::BK / S::UMMA_K; ++k) {
                        mma_i8_pair(d_tmem, a_st + static_cast<uint64_t>((k * S::UMMA_K) >> 4),
                                    b_st + static_cast<uint64_t>((k * S::UMMA_K) >> 4), idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    const uint32_t e = smem_u32(&empty_bar[st]);
                    mma_commit_pair(map_to_rank(e, 0));
                    mma_commit_pair(map_to_rank(e, 1));
                    if (kb == num_kb - 1) {
                        const uint32_t f = smem_u32(&tfull_bar[acc]);
                        mma_commit_pair(map_to_rank(f, 0));
                        mma_commit_pair(map_to_rank(f, 1));
                    }
                }
            }
            mma_commit_pair(map_to_rank(smem_u32(drain_bar), 0));
            mbar_wait(drain_bar, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else {
        // ------------------------------- epilogue (both CTAs) ------------------------
        const int q4 = warp & 3;
        const int row_local = static_cast<int>(rank) * 128 + q4 * 32 + lane;
        const int ew = warp - 2;
        uint8_t* my_boxes = smem_epi + ew * 2 * S::BOX_BYTES;
        int box_count = 0;
        int local = 0;
        const uint64_t pol_c = policy_evict_first();   // output: written once, leave L2 to the weights
        constexpr int COLS_PER_BOX = 128 / static_cast<int>(sizeof(OutT));
        constexpr int CHUNKS_PER_BOX = COLS_PER_BOX / 32;
        constexpr int BOXES = BN / COLS_PER_BOX;
        for (int tile = cluster_id; tile < num_tiles; tile += num_clusters, ++local) {
            int mt, nt;
            tile_origin(tile, num_m, num_n, args.panel, mt, nt);
            const int m0 = mt * S::BM;
            const int n0 = nt * BN;
            const int acc = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            // row scale and column-vector lines fetched before the accumulator wait (gemm_i8.cuh)
            const int grow = m0 + row_local;
            const float sa_v = grow < M ? __ldg(args.sa + grow) : 0.f;
            if (lane * 32 < BN && n0 + lane * 32 < N) {
                prefetch_l1(args.sb + n0 + lane * 32);
                if (args.bias != nullptr) prefetch_l1(args.bias + n0 + lane * 32);
            }
            float4 sb_cur[8];                                // the first chunk's scales (load_sb4)
            load_sb4(args, n0, N, sb_cur);
            bool w = true;
            if (lane == 0) w = mbar_wait(&tfull_bar[acc], acc_ph, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (!__shfl_sync(0xffffffffu, w, 0)) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q4 * 32) << 16) + acc * S::ACC_COLS;
#pragma unroll 1
            for (int bx = 0; bx < BOXES; ++bx, ++box_count) {
                uint8_t* box = my_boxes + (box_count & 1) * S::BOX_BYTES;
                if (lane == 0) tma_store_wait_read<1>();
                __syncwarp();
                const uint32_t box_row = smem_u32(box) + lane * 128;
#pragma unroll
                for (int cc = 0; cc < CHUNKS_PER_BOX; ++cc) {
                    const int col0 = bx * COLS_PER_BOX + cc * 32;
                    const int ncol = col0 + 32;                  // the next chunk's scales in flight
                    float4 sb_nxt[8];
                    if (ncol < BN) load_sb4(args, n0 + ncol, N, sb_nxt);
                    dequant_chunk<OutT>(args, t_row + col0, n0 + col0, N, sa_v, sb_cur, box_row, cc);
                    if (ncol < BN) {
#pragma unroll
                        for (int v = 0; v < 8; ++v) sb_cur[v] = sb_nxt[v];
                    }
                }
                if (bx == BOXES - 1) {
                    // this warp's last read of the accumulator: one arrival for the warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&tempty_bar[acc]), 0));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int x = n0 + bx * COLS_PER_BOX, y = m0 + static_cast<int>(rank) * 128 + q4 * 32;
                    if (x < N && y < M) tma_store_2d_hint(&tmap_c, box, x, y, pol_c);   // edge boxes hold nothing
                    tma_store_commit();
                }
            }
        }
        if (lane == 0) tma_store_wait_all<0>();
        __syncwarp();
    }

    // A CTA that gave up may still have TMA loads in flight that count on the other CTA's
    // barrier; give them time to land before the pair's shared memory is released.
    if (*abort_flag) {
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_before();
    cluster_sync();            // the even CTA's MMAs read this CTA's smem: leave together
    if (warp == 1) {
        tc_fence_after();
        tmem_free_pair(tmem_base, S::TMEM_COLS);
    }
}

}  // namespace mica
