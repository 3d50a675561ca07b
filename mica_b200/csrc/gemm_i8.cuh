// gemm_i8.cuh -- W8A8 GEMM for sm_100a on tcgen05 tensor cores.
//
//   C[m, n] = epilogue( sum_k A[m, k] * B[n, k] )      A int8 [M, K], B int8 [N, K] (K-major)
//
// One persistent CTA per SM walks output tiles of 128 x BN. Warp roles:
//   warp 0      TMA producer: 128 x 128-byte A and BN x 128-byte B tiles into a ring of
//               shared-memory stages (128-byte swizzle), completion on mbarriers;
//   warp 1      tensor-memory owner and MMA issuer: four tcgen05.mma.kind::i8 (128 x BN x 32)
//               per stage into an int32 accumulator in TMEM, double-buffered (2 x BN columns)
//               so the epilogue of tile i overlaps the main loop of tile i+1;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, fp32 dequant (and SwiGLU),
//               16-bit/fp32 pack into a swizzled shared tile, TMA store per 32-row box.
// Every wait is bounded (common.cuh); a wait that runs out unwinds the CTA.
//
// Reference semantics: v0.5/serving/kernel_src/kernels.py:41-69 (mm_i8): int32 accumulate,
// y = acc * SA[m] * SB[n] (+ BIAS[n]) evaluated left to right in fp32, cast to the output type.
#pragma once

#include "common.cuh"

namespace mica {

enum EpiKind { EPI_DEQUANT = 0, EPI_SWIGLU = 1 };

template <int BN_, int EW_ = 4>
struct GemmShape {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int EW = EW_;                      // epilogue warps: 4, or 8 (two per TMEM lane quarter)
    static constexpr int BK = 128;                      // bytes (= int8 elements) of K per stage
    static constexpr int UMMA_K = 32;                   // K of one kind::i8 MMA
    static constexpr int A_BYTES = BM * BK;             // 16 KB
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_WARPS = EW;
    static constexpr int BOX_BYTES = 32 * 128;          // one 32-row x 128-byte store box
    static constexpr int BOX_BUFS = EW == 4 ? 2 : 1;    // store boxes per epilogue warp
    static constexpr int EPI_BYTES = EPI_WARPS * BOX_BUFS * BOX_BYTES;
    static constexpr int COL_BYTES = BN * 4;            // the current tile's column scales (dequant)
    static constexpr int AUX_BYTES = 256;               // mbarriers, TMEM address, abort flag
    static constexpr int SMEM_OPTIN = 232448;           // sm_100 opt-in shared memory per block
    static constexpr int STAGES_RAW = (SMEM_OPTIN - 1024 - EPI_BYTES - COL_BYTES - AUX_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + COL_BYTES + AUX_BYTES;
    static constexpr int ACC_COLS = BN;                 // int32 accumulator columns per buffer
    // BN = 320 (wider than one MMA or one TMA box): two 160-wide halves per k-step, and one
    // accumulator buffer only (2 x 320 columns exceed the 512 of tensor memory), so the host
    // launches it with at most one tile per CTA.
    static constexpr int HALVES = BN > 256 ? 2 : 1;
    static constexpr int MMA_N = BN / HALVES;
    static constexpr int ACC_BUFS = BN > 256 ? 1 : 2;
    static constexpr int TMEM_COLS = ACC_BUFS * BN <= 32 ? 32 : (ACC_BUFS * BN <= 256 ? (ACC_BUFS * BN <= 128 ? 128 : 256) : 512);
    static constexpr int THREADS = 64 + 32 * EW;
    static_assert(EW == 4 || EW == 8, "epilogue warps");
    static_assert(STAGES >= 2, "not enough shared memory for a pipeline");
    static_assert(BN % 32 == 0 && BN >= 64 && (BN <= 256 || BN == 320), "BN");
    static_assert(ACC_BUFS * BN <= TMEM_COLS && TMEM_COLS <= 512, "tensor memory");
    static_assert(SMEM_BYTES <= SMEM_OPTIN, "smem");
};

struct GemmArgs {
    const float* sa;      // [M] token scales
    const float* sb;      // [N] channel scales
    const float* bias;    // [N] or nullptr
    int M, N, K;
    int round_mode;       // swiglu: rounding of the fused requantisation
    // swiglu only
    unsigned* row_amax;   // [M] float bits of max |h|
    unsigned* grid_sync;  // grid barrier counter (zeroed before launch)
    const __nv_bfloat16* h;  // [M, I] (read back in phase 2)
    long ldh;
    int8_t* q_out;        // [M, I]
    long ldq;
    float* s_out;         // [M]
    const float* inv_h;   // [I] or nullptr: down_proj's inv_smooth, applied before the requant
    int panel;            // n-tiles per weight panel (tile_origin); 0 = row-major over all of N
};

// Origin (m-tile, n-tile) of persistent tile `tile` in an num_m x num_n grid. With panel > 0 the
// n-tiles are cut into panels of `panel` columns and each panel is swept over all of M (m-major
// inside the panel), so consecutive waves share one panel of weights and it stays in L2; row-major
// order makes every wave touch all N x K weight bytes. Odd panels sweep M backwards, so a panel
// starts on the activation rows the previous one read last, which L2 still holds. The last panel
// may be narrower.
__device__ __forceinline__ void tile_origin(int tile, int num_m, int num_n, int panel, int& mt, int& nt) {
    if (panel <= 0 || panel >= num_n) {
        mt = tile / num_n;
        nt = tile % num_n;
        return;
    }
    const int per = num_m * panel;               // tiles in a full panel
    const int p = tile / per;
    const int n_base = p * panel;
    const int w = min(panel, num_n - n_base);
    const int u = tile - p * per;
    mt = (p & 1) ? num_m - 1 - u / w : u / w;
    nt = n_base + u % w;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// One 32-column chunk of the dequant epilogue for this lane's row: y = (acc * sa) * sb (+ bias)
// in fp32, no FMA, cast to OutT and written to chunk `cc` of the lane's 128-byte row of a
// 128-byte-swizzled store box. Lane j of the warp holds sb / bias of column j of the chunk.
template <typename OutT>
__device__ __forceinline__ void dequant_chunk_to_box(const uint32_t (&r)[32], float sa_v, float sb_l, float bias_l,
                                                     bool has_bias, uint32_t box_row, int cc) {
    const int lane = threadIdx.x & 31;
    float y[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float sbj = __shfl_sync(0xffffffffu, sb_l, j);
        y[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), sa_v), sbj);
    }
    if (has_bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = __fadd_rn(y[j], __shfl_sync(0xffffffffu, bias_l, j));
    }
    if constexpr (sizeof(OutT) == 2) {
        uint32_t p[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if constexpr (std::is_same<OutT, __half>::value) p[j] = pack_f16(y[2 * j], y[2 * j + 1]);
            else p[j] = pack_bf16(y[2 * j], y[2 * j + 1]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int chunk = cc * 4 + c;
            st_shared_v4(box_row + ((chunk ^ (lane & 7)) << 4), p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
        }
    } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            st_shared_v4(box_row + ((c ^ (lane & 7)) << 4), __float_as_uint(y[4 * c]), __float_as_uint(y[4 * c + 1]),
                         __float_as_uint(y[4 * c + 2]), __float_as_uint(y[4 * c + 3]));
        }
    }
}

// True when a chunk's 32 column scales (and biases) can be read as 16-byte vectors: the chunk
// lies inside N and both vectors are 16-byte aligned at its first column.
__device__ __forceinline__ bool chunk_vectorisable(const GemmArgs& a, int col, int N) {
    const uintptr_t bits = reinterpret_cast<uintptr_t>(a.sb + col) |
                           (a.bias != nullptr ? reinterpret_cast<uintptr_t>(a.bias + col) : 0u);
    return col + 32 <= N && (bits & 15u) == 0;
}

// The dequant epilogue of one whole 32-column chunk on packed fp32 pairs: the same
// y = (acc * sa) * sb (+ bias) per element, each step one IEEE round-to-nearest operation, as
// dequant_chunk_to_box, but the column scales arrive as eight uniform 16-byte loads (served
// from L1 after the first warp) instead of 32 shuffles, and every multiply covers two columns.
// sb4 holds the chunk's 32 scales; biasp is the chunk's first bias or nullptr.
template <typename OutT>
__device__ __forceinline__ void dequant_chunk_packed(const uint32_t (&r)[32], float sa_v, const float4 (&sb4)[8],
                                                     const float* biasp, uint32_t box_row, int cc) {
    const int lane = threadIdx.x & 31;
    const unsigned long long sa2 = f2_pack(sa_v, sa_v);
    unsigned long long y2[16];
#pragma unroll
    for (int v = 0; v < 8; ++v) {
        const unsigned long long a0 = f2_pack(__int2float_rn(static_cast<int>(r[4 * v])),
                                              __int2float_rn(static_cast<int>(r[4 * v + 1])));
        const unsigned long long a1 = f2_pack(__int2float_rn(static_cast<int>(r[4 * v + 2])),
                                              __int2float_rn(static_cast<int>(r[4 * v + 3])));
        y2[2 * v] = f2_mul(f2_mul(a0, sa2), f2_pack(sb4[v].x, sb4[v].y));
        y2[2 * v + 1] = f2_mul(f2_mul(a1, sa2), f2_pack(sb4[v].z, sb4[v].w));
    }
    if (biasp != nullptr) {
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(biasp) + v);
            y2[2 * v] = f2_add(y2[2 * v], f2_pack(b4.x, b4.y));
            y2[2 * v + 1] = f2_add(y2[2 * v + 1], f2_pack(b4.z, b4.w));
        }
    }
    if constexpr (sizeof(OutT) == 2) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            float lo, hi;
            f2_unpack(y2[j], lo, hi);
            if constexpr (std::is_same<OutT, __half>::value) pk[j] = pack_f16(lo, hi);
            else pk[j] = pack_bf16(lo, hi);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int chunk = cc * 4 + c;
            st_shared_v4(box_row + ((chunk ^ (lane & 7)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                         pk[4 * c + 3]);
        }
    } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float a, b, d, e;
            f2_unpack(y2[2 * c], a, b);
            f2_unpack(y2[2 * c + 1], d, e);
            st_shared_v4(box_row + ((c ^ (lane & 7)) << 4), __float_as_uint(a), __float_as_uint(b),
                         __float_as_uint(d), __float_as_uint(e));
        }
    }
}

// The column scales of one 32-column chunk as eight uniform 16-byte loads, when the chunk is
// vectorisable (else nothing: its gathered form loads its own). The CTA-pair kernel issues them
// one chunk ahead of use (gemm_i8_kernel stages a whole tile's in shared memory instead): a chunk
// that loads its scales at its own start waits an L2 round trip.
__device__ __forceinline__ void load_sb4(const GemmArgs& a, int gcol0, int N, float4 (&sb4)[8]) {
    if (chunk_vectorisable(a, gcol0, N)) {
#pragma unroll
        for (int v = 0; v < 8; ++v) sb4[v] = __ldg(reinterpret_cast<const float4*>(a.sb + gcol0) + v);
    }
}

// One 32-column chunk of the dequant epilogue: tensor-memory load of the lane's row, then the
// packed form (with the chunk's scales sb4 already loaded by load_sb4) when the chunk's column
// vectors allow it, else the gathered form.
template <typename OutT>
__device__ __forceinline__ void dequant_chunk(const GemmArgs& args, uint32_t t_addr, int gcol0, int N, float sa_v,
                                              const float4 (&sb4)[8], uint32_t box_row, int cc) {
    const int lane = threadIdx.x & 31;
    uint32_t r[32];
    if (chunk_vectorisable(args, gcol0, N)) {
        tmem_ld_32x32b_x32(t_addr, r);
        tmem_ld_wait();
        dequant_chunk_packed<OutT>(r, sa_v, sb4, args.bias != nullptr ? args.bias + gcol0 : nullptr, box_row, cc);
    } else {
        const int gcol = gcol0 + lane;
        const float sb_l = gcol < N ? args.sb[gcol] : 0.f;
        const float bias_l = (args.bias != nullptr && gcol < N) ? args.bias[gcol] : 0.f;
        tmem_ld_32x32b_x32(t_addr, r);
        tmem_ld_wait();
        dequant_chunk_to_box<OutT>(r, sa_v, sb_l, bias_l, args.bias != nullptr, box_row, cc);
    }
}

// The SwiGLU epilogue's per-lane column values of one 32-column chunk at tile column col0: lane
// j's gate/up bias of column col0 + j and down_proj's smoothing of h column col0 / 2 + (j & 15),
// each only when present (the scales come from the tile's shared-memory copy). Loaded one chunk
// ahead of use.
struct SwigluCols {
    float bias, inv;
};
__device__ __forceinline__ SwigluCols load_swiglu_cols(const GemmArgs& a, int gcol0, int N) {
    const int lane = threadIdx.x & 31;
    const int gcol = gcol0 + lane;
    const int hcol = gcol0 / 2 + (lane & 15);
    SwigluCols c;
    c.bias = (a.bias != nullptr && gcol < N) ? a.bias[gcol] : 0.f;
    c.inv = (a.inv_h != nullptr && hcol < N / 2) ? a.inv_h[hcol] : 1.f;
    return c;
}

// Two floats rounded to bf16 by one cvt.rn.bf16x2.f32 (each element RN, as a scalar cast) and
// widened back; `packed` keeps the bf16 pair (lo in the low half).
__device__ __forceinline__ void bf16_round2(float& lo, float& hi, uint32_t& packed) {
    packed = pack_bf16(lo, hi);
    lo = __uint_as_float(packed << 16);
    hi = __uint_as_float(packed & 0xFFFF0000u);
}

// f[e] = RN(f[e] * inv[e]) for eight consecutive columns (inv 16-byte aligned).
__device__ __forceinline__ void scale8(float (&f)[8], const float* inv) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(inv));
    const float4 b = __ldg(reinterpret_cast<const float4*>(inv) + 1);
    const float iv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = __fmul_rn(f[e], iv[e]);
}

// Phase 2 of the fused SwiGLU kernel: each warp requantises whole rows of h [M, N/2] with
// the row scale from the absmax that phase 1 accumulated (row_amax). Eight 8-element vectors
// per lane are loaded before any is used, so a warp keeps 8 KB of its row in flight: phase 2
// runs on the GEMM's ten warps per SM, and the bytes in flight set its bandwidth.
template <int MODE>
__device__ __forceinline__ void swiglu_requant_rows(const GemmArgs& args, int warp, int lane) {
    const int I = args.N / 2;
    const int warps_total = gridDim.x * (blockDim.x >> 5);
    constexpr int U = 8;
    for (int row = blockIdx.x * (blockDim.x >> 5) + warp; row < args.M; row += warps_total) {
        const unsigned bits = __ldcg(args.row_amax + row);
        const float scale = __fdiv_rn(fmaxf(__uint_as_float(bits), 1e-8f), 127.0f);
        const float rscale = __frcp_rn(scale);
        const __nv_bfloat16* hrow = args.h + static_cast<long>(row) * args.ldh;
        int8_t* qrow = args.q_out + static_cast<long>(row) * args.ldq;
        for (int c0 = lane * 8; c0 < I; c0 += 32 * 8 * U) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + u * 32 * 8;
                v[u] = c < I ? __ldcg(reinterpret_cast<const uint4*>(hrow + c)) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + u * 32 * 8;
                if (c >= I) break;
                float f[8];
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    f[2 * j] = __uint_as_float(w[j] << 16);
                    f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
                }
                if (args.inv_h != nullptr) scale8(f, args.inv_h + c);
                *reinterpret_cast<uint2*>(qrow + c) = quant8<MODE>(f, scale, rscale);
            }
        }
        if (lane == 0) args.s_out[row] = scale;
    }
}

template <int BN, int EPI, typename OutT, int EW = 4>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               const __grid_constant__ CUtensorMap tmap_c, const GemmArgs args) {
    using S = GemmShape<BN, EW>;
    constexpr int STAGES = S::STAGES;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment: the 128-byte swizzle pattern is a function of address bits [4,10).
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* smem_a = smem;                                   // STAGES x A_BYTES
    uint8_t* smem_b = smem + STAGES * S::A_BYTES;             // STAGES x B_BYTES
    uint8_t* smem_epi = smem_b + STAGES * S::B_BYTES;         // 4 warps x 2 boxes
    float* smem_cols = reinterpret_cast<float*>(smem_epi + S::EPI_BYTES);   // BN column scales
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + S::EPI_BYTES + S::COL_BYTES);
    uint64_t* full_bar = bars;                                // [STAGES]  TMA -> MMA
    uint64_t* empty_bar = bars + STAGES;                      // [STAGES]  MMA -> TMA
    uint64_t* tfull_bar = bars + 2 * STAGES;                  // [2]       MMA -> epilogue
    uint64_t* tempty_bar = bars + 2 * STAGES + 2;             // [2]       epilogue -> MMA
    uint64_t* drain_bar = bars + 2 * STAGES + 4;              // [1]       teardown
    uint64_t* cols_full = bars + 2 * STAGES + 5;              // [1]       epilogue: tile's scales stored
    uint64_t* cols_free = bars + 2 * STAGES + 6;              // [1]       epilogue: tile's scales read
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 7);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int M = args.M, N = args.N, K = args.K;
    const int num_m = (M + S::BM - 1) / S::BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + S::BK - 1) / S::BK;
    if constexpr (S::ACC_BUFS == 1) {
        // one accumulator buffer: every CTA may own one tile at most (the host sizes the grid)
        if (static_cast<int>(gridDim.x) < num_tiles) {
            if (threadIdx.x == 0) atomicExch(&g_dev_error, MICA_DEV_BAD_LAUNCH);
            return;
        }
    }

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
        mbar_init(cols_full, EW);
        mbar_init(cols_free, EW);
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
            uint32_t it = 0;  // k-blocks issued so far (stage = it % STAGES)
            bool ok = true;
            const uint64_t pol_b = policy_evict_last();   // weights: re-read by every M block
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
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
                    mbar_arrive_expect_tx(&full_bar[st], S::STAGE_BYTES);
                    tma_load_2d(smem_a + st * S::A_BYTES, &tmap_a, &full_bar[st], kb * S::BK, m0);
#pragma unroll
                    for (int hf = 0; hf < S::HALVES; ++hf)
                        tma_load_2d_hint(smem_b + st * S::B_BYTES + hf * S::MMA_N * S::BK, &tmap_b, &full_bar[st],
                                         kb * S::BK, n0 + hf * S::MMA_N, pol_b);
                }
            }
            // Drain: the last loads of each stage must land before this CTA's smem goes away.
            const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
            for (uint32_t j = first; j < it; ++j) {
                mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1u, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------- MMA issuer ---------------------------------
        // One lane runs the whole loop: per stage a wait on its full barrier, the k-step MMAs
        // and a commit that frees the stage. The TMA bytes' completion on the barrier orders the
        // shared-memory tiles before the MMAs; a tcgen05 fence is needed only after taking an
        // accumulator back from the epilogue warps.
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(S::BM, S::MMA_N);
            // descriptors of stage 0; a stage / k-step is a plain offset of the address field
            const uint64_t a_desc0 = smem_desc_k128(smem_u32(smem_a));
            const uint64_t b_desc0 = smem_desc_k128(smem_u32(smem_b));
            uint32_t it = 0;
            int local = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
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
#pragma unroll
                        for (int hf = 0; hf < S::HALVES; ++hf)
                            mma_i8(d_tmem + hf * S::MMA_N, a_st + static_cast<uint64_t>((k * S::UMMA_K) >> 4),
                                   b_st + static_cast<uint64_t>((hf * S::MMA_N * S::BK + k * S::UMMA_K) >> 4), idesc,
                                   (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty_bar[st]);          // frees the stage when these MMAs finish
                    if (kb == num_kb - 1) mma_commit(&tfull_bar[acc]);  // accumulator complete
                }
            }
            // Drain: every MMA issued must finish before tensor memory is released.
            mma_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, MICA_DEV_TIMEOUT_DRAIN);
        }
        __syncwarp();
    } else {
        // ------------------------------- epilogue -----------------------------------
        const int q4 = warp & 3;                  // TMEM lane quarter this warp may access
        const int row_local = q4 * 32 + lane;
        const int ew = warp - 2;                  // epilogue warp 0..EW-1
        const int part = ew >> 2;                 // with 8 warps, two share a lane quarter
        constexpr int PARTS = EW / 4;
        uint8_t* my_boxes = smem_epi + ew * S::BOX_BUFS * S::BOX_BYTES;
        int box_count = 0;
        int local = 0;
        // The dequantised output is written once: evict it before the weights (evict_last).
        const uint64_t pol_c = policy_evict_first();
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            int mt, nt;
            tile_origin(tile, num_m, num_n, args.panel, mt, nt);
            const int m0 = mt * S::BM;
            const int n0 = nt * BN;
            const int acc = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            // The tile's row scale and column vectors do not depend on the accumulator: start their
            // loads before waiting for it, so a cold L2 (first tile, small grids) costs no DRAM round
            // trips after the main loop. One 32-column line per lane.
            const int grow = m0 + row_local;
            const float sa_v = grow < M ? __ldg(args.sa + grow) : 0.f;
            if (lane * 32 < BN && n0 + lane * 32 < N) {
                prefetch_l1(args.sb + n0 + lane * 32);
                if (args.bias != nullptr) prefetch_l1(args.bias + n0 + lane * 32);
            }
            if constexpr (EPI == EPI_SWIGLU) {
                if (args.inv_h != nullptr && lane * 32 < BN / 2 && (n0 / 2) + lane * 32 < N / 2)
                    prefetch_l1(args.inv_h + n0 / 2 + lane * 32);
            }
            // The tile's BN column scales go to shared memory while the accumulator is computed
            // (cols_free: every epilogue warp is done with the previous tile's; cols_full: all of
            // this tile's are stored; one arrival per warp, bounded waits). Measured on B200, a chunk that loaded its scales at
            // its own start waited ~450 cycles for L2, which on one-tile-per-CTA grids left ~1.4 us
            // of epilogue exposed per warp; the values do not stay in the small L1 beside 227 KB of
            // shared memory. SwiGLU also loads the first chunk's per-lane bias and smoothing values
            // (when present), one chunk ahead.
            SwigluCols sw_cur;
            {
                bool cw = true;
                if (lane == 0 && local > 0)
                    cw = mbar_wait(cols_free, (local - 1) & 1, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
                if (!__shfl_sync(0xffffffffu, cw, 0)) break;
                for (int c = ew * 32 + lane; c < BN; c += EW * 32)
                    smem_cols[c] = n0 + c < N ? __ldg(args.sb + n0 + c) : 0.f;
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(cols_full);
                    cw = mbar_wait(cols_full, local & 1, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
                }
                if (!__shfl_sync(0xffffffffu, cw, 0)) break;
                __syncwarp();                  // orders the lanes' reads after lane 0's acquire
                if constexpr (EPI == EPI_SWIGLU) sw_cur = load_swiglu_cols(args, n0 + part * 128, N);
            }
            bool w = true;
            if (lane == 0) w = mbar_wait(&tfull_bar[acc], acc_ph, abort_flag, MICA_DEV_TIMEOUT_EPILOGUE);
            if (!__shfl_sync(0xffffffffu, w, 0)) break;
            tc_fence_after();

            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q4 * 32) << 16) + acc * S::ACC_COLS;

            if constexpr (EPI == EPI_DEQUANT) {
                constexpr int COLS_PER_BOX = 128 / static_cast<int>(sizeof(OutT));
                constexpr int CHUNKS_PER_BOX = COLS_PER_BOX / 32;
                constexpr int BOXES = BN / COLS_PER_BOX;
#pragma unroll 1
                for (int bx = part; bx < BOXES; bx += PARTS, ++box_count) {
                    uint8_t* box = my_boxes + (box_count % S::BOX_BUFS) * S::BOX_BYTES;
                    // the store that last used this box must have finished reading it
                    if (lane == 0) {
                        if constexpr (S::BOX_BUFS == 2) tma_store_wait_read<1>();
                        else tma_store_wait_read<0>();
                    }
                    __syncwarp();
                    const uint32_t box_row = smem_u32(box) + lane * 128;
#pragma unroll
                    for (int cc = 0; cc < CHUNKS_PER_BOX; ++cc) {
                        const int col0 = bx * COLS_PER_BOX + cc * 32;
                        float4 sb4[8];             // uniform shared loads: one broadcast each
#pragma unroll
                        for (int v = 0; v < 8; ++v) sb4[v] = reinterpret_cast<const float4*>(smem_cols + col0)[v];
                        dequant_chunk<OutT>(args, t_row + col0, n0 + col0, N, sa_v, sb4, box_row, cc);
                    }
                    if (bx + PARTS >= BOXES) {
                        // this warp's last read of the accumulator: hand it back to the MMA warp
                        tc_fence_before();
                        mbar_arrive(&tempty_bar[acc]);
                        if (lane == 0) mbar_arrive(cols_free);   // and its last read of the scales
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int x = n0 + bx * COLS_PER_BOX, y = m0 + q4 * 32;
                        if (x < N && y < M) tma_store_2d_hint(&tmap_c, box, x, y, pol_c);   // edge boxes hold nothing
                        tma_store_commit();
                    }
                }
            } else {
                // SwiGLU: each 32-column chunk holds 16 gate and 16 up columns of the same
                // 16 outputs; h = bf16(bf16(silu(g)) * u), running max |h| per row.
                constexpr int H_PER_BOX = 64;                 // bf16 h columns per 128-byte box row
                constexpr int CHUNKS_PER_BOX = 4;             // 4 x 16 h columns
                constexpr int BOXES = BN / 128;
                float amax = 0.f;
#pragma unroll 1
                for (int bx = part; bx < BOXES; bx += PARTS, ++box_count) {
                    uint8_t* box = my_boxes + (box_count % S::BOX_BUFS) * S::BOX_BYTES;
                    if (lane == 0) {
                        if constexpr (S::BOX_BUFS == 2) tma_store_wait_read<1>();
                        else tma_store_wait_read<0>();
                    }
                    __syncwarp();
                    const uint32_t box_row = smem_u32(box) + lane * 128;
#pragma unroll
                    for (int cc = 0; cc < CHUNKS_PER_BOX; ++cc) {
                        const int col0 = bx * 128 + cc * 32;
                        const float bias_l = sw_cur.bias;
                        const float inv_l = sw_cur.inv;   // down_proj's smoothing of h column (n0 + col0) / 2 + (lane & 15)
                        // this warp's next chunk's values, in flight while this chunk is processed
                        const int ncol = cc + 1 < CHUNKS_PER_BOX ? col0 + 32 : (bx + PARTS) * 128;
                        if (ncol < BN) sw_cur = load_swiglu_cols(args, n0 + ncol, N);
                        // the chunk's 16 gate and 16 up scales: uniform shared loads, one broadcast each
                        float4 sb4[8];
#pragma unroll
                        for (int v = 0; v < 8; ++v) sb4[v] = reinterpret_cast<const float4*>(smem_cols + col0)[v];
                        const float* sbc = reinterpret_cast<const float*>(sb4);
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(t_row + col0, r);
                        tmem_ld_wait();
                        uint32_t p[8];
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            // outputs j and j + 1: g, u dequantised, each rounded to bf16 (the two
                            // QLinears' outputs), silu(g) rounded, h = bf16(silu(g) * u); the
                            // roundings run on pairs
                            float g0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), sa_v), sbc[j]);
                            float g1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j + 1])), sa_v), sbc[j + 1]);
                            float u0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[16 + j])), sa_v), sbc[16 + j]);
                            float u1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[17 + j])), sa_v), sbc[17 + j]);
                            if (args.bias != nullptr) {
                                g0 = __fadd_rn(g0, __shfl_sync(0xffffffffu, bias_l, j));
                                g1 = __fadd_rn(g1, __shfl_sync(0xffffffffu, bias_l, j + 1));
                                u0 = __fadd_rn(u0, __shfl_sync(0xffffffffu, bias_l, 16 + j));
                                u1 = __fadd_rn(u1, __shfl_sync(0xffffffffu, bias_l, 17 + j));
                            }
                            uint32_t pk;
                            bf16_round2(g0, g1, pk);
                            bf16_round2(u0, u1, pk);
                            // silu in fp32 with branch-free intrinsics (few-ulp fp32 error, below
                            // the bf16 rounding that follows), so the 16 independent chains of a
                            // chunk interleave instead of serialising on slow paths
                            float a0 = __fdividef(g0, 1.0f + __expf(-g0));
                            float a1 = __fdividef(g1, 1.0f + __expf(-g1));
                            bf16_round2(a0, a1, pk);
                            float h0 = __fmul_rn(a0, u0), h1 = __fmul_rn(a1, u1);
                            bf16_round2(h0, h1, p[j / 2]);
                            // the requant's input is RN(h * inv) (act_quant's xf * inv_smooth)
                            if (args.inv_h != nullptr) {
                                h0 = __fmul_rn(h0, __shfl_sync(0xffffffffu, inv_l, j));
                                h1 = __fmul_rn(h1, __shfl_sync(0xffffffffu, inv_l, j + 1));
                            }
                            amax = fmaxf(fmaxf(amax, fabsf(h0)), fabsf(h1));
                        }
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            const int chunk = cc * 2 + c;
                            st_shared_v4(box_row + ((chunk ^ (lane & 7)) << 4), p[4 * c], p[4 * c + 1], p[4 * c + 2],
                                         p[4 * c + 3]);
                        }
                    }
                    if (bx + PARTS >= BOXES) {
                        tc_fence_before();
                        mbar_arrive(&tempty_bar[acc]);
                        if (lane == 0) mbar_arrive(cols_free);   // and its last read of the scales
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int x = n0 / 2 + bx * H_PER_BOX, y = m0 + q4 * 32;
                        if (x < N / 2 && y < M) tma_store_2d(&tmap_c, box, x, y);
                        tma_store_commit();
                    }
                }
                if (part >= BOXES) {
                    // no box of this tile for this warp (BN = 128: one box, two warps per lane
                    // quarter): it reads neither the accumulator nor the scales, and hands both back
                    mbar_arrive(&tempty_bar[acc]);
                    if (lane == 0) mbar_arrive(cols_free);
                }
                if (grow < M) atomicMax(args.row_amax + grow, __float_as_uint(amax));
            }
        }
        // all stores must be complete (not only read) before the grid-wide phase or exit
        if (lane == 0) tma_store_wait_all<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_free(tmem_base, S::TMEM_COLS);
    }

    if constexpr (EPI == EPI_SWIGLU) {
        // ---- phase 2: per-token requantisation of h once every row max is final ----
        // Grid barrier (all CTAs are co-resident: cooperative launch, one CTA per SM).
        if (threadIdx.x == 0) {
            fence_proxy_async_global();
            __threadfence();
            atomicAdd(args.grid_sync, 1u);
            const unsigned target = gridDim.x;
            const unsigned long long t0 = global_ns();
            for (uint32_t it = 0;; ++it) {
                unsigned v;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(args.grid_sync) : "memory");
                if (v >= target) break;
                if ((it & 15u) == 15u && global_ns() - t0 > kWaitLimitNs) {
                    *abort_flag = 1u;
                    atomicExch(&g_dev_error, MICA_DEV_TIMEOUT_GRID);
                    break;
                }
                __nanosleep(64);
            }
            __threadfence();
        }
        __syncthreads();
        if (*abort_flag) return;
        if (args.round_mode == MICA_ROUND_HALF_EVEN) swiglu_requant_rows<MICA_ROUND_HALF_EVEN>(args, warp, lane);
        else swiglu_requant_rows<MICA_ROUND_HALF_AWAY>(args, warp, lane);
    }
}

}  // namespace mica
