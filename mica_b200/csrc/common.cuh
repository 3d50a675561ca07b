// common.cuh -- sm_100a building blocks shared by the mica_w8a8 kernels:
// mbarriers with bounded waits, TMA (cp.async.bulk.tensor) loads/stores, tcgen05 MMA,
// tensor-memory allocation and loads, and the host-side launch/status helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/mica_w8a8.h"

namespace mica {

// ------------------------------------------------------------------------------------
// Device error word. One per device (module-scope __device__ variable); kernels write
// it only when a bounded wait gives up. mica_device_error() reads and clears it.
// The library is one translation unit (mica_w8a8.cu), so the definition lives here.
// ------------------------------------------------------------------------------------
__device__ int g_dev_error = 0;

// A wait that has not finished after this many nanoseconds is treated as a failure:
// the waiting kernel records an error code and unwinds instead of spinning forever.
// The longest legitimate wait (one 128-row tile of a K=32768 GEMM) is a few hundred us.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() {
    uint32_t l;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
    return l;
}

// ---- mbarrier ----------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, but a thread whose phase is not complete sleeps in hardware until the
// phase completes or about kSleepHintNs pass. A polling loop of non-blocking tests keeps the
// shared-memory pipe busy with barrier probes; on B200 that slowed a CTA pair's stage
// hand-off (MMA commit -> empty barrier -> producer -> full barrier -> MMA) by a fifth, where
// the sleeping form wakes on the phase change and keeps the tensor pipe fed.
constexpr uint32_t kSleepHintNs = 1000000;   // 1 ms; a completed phase ends the sleep at once
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSleepHintNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on phase `parity` of `bar`. Returns false when the CTA-wide abort flag is
// raised or the wait outlives limit_ns (then it raises the flag and records `code`).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                          int code, unsigned long long limit_ns = kWaitLimitNs) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > limit_ns) {
            *abort_flag = 1u;
            atomicExch(&g_dev_error, code);
            return false;
        }
    }
}

// ---- TMA ---------------------------------------------------------------------------
// Starts fetching the 128-byte line holding p into L1 (and L2); nothing waits for it.
__device__ __forceinline__ void prefetch_l1(const void* p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load into this CTA's shared memory; completes `bytes` on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// Same with an L2 cache-policy hint (createpolicy value).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)),
        "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 2-D tiled store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
// Same with an L2 cache-policy hint (createpolicy value).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, const void* src, int x, int y,
                                                  uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- tcgen05 ------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole-warp tensor-memory allocation; writes the base address to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart): start address >> 4 in
// bits [0,14), leading offset unused for this layout, stride offset 1024 >> 4 in bits
// [32,46), descriptor version 1 at bit 46, swizzle mode 2 (128B) in bits [61,64).
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

// Instruction descriptor for tcgen05.mma kind::i8: signed int8 A and B, both K-major,
// int32 accumulator (format 2 at bits [4,6)), N >> 3 at bits [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one 128 x N x 32 int8 step issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i receives lane (base + i), columns
// [col, col + 32) of the address `taddr` = (lane << 16) | col.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 32 columns of 32-bit words from registers into tensor memory (this warp's lane
// quarter); tmem_st_wait() orders them before later tensor-memory reads.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// ---- packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE round-to-nearest operations per
// instruction, no contraction, so each lane equals the scalar __fmul_rn / __fadd_rn) --------
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long v;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
    return v;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Ties 32 registers written by tcgen05.ld to this point of the program, so no use of them is
// scheduled above the tcgen05.wait::ld that precedes it (emits no instruction).
__device__ __forceinline__ void reg_pin32(uint32_t (&r)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

// ---- 2-SM (CTA pair) forms ------------------------------------------------------------
// A cluster of two CTAs on a pair of SMs shares one 256-row MMA: each CTA holds 128 rows of
// A and half of B's rows in its own shared memory at identical offsets; the even CTA issues
// the MMA and each CTA's tensor memory receives its 128 rows of the accumulator.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the variable at `local_addr` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier that may live in the peer CTA (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into the shared memory of either CTA of the pair (`dst_cluster_addr`, a
// shared::cluster address) whose completion bytes are counted on the mbarrier at
// `bar_cluster_addr`, which may also live in either CTA (the .cta_group::2 form).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst_cluster_addr, const CUtensorMap* map,
                                                 uint32_t bar_cluster_addr, int x, int y, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(dst_cluster_addr), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster_addr),
        "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at `bar_cluster_addr` (either CTA of the pair) when every
// pair MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar_cluster_addr)
                 : "memory");
}

// Named barrier among `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- division by a per-row scale -----------------------------------------------------
// RN(x / s) given r = RN(1 / s) (one __frcp_rn per row). Markstein's theorem: when r is the
// correctly rounded reciprocal, q0 = RN(x * r) is within one ulp of x / s, the residual
// x - q0 * s is exact in one FMA, and RN(q0 + residual * r) equals RN(x / s) -- for every
// quotient in the normal range. Smaller quotients (|x / s| < 2^-126) quantise to 0 under
// either rounding mode, so the codes are those of the IEEE division. Three instructions,
// no slow-path branch, unlike a full division per element.
__device__ __forceinline__ float div_by_scale(float x, float s, float r) {
    const float q0 = __fmul_rn(x, r);
    const float e = __fmaf_rn(-q0, s, x);
    return __fmaf_rn(e, r, q0);
}

// ---- rounding shared by the quantisers ---------------------------------------------
// v = x / scale in IEEE fp32. HALF_AWAY follows the reference GPU kernel literally:
// add +-0.5 in fp32 (so the sum itself is rounded) and truncate toward zero.
// copysign(0.5, v) equals the reference's (v >= 0 ? +0.5 : -0.5) for every v that matters:
// only -0.0 differs, and -0.0 - 0.5 = -0.5 truncates to the same 0.
__device__ __forceinline__ int quant_round(float v, int round_mode) {
    const int r = round_mode == MICA_ROUND_HALF_EVEN ? __float2int_rn(v)
                                                      : __float2int_rz(__fadd_rn(v, copysignf(0.5f, v)));
    return min(max(r, -127), 127);
}

// The same rounding without the +-127 clamp, for quantisers whose scale comes from the
// absmax of the very values they quantise. With s = RN(max(amax, 1e-8) / 127) and
// |x| <= amax, x / s <= 127 / (1 - 2^-24), so |RN(x / s)| <= 127 + 2^-17 (the fp32 spacing
// at 127) and both modes give |q| <= 127: the reference's clamp never acts on finite input.
template <int MODE>
__device__ __forceinline__ int quant_code(float v) {
    if constexpr (MODE == MICA_ROUND_HALF_EVEN) return __float2int_rn(v);
    else return __float2int_rz(__fadd_rn(v, copysignf(0.5f, v)));
}
// Four codes, each within int8 range, packed little-endian (q0 in the low byte) by two
// saturating pack instructions: cvt.pack.sat d, a, b, c puts sat(b) in bits 0-7, sat(a) in
// bits 8-15 and the low half of c in bits 16-31.
__device__ __forceinline__ uint32_t pack4_s8(int q0, int q1, int q2, int q3) {
    uint32_t hi, w;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(q3), "r"(q2), "r"(0));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(q1), "r"(q0), "r"(hi));
    return w;
}
// Eight values quantised with RN(x / s) (div_by_scale) into two packed words.
template <int MODE>
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float scale, float rscale) {
    int q[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = quant_code<MODE>(div_by_scale(v[e], scale, rscale));
    return make_uint2(pack4_s8(q[0], q[1], q[2], q[3]), pack4_s8(q[4], q[5], q[6], q[7]));
}

}  // namespace mica

// ---- host helpers --------------------------------------------------------------------
namespace mica_host {

// Records the message of a failed CUDA call for mica_last_cuda_error().
void set_cuda_error(cudaError_t e);
int check_device(int* sm_count);                  // MICA_OK when the current device is sm_100
bool aligned16(const void* p);
// Encodes a 2-D row-major tensor map: dims {inner, outer}, row pitch in bytes, box
// {box_inner, box_outer}, 128-byte swizzle, zero fill out of bounds.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

}  // namespace mica_host
