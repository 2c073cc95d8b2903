// Batched scaled-scores softmax: Y[b] = softmax_rows(scale * Q[b] * K[b]^T).
//
// The reference has no fused operator: its composition is Call(MatMul) ->
// scale map -> Call(Softmax) (runtime/src/execution/kernel_buffers.cpp:
// 1001-1085, :342-402, :290-340), evaluated in f64 with K^T materialised.
// Q is f16 [batch, m, d] row-major. K comes in either of two layouts and
// neither is ever transposed in memory:
//   * K  [batch, s, d] (the direct entry): the K-major operand the MMA takes;
//   * Kt [batch, d, s] (the module route): the reference's MatMul B operand,
//     [K, N] row-major (kernel_buffers.cpp:1030-1036), which the MMA reads as
//     an MN-major operand from the same shared-memory ring.
//
// Fused kernel (s % 128 == 0, d in {64, 128}); one CTA per SM, persistent
// over units = (batch, 128-row band). The output write (4 B per score) is the
// roofline, so every score is written exactly once and nothing else is. Each
// unit needs two passes over its scores (row statistics, then the normalised
// write); running them back to back would leave HBM idle during the first.
// Instead the CTA overlaps pass 1 of unit i with pass 2 of unit i-1. Each CTA
// takes runs of consecutive bands of one batch, so units i-1 and i mostly
// share a batch and then one K load feeds both passes' MMAs.
//   warp 0       TMA producer: Q bands into three slots, K in [128 x 64] boxes
//                through a 5-stage ring, in the MMA's consumption order;
//   warp 1       MMA issuer: per 128-column chunk, tcgen05.mma M128 N128 K16
//                (both operands K-major) for pass 2 of unit i-1 and pass 1 of
//                unit i, into four 128-column TMEM accumulators (two per pass);
//   warps 2-5    group A (pass 1), one warp per TMEM lane quarter: online row
//                max / sum of exp2(scale*log2e*s), handed to group B through a
//                double-buffered statistics slot;
//   warps 6-17   group B (pass 2), three warps per lane quarter sharing each
//                chunk's four 32-row groups round-robin: recompute,
//                exp2(s*c - (m + log2 l)). Pass 2's MMA swaps its operands
//                (K chunk as A, Q band as B), so its accumulator holds the
//                scores transposed: TMEM lane = key, column = score row. A
//                warp's 32 lanes then hold 32 consecutive keys of one row, and
//                each store instruction writes a full 128-byte row segment
//                straight from registers, with no shared-memory transpose.
// The row length is a template constant for s = 1024, 2048 and 4096 (a
// runtime value otherwise), so pass-2 stores use immediate row offsets.
// Every mbarrier wait is bounded (2 s); on a timeout the CTA raises the
// device status word, drains its copies, frees TMEM and returns.
// Other shapes use the two-step form (tcgen05 GEMM with the scale folded into
// its epilogue, then the row softmax in place).
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "tc_common.cuh"

namespace mlkb {
int launchGemmTc(const void* a, const void* b, float* c, int64_t batch, int64_t m, int64_t n,
                 int64_t k, bool b_kmajor, int accumulate, float scale, cudaStream_t s);
int makeTmapF16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows,
                int box_cols);

namespace {

constexpr int kRows = 128;   // score rows per unit (M of the MMA)
constexpr int kChunk = 128;  // score columns per accumulator (N of the MMA)
constexpr int kKStages = 5;  // K ring depth, [128 x 64] f16 boxes
constexpr int kRun = 4;      // longest run of consecutive bands of one batch per CTA
constexpr int kQSlots = 3;   // Q bands resident: units i-1, i and the prefetched i+1
constexpr uint32_t kKBox = kChunk * 64 * 2;  // 16 KB
constexpr uint32_t kQBox = kRows * 64 * 2;   // 16 KB (one d-half)
constexpr int kAWarps = 4;                   // pass 1: one warp per lane quarter
constexpr int kBWarps = 12;                  // pass 2: three warps per lane quarter
constexpr int kThreads = 64 + (kAWarps + kBWarps) * 32;  // 576
constexpr uint64_t kLimitNs = 2000000000ull;

struct QkSmem {
    uint8_t k[kKStages][kKBox];              // 80 KB
    uint8_t q[kQSlots][2][kQBox];            // 96 KB
    alignas(16) float nmi[2][kRows];         // [slot][row] = -(max + log2 sum)
    uint64_t kfull[kKStages], kempty[kKStages];
    uint64_t qfull[kQSlots], qempty[kQSlots];
    uint64_t afull[2], aempty[2], bfull[2], bempty[2];
    uint64_t sfull[2], sempty[2];
    uint32_t tmem_base;
    int abort;
};

constexpr size_t kSmemBytes = sizeof(QkSmem);

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max of three (NaN-avoiding like fmaxf: a NaN operand never wins).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Lane-0 arrive after the whole warp is done with the guarded resource.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar);
}

// kKt: K arrives as Kt [batch, d, s] (MN-major operand); else K [batch, s, d].
// m: score rows per batch (Q rows, a multiple of 128); s: keys per batch.
template <int kS, bool kKt>
__global__ void __launch_bounds__(kThreads, 1)
qk_softmax_tcgen05(const __grid_constant__ CUtensorMap tma_q,
                   const __grid_constant__ CUtensorMap tma_k, float* __restrict__ y, int batch,
                   int m_in, int s_in, int d, int run, float c2, int* __restrict__ status) {
    // Row length (keys) and rows per batch: constants in the instances
    // specialised on square batches (m == s), run-time values otherwise.
    const int s = kS != 0 ? kS : s_in;
    const int m = kS != 0 ? kS : m_in;
    // The kernel has no static shared memory, so the dynamic window starts at
    // the 1024-byte aligned base the 128B-swizzled tiles need.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    QkSmem& sm = *reinterpret_cast<QkSmem*>(smem_raw);
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {  // uniform across the CTA
        if (threadIdx.x == 0 && status != nullptr) atomicExch(status, MLKB_ERR_INVALID);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bands = m / kRows;
    const int units = batch * bands;
    const int chunks = s / kChunk;
    const int dh = d / 64;  // d-halves (1 or 2)
    // This CTA's units: runs of `run` consecutive bands of one batch (run
    // divides bands; chosen on the host), the runs
    // dealt round-robin over the CTAs. Within a run pass 2 of unit i-1 and
    // pass 1 of unit i read the same K (one load feeds both), while the CTAs
    // together stay on a few batches at a time, so K and Q stay L2-resident.
    const int runs = units / run;
    const int nruns = runs > static_cast<int>(blockIdx.x)
                          ? (runs - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                          : 0;
    const int n = nruns * run;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kKStages; ++i) {
            tc::mbar_init(&sm.kfull[i], 1);
            tc::mbar_init(&sm.kempty[i], 1);
        }
        for (int i = 0; i < kQSlots; ++i) {
            tc::mbar_init(&sm.qfull[i], 1);
            tc::mbar_init(&sm.qempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&sm.afull[i], 1);
            tc::mbar_init(&sm.aempty[i], kAWarps);
            tc::mbar_init(&sm.bfull[i], 1);
            tc::mbar_init(&sm.bempty[i], kBWarps);
            tc::mbar_init(&sm.sfull[i], kAWarps);
            tc::mbar_init(&sm.sempty[i], kBWarps);
        }
        sm.abort = 0;
        tc::fence_barrier_init();
        tc::fence_proxy_async();
    }
    if (warp == 0) tc::tmem_alloc(&sm.tmem_base, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    volatile int* abort = &sm.abort;
    auto unit_of = [&](int i) {
        return (static_cast<int>(blockIdx.x) + (i / run) * static_cast<int>(gridDim.x)) * run +
               i % run;
    };
    // Step `step` (1 <= step < n) runs both passes on the same K chunks when
    // units step-1 and step belong to the same batch: one load feeds both MMAs.
    auto shares_k = [&](int step) {
        return step > 0 && step < n && unit_of(step - 1) / bands == unit_of(step) / bands;
    };

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        tc::prefetch_tmap(&tma_q);
        tc::prefetch_tmap(&tma_k);
        uint32_t kit = 0;
        auto load_q = [&](int i) -> bool {
            const int slot = i % kQSlots;
            if (i >= kQSlots &&
                !tc::mbar_wait(&sm.qempty[slot], ((i / kQSlots) - 1) & 1, abort, kLimitNs)) {
                return false;
            }
            const int u = unit_of(i);
            const int b = u / bands, band = u - b * bands;
            tc::mbar_arrive_expect_tx(&sm.qfull[slot], kQBox * dh);
            for (int h = 0; h < dh; ++h) {
                tc::tma_load_2d(sm.q[slot][h], &tma_q, &sm.qfull[slot], h * 64,
                                b * m + band * kRows);
            }
            return true;
        };
        auto load_k = [&](int i, int c) -> bool {
            const int b = unit_of(i) / bands;
            for (int h = 0; h < dh; ++h, ++kit) {
                const int st = static_cast<int>(kit % kKStages);
                if (!tc::mbar_wait(&sm.kempty[st], ((kit / kKStages) & 1u) ^ 1u, abort,
                                   kLimitNs)) {
                    return false;
                }
                tc::mbar_arrive_expect_tx(&sm.kfull[st], kKBox);
                if constexpr (kKt) {
                    // d rows h*64.. of Kt, keys c*128..: two [64 x 64] boxes
                    // side by side along the keys (MN-major, 128B swizzle)
                    tc::tma_load_2d(sm.k[st], &tma_k, &sm.kfull[st], c * kChunk, b * d + h * 64);
                    tc::tma_load_2d(sm.k[st] + kKBox / 2, &tma_k, &sm.kfull[st],
                                    c * kChunk + 64, b * d + h * 64);
                } else {
                    tc::tma_load_2d(sm.k[st], &tma_k, &sm.kfull[st], h * 64, b * s + c * kChunk);
                }
            }
            return true;
        };
        bool ok = true;
        for (int i = 0; i < n && i < 2 && ok; ++i) ok = load_q(i);
        // Q of unit step+1 reuses the slot of unit step-2, free once the MMA has
        // finished step-1; a chunk into this step that is the case, and the
        // band still lands a whole step before it is needed.
        const int qload_at = chunks > 1 ? 1 : 0;
        for (int step = 0; step <= n && ok; ++step) {
            for (int c = 0; c < chunks && ok; ++c) {
                if (shares_k(step)) {
                    ok = load_k(step, c);  // both passes
                } else {
                    if (step > 0) ok = load_k(step - 1, c);   // pass 2 of unit step-1
                    if (ok && step < n) ok = load_k(step, c);  // pass 1 of unit step
                }
                if (ok && c == qload_at && step + 1 < n && step + 1 >= 2) ok = load_q(step + 1);
            }
        }
        for (uint32_t j = kit > kKStages ? kit - kKStages : 0; j < kit; ++j) {
            int never = 0;
            (void)tc::mbar_wait(&sm.kfull[j % kKStages], (j / kKStages) & 1u, &never, kLimitNs);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        // Pass 1: Q (A, K-major) x K chunk (B); pass 2 swaps them: K chunk (A)
        // x Q (B). With Kt the K chunk is the MN-major operand of both.
        constexpr uint32_t kIdescP1 = tc::idesc_f16_f32(kRows, kChunk, 0, kKt ? 1 : 0);
        constexpr uint32_t kIdescP2 = tc::idesc_f16_f32(kRows, kChunk, kKt ? 1 : 0, 0);
        // K16 step kk of a K stage: K-major steps 32 B along the swizzled
        // row; MN-major steps 16 d-rows (2 KB), the second 64-key box 8 KB on.
        auto kdesc = [](uint32_t k0, int kk) -> uint64_t {
            return kKt ? tc::smem_desc_sw128(k0 + kk * 2048, kKBox / 2, 1024)
                       : tc::smem_desc_sw128(k0 + kk * 32, 16, 1024);
        };
        uint32_t kit = 0, ait = 0, bit = 0;
        // One accumulator chunk: Q slot x K chunk -> TMEM columns `dst`; with
        // `keys_as_rows` the operands swap and the chunk lands transposed.
        auto mma_chunk = [&](int qslot, uint32_t dst, bool keys_as_rows) -> bool {
            for (int h = 0; h < dh; ++h, ++kit) {
                const int st = static_cast<int>(kit % kKStages);
                if (!tc::mbar_wait(&sm.kfull[st], (kit / kKStages) & 1u, abort, kLimitNs)) {
                    return false;
                }
                tc::tc_fence_after();
                const uint32_t q0 = tc::smem_u32(sm.q[qslot][h]);
                const uint32_t k0 = tc::smem_u32(sm.k[st]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t dq = tc::smem_desc_sw128(q0 + kk * 32, 16, 1024);
                    const uint64_t dk = kdesc(k0, kk);
                    tc::mma_f16(dst, keys_as_rows ? dk : dq, keys_as_rows ? dq : dk,
                                keys_as_rows ? kIdescP2 : kIdescP1, (h > 0 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit(&sm.kempty[st]);
            }
            return true;
        };
        // Both passes of a chunk from one K stage: pass 2 of unit step-1 into
        // `db` (Q slot qb, transposed) and pass 1 of unit step into `da` (Q
        // slot qa).
        auto mma_chunk2 = [&](int qb, uint32_t db, int qa, uint32_t da) -> bool {
            for (int h = 0; h < dh; ++h, ++kit) {
                const int st = static_cast<int>(kit % kKStages);
                if (!tc::mbar_wait(&sm.kfull[st], (kit / kKStages) & 1u, abort, kLimitNs)) {
                    return false;
                }
                tc::tc_fence_after();
                const uint32_t k0 = tc::smem_u32(sm.k[st]);
                const uint32_t qb0 = tc::smem_u32(sm.q[qb][h]);
                const uint32_t qa0 = tc::smem_u32(sm.q[qa][h]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    tc::mma_f16(db, kdesc(k0, kk), tc::smem_desc_sw128(qb0 + kk * 32, 16, 1024),
                                kIdescP2, (h > 0 || kk > 0) ? 1u : 0u);
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    tc::mma_f16(da, tc::smem_desc_sw128(qa0 + kk * 32, 16, 1024), kdesc(k0, kk),
                                kIdescP1, (h > 0 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit(&sm.kempty[st]);
            }
            return true;
        };
        for (int step = 0; step <= n; ++step) {
            if (step < n &&
                !tc::mbar_wait(&sm.qfull[step % kQSlots], (step / kQSlots) & 1, abort, kLimitNs)) {
                break;
            }
            tc::tc_fence_after();
            bool ok = true;
            const bool shared = shares_k(step);
            for (int c = 0; c < chunks && ok; ++c) {
                if (shared) {  // both passes from the same K stages
                    const uint32_t accb = bit & 1u, acca = ait & 1u;
                    ok = tc::mbar_wait(&sm.bempty[accb], ((bit >> 1) & 1u) ^ 1u, abort, kLimitNs);
                    ok = ok &&
                         tc::mbar_wait(&sm.aempty[acca], ((ait >> 1) & 1u) ^ 1u, abort, kLimitNs);
                    tc::tc_fence_after();
                    ok = ok && mma_chunk2((step - 1) % kQSlots, tmem + 256 + accb * kChunk,
                                          step % kQSlots, tmem + acca * kChunk);
                    if (ok) {
                        tc::mma_commit(&sm.bfull[accb]);
                        tc::mma_commit(&sm.afull[acca]);
                    }
                    ++bit;
                    ++ait;
                    continue;
                }
                if (step > 0) {  // pass 2 of unit step-1 -> accumulators B (256, 384)
                    const uint32_t acc = bit & 1u;
                    ok = tc::mbar_wait(&sm.bempty[acc], ((bit >> 1) & 1u) ^ 1u, abort, kLimitNs);
                    tc::tc_fence_after();
                    ok = ok && mma_chunk((step - 1) % kQSlots, tmem + 256 + acc * kChunk, true);
                    if (ok) tc::mma_commit(&sm.bfull[acc]);
                    ++bit;
                }
                if (ok && step < n) {  // pass 1 of unit step -> accumulators A (0, 128)
                    const uint32_t acc = ait & 1u;
                    ok = tc::mbar_wait(&sm.aempty[acc], ((ait >> 1) & 1u) ^ 1u, abort, kLimitNs);
                    tc::tc_fence_after();
                    ok = ok && mma_chunk(step % kQSlots, tmem + acc * kChunk, false);
                    if (ok) tc::mma_commit(&sm.afull[acc]);
                    ++ait;
                }
            }
            if (!ok) break;
            // unit step-1 has had both passes: its Q slot is free once they finish
            if (step > 0) tc::mma_commit(&sm.qempty[(step - 1) % kQSlots]);
        }
    } else if (warp >= 2 && warp < 2 + kAWarps) {
        // ---------------- group A: pass 1 (row statistics) ----------------
        const int quarter = warp & 3;  // TMEM lanes this warp may read
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        uint32_t ait = 0;
        for (int i = 0; i < n; ++i) {
            float m = -INFINITY, l = 0.0f;
            for (int c = 0; c < chunks; ++c, ++ait) {
                const uint32_t acc = ait & 1u;
                if (!tc::mbar_wait(&sm.afull[acc], (ait >> 1) & 1u, abort, kLimitNs)) goto a_done;
                tc::tc_fence_after();
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {  // the chunk's two 64-column halves
                    uint32_t r[2][32];
                    const uint32_t col = lane_addr + acc * kChunk + h * 64;
                    tc::tmem_ld32(tmem + col, r[0]);
                    tc::tmem_ld32(tmem + col + 32, r[1]);
                    tc::tmem_ld_wait();
                    if (h == 1) {
                        tc::tc_fence_before();
                        warp_arrive(&sm.aempty[acc], lane);  // values are in registers now
                    }
                    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                    for (int j = 0; j < 64; j += 2) {
                        mx[(j >> 1) & 3] =
                            max3(mx[(j >> 1) & 3], __uint_as_float(r[j >> 5][j & 31]),
                                 __uint_as_float(r[j >> 5][(j & 31) + 1]));
                    }
                    const float gm = max3(mx[0], mx[1], fmaxf(mx[2], mx[3])) * c2;
                    const float mn = fmaxf(m, gm);
                    // exponent arguments and partial sums two at a time (packed f32x2)
                    float2 sum[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
                    for (int j = 0; j < 64; j += 2) {
                        const float2 t =
                            __ffma2_rn(make_float2(__uint_as_float(r[j >> 5][j & 31]),
                                                   __uint_as_float(r[j >> 5][(j & 31) + 1])),
                                       make_float2(c2, c2), make_float2(-mn, -mn));
                        sum[(j >> 1) & 1] =
                            __fadd2_rn(sum[(j >> 1) & 1], make_float2(ex2(t.x), ex2(t.y)));
                    }
                    l = l * ex2(m - mn) + ((sum[0].x + sum[0].y) + (sum[1].x + sum[1].y));
                    m = mn;
                }
            }
            // hand -(m + log2 l) of the row to group B: y = exp2(s*c2 - m) / l
            {
                const int slot = i & 1;
                if (i >= 2 &&
                    !tc::mbar_wait(&sm.sempty[slot], ((i >> 1) - 1) & 1, abort, kLimitNs)) {
                    goto a_done;
                }
                // +inf score: the reference's exp(inf - inf) poisons the row
                sm.nmi[slot][row] = (m == INFINITY) ? __int_as_float(0x7fffffff) : -(m + log2f(l));
                warp_arrive(&sm.sfull[slot], lane);
            }
        }
    a_done:;
    } else if (warp >= 2 + kAWarps) {
        // ---------------- group B: pass 2 (normalised write) ----------------
        const int ew = warp - 2 - kAWarps;
        const int quarter = warp & 3;  // TMEM lanes = the chunk's keys quarter*32 + lane
        const int sub = ew >> 2;       // 0..2: which of the quarter's three warps
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        uint32_t bit = 0;
        for (int i = 0; i < n; ++i) {
            const int u = unit_of(i);
            const int b = u / bands, band = u - b * bands;
            const int slot = i & 1;
            if (!tc::mbar_wait(&sm.sfull[slot], (i >> 1) & 1, abort, kLimitNs)) goto b_done;
            const float* const nmi = sm.nmi[slot];
            float* const yband =
                y + (static_cast<int64_t>(b) * m + band * kRows) * s + quarter * 32 + lane;
            for (int c = 0; c < chunks; ++c, ++bit) {
                const uint32_t acc = bit & 1u;
                if (!tc::mbar_wait(&sm.bfull[acc], (bit >> 1) & 1u, abort, kLimitNs)) goto b_done;
                tc::tc_fence_after();
                // The chunk's four 32-row groups, numbered 4*bit + g over the
                // whole run, are dealt round-robin to the quarter's three warps:
                // this warp takes one or two of them.
                const int g0 = (sub - static_cast<int>((4u * bit) % 3u) + 3) % 3;  // first g of ours
                const int g1 = g0 + 3;                                          // second, if < 4
                // One 32-row group: register j holds row g*32 + j at this lane's
                // key, so every store is one row's 32 consecutive keys (128 B).
                auto write_group = [&](const uint32_t (&r)[32], int g) {
                    float* const p = yband + c * kChunk + static_cast<int64_t>(g * 32) * s;
                    const float4* const nm = reinterpret_cast<const float4*>(nmi + g * 32);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 v = nm[j];  // same address in every lane
                        // exponent arguments two at a time (packed f32x2 FMA)
                        const float2 t0 = __ffma2_rn(
                            make_float2(__uint_as_float(r[4 * j + 0]), __uint_as_float(r[4 * j + 1])),
                            make_float2(c2, c2), make_float2(v.x, v.y));
                        const float2 t1 = __ffma2_rn(
                            make_float2(__uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])),
                            make_float2(c2, c2), make_float2(v.z, v.w));
                        __stcs(p + (4 * j + 0) * s, ex2(t0.x));
                        __stcs(p + (4 * j + 1) * s, ex2(t0.y));
                        __stcs(p + (4 * j + 2) * s, ex2(t1.x));
                        __stcs(p + (4 * j + 3) * s, ex2(t1.y));
                    }
                };
                const uint32_t col = lane_addr + 256 + acc * kChunk;
                uint32_t r0[32], r1[32];
                tc::tmem_ld32(tmem + col + g0 * 32, r0);
                if (g1 < 4) tc::tmem_ld32(tmem + col + g1 * 32, r1);
                tc::tmem_ld_wait(r0);
                if (g1 < 4) tc::tmem_ld_wait(r1);
                tc::tc_fence_before();
                warp_arrive(&sm.bempty[acc], lane);  // values are in registers now
                write_group(r0, g0);
                if (g1 < 4) write_group(r1, g1);
            }
            warp_arrive(&sm.sempty[slot], lane);  // done with this unit's statistics
        }
    b_done:;
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && sm.abort && status != nullptr) atomicExch(status, MLKB_ERR_TIMEOUT);
}

}  // namespace
}  // namespace mlkb

namespace mlkb {

// Y[b] = softmax_rows(scale * Q[b] * K[b]^T) over Q [batch, m, d] and either
// K [batch, s, d] (kt == false) or Kt [batch, d, s] (kt == true); Y is
// [batch, m, s]. Fused kernel for m, s multiples of 128 and d in {64, 128};
// otherwise the two-step form (tcgen05 GEMM with the scale in its epilogue,
// then the row softmax in place).
int launchQkSoftmax(const void* q, const void* k, float* y, int64_t batch, int64_t m, int64_t s,
                    int64_t d, double scale, bool kt, cudaStream_t st) {
    if (q == nullptr || k == nullptr || y == nullptr) {
        return setError(MLKB_ERR_INVALID, "qk_softmax: null buffer");
    }
    if (batch <= 0 || m <= 0 || s <= 0 || d <= 0) {
        return setError(MLKB_ERR_INVALID, "qk_softmax: shape must be positive");
    }
    if (d % 8 != 0 || s % 8 != 0 || !aligned16(q) || !aligned16(k) || !aligned16(y) ||
        batch * m > (int64_t(1) << 30) || batch * s > (int64_t(1) << 30) ||
        batch * d > (int64_t(1) << 30)) {
        return setError(MLKB_ERR_INVALID,
                        "qk_softmax: d and s must be multiples of 8 with 16-byte aligned buffers");
    }
    if (m % kRows != 0 || s % kChunk != 0 || (d != 64 && d != 128)) {
        if (!kt) {
            if (int rc = launchGemmTc(q, k, y, batch, m, s, d, true, 0,
                                      static_cast<float>(scale), st)) {
                return rc;
            }
        } else {
            // One launch per batch: each batch's Kt is its own [d, s] tensor,
            // so a K tile past d reads zeros, never the next batch's rows.
            for (int64_t b = 0; b < batch; ++b) {
                if (int rc = launchGemmTc(static_cast<const __half*>(q) + b * m * d,
                                          static_cast<const __half*>(k) + b * d * s, y + b * m * s,
                                          1, m, s, d, false, 0, static_cast<float>(scale), st)) {
                    return rc;
                }
            }
        }
        return mlkb_softmax_f32(y, y, batch * m, s, st);
    }
    CUtensorMap tq, tk;
    if (int rc = makeTmapF16(&tq, q, batch * m, d, kRows, 64)) return rc;
    if (kt) {
        if (int rc = makeTmapF16(&tk, k, batch * d, s, 64, 64)) return rc;
    } else {
        if (int rc = makeTmapF16(&tk, k, batch * s, d, kChunk, 64)) return rc;
    }
    static std::atomic<bool> attr[8][64];
    int dev = 0;
    cudaGetDevice(&dev);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (static_cast<size_t>(optin) < kSmemBytes) {
        char msg[160];
        snprintf(msg, sizeof(msg), "qk_softmax: needs %zu B of shared memory, device allows %d",
                 kSmemBytes, optin);
        return setError(MLKB_ERR_LAUNCH, msg);
    }
    // Square batches (m == s) with row lengths of 1024, 2048 and 4096 get a
    // kernel specialised on them: a pass-2 warp then addresses all 32 rows of
    // a group from one base by immediate offsets instead of stepping a 64-bit
    // pointer per store.
    const int len = m != s ? 0 : s == 1024 ? 1 : s == 2048 ? 2 : s == 4096 ? 3 : 0;
    using Kern = decltype(&qk_softmax_tcgen05<0, false>);
    static const Kern kKerns[8] = {
        qk_softmax_tcgen05<0, false>,    qk_softmax_tcgen05<1024, false>,
        qk_softmax_tcgen05<2048, false>, qk_softmax_tcgen05<4096, false>,
        qk_softmax_tcgen05<0, true>,     qk_softmax_tcgen05<1024, true>,
        qk_softmax_tcgen05<2048, true>,  qk_softmax_tcgen05<4096, true>};
    const int which = len + (kt ? 4 : 0);
    const Kern kern = kKerns[which];
    if (dev >= 0 && dev < 64 && !attr[which][dev]) {
        const cudaError_t e = cudaFuncSetAttribute(
            kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "qk smem attribute");
        attr[which][dev] = true;
    }
    const int64_t units = batch * (m / kRows);
    const int grid = static_cast<int>(units < smCount() ? units : smCount());
    // Run length: the longest of 4, 2, 1 bands that divides a batch's bands
    // and keeps the last wave of runs over the CTAs at least as full as any
    // shorter run would (within 2 %). Longer runs share K loads and keep the
    // CTAs on few batches at a time (K stays in L2); shorter runs balance
    // better when few units remain (a batch split over several GPUs).
    const int64_t bands = m / kRows;
    int run = 1;
    double best = 0.0;
    for (int r = kRun; r >= 1; r /= 2) {
        if (bands % r != 0) continue;
        const double runs = static_cast<double>(units / r);
        const double waves = std::ceil(runs / grid);
        const double fill = runs / (waves * grid);
        if (run == 1 && best == 0.0) {
            run = r;
            best = fill;
        } else if (fill > best + 0.02) {
            run = r;
            best = fill;
        }
    }
    // exp(scale * v) = exp2(scale * log2(e) * v)
    const float c2 = static_cast<float>(scale * 1.4426950408889634);
    kern<<<grid, kThreads, kSmemBytes, st>>>(tq, tk, y, static_cast<int>(batch),
                                             static_cast<int>(m), static_cast<int>(s),
                                             static_cast<int>(d), run, c2, deviceStatusPtr());
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, kern);
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "qk_softmax launch: %s (regs %d, max threads %d, static smem %zu, "
                 "max dynamic smem %d, requested %zu, threads %d)",
                 cudaGetErrorString(le), fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes,
                 fa.maxDynamicSharedSizeBytes, kSmemBytes, kThreads);
        return setError(MLKB_ERR_LAUNCH, msg);
    }
    return okStatus();
}

}  // namespace mlkb

extern "C" int mlkb_qk_softmax_f16(const void* q, const void* k, float* y, int64_t batch,
                                   int64_t s, int64_t d, double scale, void* stream) {
    return mlkb::launchQkSoftmax(q, k, y, batch, s, s, d, scale, false, mlkb::asStream(stream));
}

extern "C" int mlkb_qk_softmax_kt_f16(const void* q, const void* kt, float* y, int64_t batch,
                                      int64_t m, int64_t s, int64_t d, double scale,
                                      void* stream) {
    return mlkb::launchQkSoftmax(q, kt, y, batch, m, s, d, scale, true, mlkb::asStream(stream));
}
