// Batched scaled-scores softmax: Y[b] = softmax_rows(scale * Q[b] * K[b]^T).
//
// The reference has no fused operator: its composition is Call(MatMul) ->
// scale map -> Call(Softmax) (runtime/src/execution/kernel_buffers.cpp:
// 1001-1085, :342-402, :290-340), evaluated in f64 with K^T materialised.
// Q and K are f16 [batch, s, d] row-major here, so K is already the K-major
// operand the tcgen05 MMA wants: no transpose is materialised.
//
// Fused kernel (s % 256 == 0, d in {64, 128}); one CTA per SM, persistent
// over units = (batch, 128-row band). The output write (4 B per score) is the
// roofline, so every score is written exactly once and nothing else is:
//   warp 0     TMA producer: the Q band [128 x d] once per unit, then K in
//              [256 x 64] boxes through a 4-stage ring (128 KB in flight covers
//              the L2 latency at the MMA's consumption rate), all s/256 column
//              chunks twice (pass 1 and pass 2);
//   warp 1     MMA issuer: tcgen05.mma M128 N256 K16 (both operands K-major)
//              into one of two TMEM accumulators per chunk;
//   warps 2-17 epilogue, four warps per TMEM lane quarter (64 columns each):
//              pass 1 keeps an online row max / sum of exp2(scale*log2e*s);
//              the four parts merge their statistics through shared memory;
//              pass 2 recomputes each chunk (the MMA is far cheaper than a
//              second trip through HBM) and writes exp2(v - m) / l, transposed
//              through an XOR-swizzled shared-memory tile so that every global
//              store is a full 128-byte row segment.
// Every mbarrier wait is bounded (2 s); on a timeout the CTA raises the
// device status word, drains its copies, frees TMEM and returns.
// Other shapes use the two-step form (tcgen05 GEMM with the scale folded into
// its epilogue, then the row softmax in place).
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <cstdio>

#include "common.cuh"
#include "tc_common.cuh"

namespace mlkb {
int launchGemmTc(const void* a, const void* b, float* c, int64_t batch, int64_t m, int64_t n,
                 int64_t k, bool b_kmajor, int accumulate, float scale, cudaStream_t s);
int makeTmapF16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows,
                int box_cols);

namespace {

constexpr int kRows = 128;          // score rows per unit (M of the MMA)
constexpr int kChunk = 256;         // score columns per accumulator (N of the MMA)
constexpr int kKStages = 4;         // K ring depth, [256 x 64] f16 boxes
constexpr uint32_t kKBox = kChunk * 64 * 2;   // 32 KB
constexpr uint32_t kQBox = kRows * 64 * 2;    // 16 KB
constexpr int kEpiWarps = 16;                 // 4 per TMEM lane quarter
constexpr int kParts = kEpiWarps / 4;         // column parts of a chunk
constexpr int kPartCols = kChunk / kParts;    // 64 columns per warp per chunk
constexpr int kThreads = 64 + kEpiWarps * 32;  // 576
constexpr uint32_t kStageTile = 32 * 32 * 4;  // [32 rows x 32 cols] f32 = 4 KB
constexpr uint64_t kLimitNs = 2000000000ull;

struct QkSmem {
    uint8_t k[kKStages][kKBox];       // 128 KB
    uint8_t q[2][kQBox];              // 32 KB (two d-halves)
    uint8_t out[kEpiWarps][kStageTile];  // 64 KB; also carries the row statistics
    uint64_t kfull[kKStages], kempty[kKStages];
    uint64_t qfull, qempty;
    uint64_t tfull[2], tempty[2];
    uint32_t tmem_base;
    int abort;
};

constexpr size_t kSmemBytes = sizeof(QkSmem);

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
qk_softmax_tcgen05(const __grid_constant__ CUtensorMap tma_q,
                   const __grid_constant__ CUtensorMap tma_k,
                   float* __restrict__ y, int batch, int s, int d, float c2,
                   uint32_t stagger_ns, int* __restrict__ status) {
    // The kernel has no static shared memory, so the dynamic window starts at
    // the 1024-byte aligned base the 128B-swizzled tiles need.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    QkSmem& sm = *reinterpret_cast<QkSmem*>(smem_raw);
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {  // uniform across the CTA
        if (threadIdx.x == 0 && status != nullptr) atomicExch(status, MLKB_ERR_INVALID);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bands = s / kRows;
    const int units = batch * bands;
    const int chunks = s / kChunk;
    const int dh = d / 64;  // d-halves per chunk (1 or 2)

    if (threadIdx.x == 0) {
        for (int i = 0; i < kKStages; ++i) {
            tc::mbar_init(&sm.kfull[i], 1);
            tc::mbar_init(&sm.kempty[i], 1);
        }
        tc::mbar_init(&sm.qfull, 1);
        tc::mbar_init(&sm.qempty, 1);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&sm.tfull[i], 1);
            tc::mbar_init(&sm.tempty[i], kEpiWarps);
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

    // Pass 1 only computes and pass 2 mostly writes; CTAs that start together
    // would alternate between an idle and an oversubscribed HBM. Odd CTAs start
    // about one pass late, so at any time half the SMs are writing.
    if ((blockIdx.x & 1) && stagger_ns > 0 && warp == 0 && lane == 0) {
        const uint64_t t0 = tc::global_timer_ns();
        while (tc::global_timer_ns() - t0 < stagger_ns) __nanosleep(1000);
    }

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        tc::prefetch_tmap(&tma_q);
        tc::prefetch_tmap(&tma_k);
        uint32_t kit = 0, ui = 0;
        for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x, ++ui) {
            const int b = u / bands, band = u - b * bands;
            const int qrow = b * s + band * kRows;
            if (!tc::mbar_wait(&sm.qempty, (ui & 1u) ^ 1u, abort, kLimitNs)) break;
            tc::mbar_arrive_expect_tx(&sm.qfull, kQBox * dh);
            for (int h = 0; h < dh; ++h) tc::tma_load_2d(sm.q[h], &tma_q, &sm.qfull, h * 64, qrow);
            for (int c = 0; c < 2 * chunks; ++c) {
                const int krow = b * s + (c % chunks) * kChunk;
                for (int h = 0; h < dh; ++h, ++kit) {
                    const int st = static_cast<int>(kit % kKStages);
                    if (!tc::mbar_wait(&sm.kempty[st], ((kit / kKStages) & 1u) ^ 1u, abort,
                                       kLimitNs)) {
                        goto producer_done;
                    }
                    tc::mbar_arrive_expect_tx(&sm.kfull[st], kKBox);
                    tc::tma_load_2d(sm.k[st], &tma_k, &sm.kfull[st], h * 64, krow);
                }
            }
        }
    producer_done:
        for (uint32_t j = kit > kKStages ? kit - kKStages : 0; j < kit; ++j) {
            int never = 0;
            (void)tc::mbar_wait(&sm.kfull[j % kKStages], (j / kKStages) & 1u, &never, kLimitNs);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t kIdesc = tc::idesc_f16_f32(kRows, kChunk, 0, 0);
        uint32_t kit = 0, acc_it = 0, ui = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++ui) {
            if (!tc::mbar_wait(&sm.qfull, ui & 1u, abort, kLimitNs)) goto mma_done;
            tc::tc_fence_after();
            for (int c = 0; c < 2 * chunks; ++c, ++acc_it) {
                const uint32_t acc = acc_it & 1u;
                if (!tc::mbar_wait(&sm.tempty[acc], ((acc_it >> 1) & 1u) ^ 1u, abort, kLimitNs)) {
                    goto mma_done;
                }
                tc::tc_fence_after();
                const uint32_t dst = tmem + acc * kChunk;
                for (int h = 0; h < dh; ++h, ++kit) {
                    const int st = static_cast<int>(kit % kKStages);
                    if (!tc::mbar_wait(&sm.kfull[st], (kit / kKStages) & 1u, abort, kLimitNs)) {
                        goto mma_done;
                    }
                    tc::tc_fence_after();
                    const uint32_t q0 = tc::smem_u32(sm.q[h]);
                    const uint32_t k0 = tc::smem_u32(sm.k[st]);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        tc::mma_f16(dst, tc::smem_desc_sw128(q0 + kk * 32, 16, 1024),
                                    tc::smem_desc_sw128(k0 + kk * 32, 16, 1024), kIdesc,
                                    (h > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc::mma_commit(&sm.kempty[st]);
                }
                tc::mma_commit(&sm.tfull[acc]);
            }
            tc::mma_commit(&sm.qempty);  // Q band free once this unit's MMAs finish
        }
    mma_done:;
    } else if (warp >= 2) {
        // ---------------- epilogue ----------------
        const int ew = warp - 2;            // 0..15
        const int quarter = warp & 3;       // TMEM lanes this warp may read
        const int part = ew >> 2;           // which 64 columns of a chunk
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        uint8_t* const tile = sm.out[ew];
        uint32_t acc_it = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const int b = u / bands, band = u - b * bands;
            const int ybase_row = b * s + band * kRows + quarter * 32;
            float m = -INFINITY, l = 0.0f;
            // pass 1: online max / sum over this thread's row, 64 columns per chunk
            for (int c = 0; c < chunks; ++c, ++acc_it) {
                const uint32_t acc = acc_it & 1u;
                if (!tc::mbar_wait(&sm.tfull[acc], (acc_it >> 1) & 1u, abort, kLimitNs)) {
                    goto epi_done;
                }
                tc::tc_fence_after();
                uint32_t r[2][32];
                const uint32_t col = lane_addr + acc * kChunk + part * kPartCols;
                tc::tmem_ld32(tmem + col, r[0]);
                tc::tmem_ld32(tmem + col + 32, r[1]);
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sm.tempty[acc]);  // values are in registers now
                float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(r[i >> 5][i & 31]));
                }
                const float gm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * c2;
                const float mn = fmaxf(m, gm);
                float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    sum[i & 3] += ex2(fmaf(__uint_as_float(r[i >> 5][i & 31]), c2, -mn));
                }
                l = l * ex2(m - mn) + ((sum[0] + sum[1]) + (sum[2] + sum[3]));
                m = mn;
            }
            // merge the four column parts of each row; the statistics travel in
            // the staging tiles, once this warp's last TMA store has read them
            __syncwarp();
            reinterpret_cast<float2*>(tile)[lane] = make_float2(m, l);
            named_sync(1, kEpiWarps * 32);
            {
                float2 st[kParts];
#pragma unroll
                for (int p = 0; p < kParts; ++p) {
                    st[p] = reinterpret_cast<const float2*>(sm.out[4 * p + ((quarter + 2) & 3)])[lane];
                }
                float mm = st[0].x;
#pragma unroll
                for (int p = 1; p < kParts; ++p) mm = fmaxf(mm, st[p].x);
                float ll = 0.0f;
#pragma unroll
                for (int p = 0; p < kParts; ++p) ll += st[p].y * ex2(st[p].x - mm);
                m = mm;
                l = ll;
            }
            named_sync(1, kEpiWarps * 32);  // statistics read before the tiles are reused
            const float inv = 1.0f / l;
            // pass 2: recompute, normalise, transpose through the tile and store
            for (int c = 0; c < chunks; ++c, ++acc_it) {
                const uint32_t acc = acc_it & 1u;
                if (!tc::mbar_wait(&sm.tfull[acc], (acc_it >> 1) & 1u, abort, kLimitNs)) {
                    goto epi_done;
                }
                tc::tc_fence_after();
                const uint32_t col = lane_addr + acc * kChunk + part * kPartCols;
                float* const ydst0 = y + static_cast<int64_t>(ybase_row) * s + c * kChunk +
                                     part * kPartCols;
#pragma unroll 1
                for (int g = 0; g < 2; ++g) {
                    uint32_t r[32];
                    tc::tmem_ld32(tmem + col + g * 32, r);
                    tc::tmem_ld_wait();
                    if (g == 1) {
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&sm.tempty[acc]);
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float4 v;
                        v.x = ex2(fmaf(__uint_as_float(r[4 * j + 0]), c2, -m)) * inv;
                        v.y = ex2(fmaf(__uint_as_float(r[4 * j + 1]), c2, -m)) * inv;
                        v.z = ex2(fmaf(__uint_as_float(r[4 * j + 2]), c2, -m)) * inv;
                        v.w = ex2(fmaf(__uint_as_float(r[4 * j + 3]), c2, -m)) * inv;
                        // row `lane`, 16-byte chunk j, XOR-swizzled (conflict-free)
                        *reinterpret_cast<float4*>(tile + lane * 128 + ((j ^ (lane & 7)) << 4)) = v;
                    }
                    __syncwarp();
                    // transpose through the tile: 8 lanes per row, 4 rows per
                    // instruction, every store a full 128-byte row segment
                    const int jj = lane & 7;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int row = i * 4 + (lane >> 3);
                        const float4 v = *reinterpret_cast<const float4*>(
                            tile + row * 128 + ((jj ^ (row & 7)) << 4));
                        __stcs(reinterpret_cast<float4*>(ydst0 + static_cast<int64_t>(row) * s +
                                                         g * 32) + jj,
                               v);
                    }
                    __syncwarp();
                }
            }
        }
    epi_done:
        __syncwarp();
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

extern "C" int mlkb_qk_softmax_f16(const void* q, const void* k, float* y, int64_t batch,
                                   int64_t s, int64_t d, double scale, void* stream) {
    using namespace mlkb;
    if (q == nullptr || k == nullptr || y == nullptr) {
        return setError(MLKB_ERR_INVALID, "qk_softmax: null buffer");
    }
    if (batch <= 0 || s <= 0 || d <= 0) {
        return setError(MLKB_ERR_INVALID, "qk_softmax: shape must be positive");
    }
    if (d % 8 != 0 || s % 8 != 0 || !aligned16(q) || !aligned16(k) || !aligned16(y) ||
        batch * s > (int64_t(1) << 30)) {
        return setError(MLKB_ERR_INVALID,
                        "qk_softmax: d and s must be multiples of 8 with 16-byte aligned buffers");
    }
    cudaStream_t st = asStream(stream);
    if (s % kChunk != 0 || (d != 64 && d != 128)) {
        if (int rc = launchGemmTc(q, k, y, batch, s, s, d, true, 0, static_cast<float>(scale), st)) {
            return rc;
        }
        return mlkb_softmax_f32(y, y, batch * s, s, stream);
    }
    CUtensorMap tq, tk;
    if (int rc = makeTmapF16(&tq, q, batch * s, d, kRows, 64)) return rc;
    if (int rc = makeTmapF16(&tk, k, batch * s, d, kChunk, 64)) return rc;
    static bool attr[64] = {false};
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
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(
            qk_softmax_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
            static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "qk smem attribute");
        attr[dev] = true;
    }
    const int64_t units = batch * (s / kRows);
    const int grid = static_cast<int>(units < smCount() ? units : smCount());
    // exp(scale * v) = exp2(scale * log2(e) * v)
    const float c2 = static_cast<float>(scale * 1.4426950408889634);
    // About one pass (s/256 chunks of ~1.4 us each at d = 128) when each CTA
    // has several units to amortise it.
    const uint32_t stagger = units >= 4 * static_cast<int64_t>(grid)
                                 ? static_cast<uint32_t>((s / kChunk) * 1400 * d / 128)
                                 : 0u;
    qk_softmax_tcgen05<<<grid, kThreads, kSmemBytes, st>>>(tq, tk, y, static_cast<int>(batch),
                                                          static_cast<int>(s), static_cast<int>(d),
                                                          c2, stagger, deviceStatusPtr());
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, qk_softmax_tcgen05);
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
