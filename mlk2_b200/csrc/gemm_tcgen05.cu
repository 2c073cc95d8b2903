// Dense GEMM C[M,N] (+)= A[M,K] * B[K,N], f16 inputs, f32 accumulation in
// TMEM, f32 output, all row-major (reference gemmRowBlock,
// runtime/src/execution/kernel_buffers.cpp:406-432, which accumulates into C).
//
// Plain GEMMs ([K,N] B, no batch) run on CTA pairs (gemm_f16_tcgen05_pair,
// 256x256 tiles, tcgen05 cta_group::2); the batched / K-major-B form used by
// the scaled-scores fallback runs on single CTAs.
//
// Single-CTA design (one CTA per SM, persistent over 128x256 output tiles):
//   warp 0      TMA producer: A tile [128 x 64] (K-major, 128B swizzle) and
//               B tile [64 x 256] as four [64 x 64] boxes (N-major, 128B
//               swizzle) per stage into a 4-stage shared-memory ring;
//   warp 1      MMA issuer: one thread issues tcgen05.mma M128 N256 K16
//               (A K-major, B MN-major descriptors) into a TMEM accumulator
//               and releases each stage with tcgen05.commit;
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (each thread owns one
//               row: its warp's TMEM lane quarter), f32 stores to C.
// The accumulator is double-buffered in TMEM (2 x 256 of the 512 columns), so
// the epilogue of tile i overlaps the MMAs of tile i+1. Tiles are visited in
// groups of 16 M-blocks so the A and B panels in flight stay L2-resident.
// Every mbarrier wait is bounded (2 s); a wait that gives up raises the
// device status word (MLKB_ERR_TIMEOUT), drains its own copies and returns.
// No TMA multicast is used anywhere.
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <climits>
#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"

namespace mlkb {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr uint32_t kAStage = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kBBox = kBK * 64 * 2;     // 8 KB: [64 K-rows x 64 N]
constexpr uint32_t kBStage = kBK * kBN * 2;  // 32 KB
constexpr int kThreads = 192;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kGroupM = 16;     // one-CTA kernel: 16 x 128-row M-blocks
constexpr int kPairGroupM = 8;  // pair kernel: 8 x 256-row M-blocks

struct GemmSmem {
    uint8_t a[kStages][kAStage];
    uint8_t b[kStages][kBStage];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
    int abort;
};

constexpr size_t kSmemBytes = sizeof(GemmSmem) + 1024;

// Tiles are visited in groups of G M-blocks (all N-blocks of a group before
// the next group) so the A and B panels in flight stay L2-resident.
template <int G>
__device__ __forceinline__ void tileCoords(int tile, int mt, int nt, int& mb, int& nb) {
    const int per_group = G * nt;
    const int g = tile / per_group;
    const int first = g * G;
    const int gsize = (mt - first) < G ? (mt - first) : G;
    const int r = tile % per_group;
    mb = first + r % gsize;
    nb = r / gsize;
}

// Bounded wait used only while draining at exit (ignores the abort flag).
__device__ __forceinline__ void drainWait(uint64_t* bar, uint32_t parity) {
    int never = 0;
    (void)tc::mbar_wait(bar, parity, &never, kWaitLimitNs);
}

// kBKMajor: B is given as [N, K] row-major (K-major, e.g. the K operand of
// Q*K^T) instead of [K, N] row-major. Batched: `batch` independent problems
// stacked along the row dimension of A ([batch*m, k]), B ([batch*n, k] when
// K-major; one shared [k, n] otherwise) and C ([batch*m, n]).
template <bool kBKMajor>
__global__ void __launch_bounds__(kThreads, 1)
gemm_f16_tcgen05(const __grid_constant__ CUtensorMap tma_a,
                 const __grid_constant__ CUtensorMap tma_b, float* __restrict__ c, int batch,
                 int m, int n, int k, int accumulate, float scale, int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    GemmSmem& s = *reinterpret_cast<GemmSmem*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (m + kBM - 1) / kBM, nt = (n + kBN - 1) / kBN, kt = (k + kBK - 1) / kBK;
    const int per_batch = mt * nt;
    const int tiles = batch * per_batch;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.tfull[i], 1);
            tc::mbar_init(&s.tempty[i], 128);
        }
        s.abort = 0;
        tc::fence_barrier_init();
        tc::fence_proxy_async();
    }
    if (warp == 0) tc::tmem_alloc(&s.tmem_base, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    volatile int* abort = &s.abort;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer ----
        tc::prefetch_tmap(&tma_a);
        tc::prefetch_tmap(&tma_b);
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int bt = tile / per_batch;
            int mb, nb;
            tileCoords<kGroupM>(tile - bt * per_batch, mt, nt, mb, nb);
            const int arow = bt * m + mb * kBM;
            for (int kb = 0; kb < kt; ++kb) {
                const int st = static_cast<int>(it % kStages);
                const uint32_t ph = (it / kStages) & 1u;
                if (!tc::mbar_wait(&s.empty[st], ph ^ 1u, abort, kWaitLimitNs)) goto producer_done;
                tc::mbar_arrive_expect_tx(&s.full[st], kAStage + kBStage);
                tc::tma_load_2d(s.a[st], &tma_a, &s.full[st], kb * kBK, arow);
                if constexpr (kBKMajor) {
                    // one [256 rows x 64 K] box, rows of the same batch
                    tc::tma_load_2d(s.b[st], &tma_b, &s.full[st], kb * kBK, bt * n + nb * kBN);
                } else {
#pragma unroll
                    for (int j = 0; j < kBN / 64; ++j) {
                        tc::tma_load_2d(s.b[st] + j * kBBox, &tma_b, &s.full[st],
                                        nb * kBN + j * 64, kb * kBK);
                    }
                }
                ++it;
            }
        }
    producer_done:
        // Drain: every issued stage has landed before the CTA may exit.
        for (uint32_t j = it > kStages ? it - kStages : 0; j < it; ++j) {
            drainWait(&s.full[j % kStages], (j / kStages) & 1u);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        constexpr uint32_t kIdesc = tc::idesc_f16_f32(kBM, kBN, 0, kBKMajor ? 0 : 1);
        uint32_t it = 0, local = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const uint32_t acc = local & 1u, aph = (local >> 1) & 1u;
            if (!tc::mbar_wait(&s.tempty[acc], aph ^ 1u, abort, kWaitLimitNs)) break;
            tc::tc_fence_after();
            const uint32_t d = tmem + acc * kBN;
            for (int kb = 0; kb < kt; ++kb, ++it) {
                const int st = static_cast<int>(it % kStages);
                const uint32_t ph = (it / kStages) & 1u;
                if (!tc::mbar_wait(&s.full[st], ph, abort, kWaitLimitNs)) goto mma_done;
                tc::tc_fence_after();
                const uint32_t a0 = tc::smem_u32(s.a[st]);
                const uint32_t b0 = tc::smem_u32(s.b[st]);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    // A: K-major, advance 16 elements = 32 B inside the swizzle atom.
                    const uint64_t ad = tc::smem_desc_sw128(a0 + kk * 32, 16, 1024);
                    // B MN-major: 16 K-rows = two 1024 B atoms; 64-column chunks 8 KB apart.
                    // B K-major: same form as A.
                    const uint64_t bd = kBKMajor ? tc::smem_desc_sw128(b0 + kk * 32, 16, 1024)
                                                 : tc::smem_desc_sw128(b0 + kk * 2048, kBBox, 1024);
                    tc::mma_f16(d, ad, bd, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit(&s.empty[st]);
            }
            tc::mma_commit(&s.tfull[acc]);
        }
    mma_done:;
    } else if (warp >= 2) {
        // ---- epilogue: TMEM -> registers -> global ----
        const int quarter = warp & 3;  // TMEM lanes this warp may read
        const int row_in_tile = quarter * 32 + lane;
        uint32_t local = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int bt = tile / per_batch;
            int mb, nb;
            tileCoords<kGroupM>(tile - bt * per_batch, mt, nt, mb, nb);
            const uint32_t acc = local & 1u, aph = (local >> 1) & 1u;
            if (!tc::mbar_wait(&s.tfull[acc], aph, abort, kWaitLimitNs)) break;
            tc::tc_fence_after();
            const int64_t row = static_cast<int64_t>(mb) * kBM + row_in_tile;
            float* crow = c + (static_cast<int64_t>(bt) * m + row) * n;
#pragma unroll 1
            for (int cc = 0; cc < kBN / 32; ++cc) {
                uint32_t r[32];
                tc::tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN +
                                  cc * 32,
                              r);
                tc::tmem_ld_wait();
                const int col0 = nb * kBN + cc * 32;
                if (row < m) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int col = col0 + q * 4;
                        if (col < n) {
                            float4 v = make_float4(__uint_as_float(r[4 * q]) * scale,
                                                   __uint_as_float(r[4 * q + 1]) * scale,
                                                   __uint_as_float(r[4 * q + 2]) * scale,
                                                   __uint_as_float(r[4 * q + 3]) * scale);
                            float4* dst = reinterpret_cast<float4*>(crow + col);
                            if (accumulate) {
                                const float4 o = *dst;
                                v.x += o.x;
                                v.y += o.y;
                                v.z += o.z;
                                v.w += o.w;
                            }
                            *dst = v;
                        }
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&s.tempty[acc]);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && s.abort && status != nullptr) atomicExch(status, MLKB_ERR_TIMEOUT);
}

// ---- CTA-pair variant: 256 x 256 tiles over a cluster of two SMs ------------
// tcgen05.mma.cta_group::2 M256 N256 K16: the even CTA of the pair issues the
// MMAs; each CTA stages its own 128 rows of A and its own 128 columns of B
// (half the B traffic of the one-CTA kernel per output element, and each SM's
// tensor core reads 8 KB of shared memory per K16 step instead of 12 KB).
// Both CTAs' TMA loads complete on the even CTA's `full` barrier; the MMA
// commit multicasts stage release and accumulator-ready to both CTAs; both
// epilogues report a drained accumulator on the even CTA's `tempty`.
constexpr int kPairBK = 128;                         // K per stage: two 64-wide halves
constexpr int kPairStages = 3;
constexpr uint32_t kPairA = kBM * kPairBK * 2;             // 32 KB: two [128 x 64] boxes
constexpr uint32_t kPairB = kPairBK * (kBN / 2) * 2;       // 32 KB: 2 K-halves x 2 N-boxes

struct PairSmem {
    uint8_t a[kPairStages][kPairA];
    uint8_t b[kPairStages][kPairB];
    uint64_t full[kPairStages];
    uint64_t empty[kPairStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
    int abort;
};

constexpr size_t kPairSmemBytes = sizeof(PairSmem) + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_f16_tcgen05_pair(const __grid_constant__ CUtensorMap tma_a,
                      const __grid_constant__ CUtensorMap tma_b, float* __restrict__ c, int m,
                      int n, int k, int accumulate, int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    PairSmem& s = *reinterpret_cast<PairSmem*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_ctarank();
    const bool leader = (rank == 0);
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int mt = (m + 2 * kBM - 1) / (2 * kBM), nt = (n + kBN - 1) / kBN;
    const int kt = (k + kPairBK - 1) / kPairBK;
    const int tiles = mt * nt;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kPairStages; ++i) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.tfull[i], 1);
            tc::mbar_init(&s.tempty[i], 2 * 4);  // the epilogue warps of both CTAs
        }
        s.abort = 0;
        tc::fence_barrier_init();
        tc::fence_proxy_async();
    }
    if (warp == 0) tc::tmem_alloc_pair(&s.tmem_base, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::cluster_sync();  // barriers of both CTAs initialised before any remote use
    tc::tc_fence_after();
    // Programmatic dependent launch: the set-up above overlaps the tail of the
    // preceding grid; wait for it (its writes visible: C may be accumulated
    // into) before any global access, and let the next grid be scheduled as
    // our CTAs retire. Both are no-ops for a plain launch.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t tmem = s.tmem_base;
    volatile int* abort = &s.abort;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer (both CTAs): own A rows and own half of B ----
        tc::prefetch_tmap(&tma_a);
        tc::prefetch_tmap(&tma_b);
        uint32_t it = 0;
        for (int tile = pair; tile < tiles && !*abort; tile += pairs) {
            int mb, nb;
            tileCoords<kPairGroupM>(tile, mt, nt, mb, nb);
            const int arow = mb * 2 * kBM + static_cast<int>(rank) * kBM;
            const int bcol = nb * kBN + static_cast<int>(rank) * (kBN / 2);
            for (int kb = 0; kb < kt; ++kb, ++it) {
                const int st = static_cast<int>(it % kPairStages);
                const uint32_t ph = (it / kPairStages) & 1u;
                if (!tc::mbar_wait(&s.empty[st], ph ^ 1u, abort, kWaitLimitNs)) goto producer_done;
                if (leader) tc::mbar_arrive_expect_tx(&s.full[st], 2 * (kPairA + kPairB));
                const uint32_t bar = tc::mapa_shared(tc::smem_u32(&s.full[st]), 0);
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // K halves of the stage
                    const int k0 = kb * kPairBK + h * 64;
                    tc::tma_load_2d_pair(s.a[st] + h * kAStage, &tma_a, bar, k0, arow);
                    tc::tma_load_2d_pair(s.b[st] + h * 2 * kBBox, &tma_b, bar, bcol, k0);
                    tc::tma_load_2d_pair(s.b[st] + h * 2 * kBBox + kBBox, &tma_b, bar, bcol + 64, k0);
                }
            }
        }
    producer_done:
        // The even CTA's full barriers count both CTAs' bytes: draining them
        // there covers every load of the pair (the final cluster barrier keeps
        // the odd CTA alive until then).
        if (leader) {
            for (uint32_t j = it > kPairStages ? it - kPairStages : 0; j < it; ++j) {
                drainWait(&s.full[j % kPairStages], (j / kPairStages) & 1u);
            }
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ---- MMA issuer (even CTA only) ----
        constexpr uint32_t kIdesc = tc::idesc_f16_f32(2 * kBM, kBN, 0, 1);
        uint32_t it = 0, local = 0;
        for (int tile = pair; tile < tiles; tile += pairs, ++local) {
            const uint32_t acc = local & 1u, aph = (local >> 1) & 1u;
            if (!tc::mbar_wait(&s.tempty[acc], aph ^ 1u, abort, kWaitLimitNs)) break;
            tc::tc_fence_after();
            const uint32_t d = tmem + acc * kBN;
            for (int kb = 0; kb < kt; ++kb, ++it) {
                const int st = static_cast<int>(it % kPairStages);
                const uint32_t ph = (it / kPairStages) & 1u;
                if (!tc::mbar_wait(&s.full[st], ph, abort, kWaitLimitNs)) goto mma_done;
                tc::tc_fence_after();
                const uint32_t a0 = tc::smem_u32(s.a[st]);
                const uint32_t b0 = tc::smem_u32(s.b[st]);
#pragma unroll
                for (int kk = 0; kk < kPairBK / 16; ++kk) {
                    const uint32_t h = kk >> 2, q = kk & 3;  // K half, K16 step inside it
                    const uint64_t ad = tc::smem_desc_sw128(a0 + h * kAStage + q * 32, 16, 1024);
                    const uint64_t bd =
                        tc::smem_desc_sw128(b0 + h * 2 * kBBox + q * 2048, kBBox, 1024);
                    tc::mma_f16_pair(d, ad, bd, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit_pair(&s.empty[st], 0x3);
            }
            tc::mma_commit_pair(&s.tfull[acc], 0x3);
        }
    mma_done:;
    } else if (warp >= 2) {
        // ---- epilogue (both CTAs): own 128 rows x 256 columns ----
        const int quarter = warp & 3;
        const int row_in_tile = static_cast<int>(rank) * kBM + quarter * 32 + lane;
        uint32_t local = 0;
        for (int tile = pair; tile < tiles; tile += pairs, ++local) {
            int mb, nb;
            tileCoords<kPairGroupM>(tile, mt, nt, mb, nb);
            const uint32_t acc = local & 1u, aph = (local >> 1) & 1u;
            if (!tc::mbar_wait(&s.tfull[acc], aph, abort, kWaitLimitNs)) break;
            tc::tc_fence_after();
            const int64_t row = static_cast<int64_t>(mb) * 2 * kBM + row_in_tile;
            float* crow = c + row * n;
#pragma unroll 1
            for (int cc = 0; cc < kBN / 32; ++cc) {
                uint32_t r[32];
                tc::tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN +
                                  cc * 32,
                              r);
                tc::tmem_ld_wait();
                const int col0 = nb * kBN + cc * 32;
                if (row < m) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int col = col0 + q * 4;
                        if (col < n) {
                            float4 v = make_float4(__uint_as_float(r[4 * q]),
                                                   __uint_as_float(r[4 * q + 1]),
                                                   __uint_as_float(r[4 * q + 2]),
                                                   __uint_as_float(r[4 * q + 3]));
                            float4* dst = reinterpret_cast<float4*>(crow + col);
                            if (accumulate) {
                                const float4 o = *dst;
                                v.x += o.x;
                                v.y += o.y;
                                v.z += o.z;
                                v.w += o.w;
                            }
                            *dst = v;
                        }
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_cluster(tc::mapa_shared(tc::smem_u32(&s.tempty[acc]), 0));
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::cluster_sync();  // no MMA, load or remote arrive of the pair is still pending
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc_pair(tmem, 512);
    }
    if (threadIdx.x == 0 && s.abort && status != nullptr) atomicExch(status, MLKB_ERR_TIMEOUT);
}

// Generic SIMT fallback for shapes or alignments TMA cannot take
// (K or N not a multiple of 8, or unaligned bases).
__global__ void gemm_f16_simt(const __half* __restrict__ a, const __half* __restrict__ b,
                              float* __restrict__ c, int64_t m, int64_t n, int64_t k,
                              int accumulate) {
    const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t row = blockIdx.y;
    if (col >= n || row >= m) return;
    float acc = 0.0f;
    for (int64_t p = 0; p < k; ++p) {
        acc = fmaf(__half2float(a[row * k + p]), __half2float(b[p * n + col]), acc);
    }
    c[row * n + col] = accumulate ? c[row * n + col] + acc : acc;
}

PFN_cuTensorMapEncodeTiled_v12000 encodeFn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    return fn;
}

}  // namespace

// 2-D tensor map over a row-major [rows, cols] matrix of `elem_bytes`-wide
// elements, box [box_rows, box_cols]; out-of-range elements load as zero.
int makeTmap2d(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes, const void* base,
               int64_t rows, int64_t cols, int box_rows, int box_cols,
               CUtensorMapSwizzle swizzle) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encodeFn();
    if (enc == nullptr) return setError(MLKB_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * elem_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? okStatus() : setError(MLKB_ERR_INVALID, "tensor map encode failed");
}

// 2-D f16 tensor map, 128-byte swizzle (box_cols * 2 must be 128).
int makeTmapF16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows,
                int box_cols) {
    return makeTmap2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, rows, cols, box_rows,
                      box_cols, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace mlkb

namespace mlkb {

// Launches the tcgen05 GEMM. b_kmajor: B is [batch*n, k] row-major; else [k, n].
int launchGemmTc(const void* a, const void* b, float* c, int64_t batch, int64_t m, int64_t n,
                 int64_t k, bool b_kmajor, int accumulate, float scale, cudaStream_t s) {
    CUtensorMap ta, tb;
    if (int st = makeTmapF16(&ta, a, batch * m, k, kBM, kBK)) return st;
    if (b_kmajor) {
        if (int st = makeTmapF16(&tb, b, batch * n, k, kBN, kBK)) return st;
    } else {
        if (int st = makeTmapF16(&tb, b, k, n, kBK, 64)) return st;
    }
    static std::atomic<bool> attr[2][64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[b_kmajor][dev]) {
        const cudaError_t e = b_kmajor
            ? cudaFuncSetAttribute(gemm_f16_tcgen05<true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kSmemBytes))
            : cudaFuncSetAttribute(gemm_f16_tcgen05<false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "gemm smem attribute");
        attr[b_kmajor][dev] = true;
    }
    const int64_t tiles = batch * ((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
    const int grid = static_cast<int>(tiles < smCount() ? tiles : smCount());
    if (b_kmajor) {
        gemm_f16_tcgen05<true><<<grid, kThreads, kSmemBytes, s>>>(
            ta, tb, c, static_cast<int>(batch), static_cast<int>(m), static_cast<int>(n),
            static_cast<int>(k), accumulate, scale, deviceStatusPtr());
    } else {
        gemm_f16_tcgen05<false><<<grid, kThreads, kSmemBytes, s>>>(
            ta, tb, c, static_cast<int>(batch), static_cast<int>(m), static_cast<int>(n),
            static_cast<int>(k), accumulate, scale, deviceStatusPtr());
    }
    return checkLaunch("gemm tcgen05 launch");
}

// Launches the CTA-pair tcgen05 GEMM (B is [k, n] row-major, no batch, no
// scale). Returns MLKB_ERR_LAUNCH when a pair launch is refused, so the caller
// can take the one-CTA kernel.
int launchGemmPair(const void* a, const void* b, float* c, int64_t m, int64_t n, int64_t k,
                   int accumulate, cudaStream_t s) {
    CUtensorMap ta, tb;
    if (int st = makeTmapF16(&ta, a, m, k, kBM, kBK)) return st;
    if (int st = makeTmapF16(&tb, b, k, n, kBK, 64)) return st;
    static std::atomic<bool> attr[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(gemm_f16_tcgen05_pair,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kPairSmemBytes));
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "gemm pair smem attribute");
        attr[dev] = true;
    }
    const int64_t tiles = ((m + 2 * kBM - 1) / (2 * kBM)) * ((n + kBN - 1) / kBN);
    const int64_t pairs_max = smCount() / 2;
    const int grid = 2 * static_cast<int>(tiles < pairs_max ? tiles : pairs_max);
    // Programmatic stream serialization (the kernel waits for its predecessor
    // itself); the cluster shape comes from the kernel's __cluster_dims__.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kPairSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, gemm_f16_tcgen05_pair, ta, tb, c,
                                              static_cast<int>(m), static_cast<int>(n),
                                              static_cast<int>(k), accumulate, deviceStatusPtr());
    if (le != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, le, "gemm tcgen05 pair launch");
    return checkLaunch("gemm tcgen05 pair launch");
}

}  // namespace mlkb

extern "C" int mlkb_gemm_f16_f32(const void* a, const void* b, float* c, int64_t m, int64_t n,
                                 int64_t k, int32_t accumulate, void* stream) {
    using namespace mlkb;
    if (a == nullptr || b == nullptr || c == nullptr) {
        return setError(MLKB_ERR_INVALID, "gemm: null buffer");
    }
    if (m <= 0 || n <= 0 || k <= 0) return setError(MLKB_ERR_INVALID, "gemm: shape must be positive");
    cudaStream_t s = asStream(stream);
    const bool tma_ok = (k % 8 == 0) && (n % 8 == 0) && aligned16(a) && aligned16(b) &&
                        aligned16(c) && m <= INT_MAX / 2 && n <= INT_MAX / 2 && k <= INT_MAX / 2;
    if (!tma_ok) {
        if (m > 65535) return setError(MLKB_ERR_INVALID, "gemm: unaligned shape with M > 65535");
        const dim3 grid(static_cast<unsigned>((n + 127) / 128), static_cast<unsigned>(m));
        gemm_f16_simt<<<grid, 128, 0, s>>>(static_cast<const __half*>(a),
                                           static_cast<const __half*>(b), c, m, n, k,
                                           accumulate ? 1 : 0);
        return checkLaunch("gemm f16 simt launch");
    }
    if (smCount() >= 2 && launchGemmPair(a, b, c, m, n, k, accumulate ? 1 : 0, s) == MLKB_OK) {
        return MLKB_OK;
    }
    return launchGemmTc(a, b, c, 1, m, n, k, false, accumulate ? 1 : 0, 1.0f, s);
}
