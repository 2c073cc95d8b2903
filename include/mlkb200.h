/*
 * mlkb200 — B200 (sm_100a) execution path for MLK+ Kernel IR modules.
 *
 * C ABI of libmlkb200.so. Plain pointers and sizes only; no torch or CUDA
 * types appear in any signature (streams are passed as `void*`, i.e. a
 * cudaStream_t, NULL = the legacy default stream of the current device).
 *
 * Three layers, top to bottom:
 *   1. The reference artifact ABI (`mlk_kernel`, `mlk_bind_module`,
 *      `mlk_last_status`): what MLK+'s backend driver dlsym()s and calls
 *      through LoadedKernel::run with host f64 buffers.
 *   2. Module entry points (`mlkb_module_*`): a Kernel IR module in the
 *      reference's `mlk-kernel` JSON wire format, run over typed device or
 *      host buffers (f16 / f32 / f64), optionally sharded over GPUs.
 *   3. Direct kernel entry points (`mlkb_map_*`, `mlkb_softmax_*`,
 *      `mlkb_gemm_*`, `mlkb_qk_softmax_*`) over device pointers on a stream.
 *
 * Every entry point returns an mlkb status (0 = ok). Codes 1-4 keep the
 * meaning the reference artifact ABI gives them
 * (reference docs/kernel_abi.md:36-41, backends/cpu/src/cuda_emitter.cpp:1912-1913);
 * 5-9 are new. A human-readable message for the last failure on the calling
 * thread is returned by mlkb_last_error().
 */
#ifndef MLKB200_H
#define MLKB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MLKB_OK 0
#define MLKB_ERR_NEG_STORE 1   /* negative store flat index (reference code 1) */
#define MLKB_ERR_CUDA_MEM 2    /* CUDA allocation or copy failed (reference code 2) */
#define MLKB_ERR_LAUNCH 3      /* kernel launch or synchronisation failed (reference code 3) */
#define MLKB_ERR_NO_DEVICE 4   /* no CUDA device (reference code 4) */
#define MLKB_ERR_NCCL 5        /* collective failure */
#define MLKB_ERR_TIMEOUT 6     /* a bounded device-side wait gave up */
#define MLKB_ERR_UNSUPPORTED 7 /* module shape not recognised by this path */
#define MLKB_ERR_INVALID 8     /* bad argument, shape, dtype or alignment */
#define MLKB_ERR_NOT_BOUND 9   /* mlk_kernel called with no module bound */

/* ---- element types ----------------------------------------------------- */
#define MLKB_F16 1
#define MLKB_F32 2
#define MLKB_F64 3

/* ---- module classes (what the pattern matcher recognised) --------------- */
#define MLKB_KIND_MAP 1        /* one or more 1-D Loop{Compute;Store} roots */
#define MLKB_KIND_SOFTMAX 2    /* Call(Softmax) */
#define MLKB_KIND_MATMUL 3     /* Call(MatMul) */
#define MLKB_KIND_REDUCESUM 4  /* Call(ReduceSum) */
#define MLKB_KIND_QK_SOFTMAX 5 /* Call(MatMul) -> scale map -> Call(Softmax) */

/*
 * One expression of a fused per-element chain: the reference's KernelExpr
 * (compiler/include/mlk/support/kernel_ir.h:89-97) with its two operands
 * (KernelOperand, kernel_ir.h:58-83) flattened.
 *   op      mlk::MathOp numbering (compiler/include/mlk/ir/math_op.h:18-36):
 *           Add=0 Sub=1 Mul=2 Div=3 Neg=4 Pow=5 Exp=6 Log=7 Sin=8 Cos=9
 *           Tan=10 Tanh=11 Sqrt=12 Rsqrt=13 Erf=14 Gelu=15
 *   *_kind  KernelOperand::Kind numbering: Const=0 ElemA=1 ElemB=2
 *           ScalarParam=3 Temp=4 (ElemIdx=5 is multi-dim only, not accepted)
 *   *_index ScalarParam: scalar slot; Temp: index of an earlier expression
 *   *_value Const payload
 */
typedef struct mlkb_expr {
    int32_t op;
    int32_t a_kind;
    int64_t a_index;
    double a_value;
    int32_t b_kind;
    int32_t reserved;
    int64_t b_index;
    double b_value;
} mlkb_expr;

typedef struct mlkb_module mlkb_module; /* opaque bound Kernel IR module */

/* ======================================================================= */
/* 1. Reference artifact ABI                                                */
/* ======================================================================= */

/*
 * Binds the module that subsequent mlk_kernel calls execute, given in the
 * reference's `mlk-kernel` JSON format (the output of KernelModule::toJson,
 * reference compiler/src/support/kernel_ir.cpp:97-254). Replaces the module
 * knowledge the reference bakes into each emitted artifact
 * (reference backends/cpu/src/cuda_emitter.cpp:1563-1937). Passing NULL
 * unbinds. When nothing is bound, mlk_kernel reads `module.json` from the
 * directory holding this library (the fastkernel artifact-cache layout,
 * reference fastkernel/src/fast_kernel.cpp:811-845).
 */
int mlk_bind_module(const char* mlk_kernel_json);

/*
 * The artifact entry point resolved by dlsym(handle, "mlk_kernel")
 * (reference backends/cpu/src/backend_driver.cpp:418-436) and invoked by
 * LoadedKernel::run (backend_driver.cpp:821-1050) in one of two forms:
 *   multi-dim:  int  mlk_kernel(const double* B0, const int64_t* B0_dims, ...,
 *                               const double* mlk_scalars, int64_t mlk_n_scalars)
 *   legacy 1-D: void mlk_kernel(const double* B0, ..., int64_t n,
 *                               const double* mlk_scalars, int64_t mlk_n_scalars)
 * (reference backends/cpu/include/mlk/backend/backend_driver.h:15-34).
 * Buffers are host f64 arrays in module table order (inputs, outputs).
 * Every argument of both forms is pointer-sized and of integer class in the
 * x86-64 System V calling convention, so this single definition with the
 * largest arity (8 pairs + scalars pair) receives the first k arguments of a
 * k-argument call exactly; arguments past the bound module's arity are
 * never read. The form is chosen from the bound module with the reference's
 * isMultiDimModule rule (reference backends/cpu/src/cpp_emitter.cpp:667-687).
 * Returns the status (the legacy caller ignores it; mlk_last_status()
 * reports it).
 */
int mlk_kernel(intptr_t a0, intptr_t a1, intptr_t a2, intptr_t a3,
               intptr_t a4, intptr_t a5, intptr_t a6, intptr_t a7,
               intptr_t a8, intptr_t a9, intptr_t a10, intptr_t a11,
               intptr_t a12, intptr_t a13, intptr_t a14, intptr_t a15,
               intptr_t a16, intptr_t a17);

/* Status of the last mlk_kernel call on this thread (the legacy form returns
 * void, reference backend_driver.h:27-30, so errors surface here). */
int mlk_last_status(void);

/* Message for the last failing call on this thread ("" when none). */
const char* mlkb_last_error(void);

/* Library version string; it also names the build target ("sm_100a"), which
 * the fastkernel artifact fingerprint must cover
 * (reference fastkernel/src/fast_kernel.cpp:727-763). */
const char* mlkb_version(void);

/* Number of CUDA devices visible to this process (0 when none). */
int mlkb_device_count(void);

/* Returns and clears the current device's sticky status word, which a kernel
 * sets when one of its bounded device-side waits gives up (MLKB_ERR_TIMEOUT);
 * 0 when clear. Synchronises with the device. */
int mlkb_take_device_error(void);

/* Launches a one-CTA kernel whose mbarrier wait can never complete; the
 * bounded wait used by every device-side spin in this library gives up after
 * limit_ns (at most 2 s) and records MLKB_ERR_TIMEOUT, which
 * mlkb_take_device_error() then returns. Exercises failure detection without
 * faulting or hanging the GPU. No reference counterpart: the reference never
 * ran on a device. */
int mlkb_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/* ======================================================================= */
/* 2. Module entry points                                                   */
/* ======================================================================= */

/* Parses and classifies an `mlk-kernel` JSON module. The classification is
 * the reference executor's dispatch (reference
 * runtime/src/execution/kernel_buffers.cpp:921-1085). */
int mlkb_module_create(const char* mlk_kernel_json, mlkb_module** out);
void mlkb_module_destroy(mlkb_module* module);
/* MLKB_KIND_* of a module, or a negative value for NULL. */
int mlkb_module_kind(const mlkb_module* module);
/* Number of bindable (input + output) buffers, in table order. */
int mlkb_module_num_buffers(const mlkb_module* module);

/* Names of the kernels mlkb_module_run_dev launches for this module with
 * these buffer dtypes, comma separated, into buf (cap bytes), e.g.
 * "map_sin_dsin_f32" or "map_chain". Launches nothing. No reference
 * counterpart: it reports which of this library's kernels a module reaches
 * (the reference's emitter has one code path per module). */
int mlkb_module_plan(const mlkb_module* module, const int32_t* dtypes, int32_t n_bufs,
                     char* buf, int64_t cap);

/*
 * Runs the module over DEVICE buffers on `device` / `stream`.
 *   bufs[i], dtypes[i]  buffer i of the module table (inputs then outputs),
 *                       MLKB_F16 / MLKB_F32 / MLKB_F64
 *   n                   element count for dynamic loop bounds
 *                       (the reference's KernelBufferBindings::elements,
 *                       runtime/include/mlk/runtime/execution.h:118-130)
 *   scalars             runtime scalar table (ScalarParam operands)
 * Semantics follow executeKernelOnBuffers (kernel_buffers.cpp:839-1106):
 * MatMul ACCUMULATES into C (C += A*B).
 */
int mlkb_module_run_dev(const mlkb_module* module, void* const* bufs,
                        const int32_t* dtypes, int32_t n_bufs, int64_t n,
                        const double* scalars, int64_t n_scalars,
                        int32_t device, void* stream);

/*
 * Runs the module over HOST buffers: stages inputs to the device(s), runs,
 * copies outputs back, synchronously. n_gpus == 1 runs on the calling
 * thread's current device; n_gpus > 1 splits the work into contiguous
 * element / row shards over devices 0..n_gpus-1 (n_gpus <= 0: all visible
 * devices), one host thread and stream per device. Page-locked (pinned)
 * host buffers are copied straight to and from the device, overlapped with
 * compute. Pageable buffers (ordinary malloc / std::vector memory, as the
 * reference's LoadedKernel::run passes) are staged by the library: a
 * multi-threaded CPU copy into pinned buffers it keeps per device (grow-only,
 * about 16 MB per buffer and pipeline step for maps, 64 MB for whole-buffer
 * kinds), then the DMA; for maps the CPU copies of one step overlap the
 * device work of the next. The same staging serves mlk_kernel.
 * Kinds: fused maps (element shards), Softmax / ReduceSum / MatMul (row
 * shards, MatMul's B on every device) and the scaled-scores composite (row
 * shards of Q, S, Sc and Y, Kt on every device). A module with nothing to
 * run (every loop range empty) returns MLKB_OK; a kind this path cannot run
 * returns MLKB_ERR_UNSUPPORTED, never MLKB_OK.
 */
int mlkb_module_run_host(const mlkb_module* module, void* const* bufs,
                         const int32_t* dtypes, int32_t n_bufs, int64_t n,
                         const double* scalars, int64_t n_scalars,
                         int32_t n_gpus);

/* Flags of mlkb_module_run_sharded: assemble every output on device 0; with
 * it, move the shards by NCCL even where peer stores could (below). */
#define MLKB_ASSEMBLE_DEVICE0 1u
#define MLKB_ASSEMBLE_VIA_NCCL 2u

/*
 * The typed multi-GPU entry: runs the module sharded over devices
 * 0..n_gpus-1 (n_gpus <= 0: all visible devices) in contiguous element / row
 * / batch shards, inputs read from HOST buffers.
 *   flags 0                       outputs are host buffers: mlkb_module_run_host.
 *   flags MLKB_ASSEMBLE_DEVICE0   output buffers are DEVICE memory on device 0.
 *                                 Maps whose outputs no root reads, Softmax,
 *                                 ReduceSum and the fused scaled-scores
 *                                 composite, on devices with peer access to
 *                                 device 0: each shard's kernel stores its
 *                                 part of every output straight into device
 *                                 0's buffer over NVLink, so computing and
 *                                 assembling are one pass (no kernel loads a
 *                                 peer's memory). Otherwise (MatMul, which
 *                                 reads C back), or with
 *                                 MLKB_ASSEMBLE_VIA_NCCL as well, every
 *                                 shard's part is assembled by grouped NCCL
 *                                 send/recv, and outputs a step reads back
 *                                 (MatMul's C, the composite's S, map outputs
 *                                 written in part) are first sent from device
 *                                 0 to the shards the same way.
 * NCCL is loaded on first use (libnccl.so.2, or the library named by the
 * environment variable MLKB_NCCL_LIB) and one communicator per device is kept
 * for the process; loading, communicator creation or a transfer failing
 * returns MLKB_ERR_NCCL. Synchronous. No reference counterpart: the reference's
 * artifact ABI is single-device (reference docs/kernel_abi.md:20-41); this is
 * the typed extension its driver would bind for n GPUs with a gather flag.
 */
int mlkb_module_run_sharded(const mlkb_module* module, void* const* bufs,
                            const int32_t* dtypes, int32_t n_bufs, int64_t n,
                            const double* scalars, int64_t n_scalars, int32_t n_gpus,
                            uint32_t flags);

/* ======================================================================= */
/* 3. Direct kernel entry points (device pointers, asynchronous on stream)  */
/* ======================================================================= */

/* Fused map y = sin(x*x + 3x) over n f32 elements. Arithmetic follows the
 * reference chain Mul, Mul, Add, Sin evaluated in f64
 * (reference kernel_buffers.cpp:130-178); result rounded once to f32. */
int mlkb_map_sin_f32(const float* x, float* y, int64_t n, void* stream);

/* Map plus its calculus-pass derivative in one pass:
 * y = sin(x*x + 3x), dy = cos(x*x + 3x) * (2x + 3). */
int mlkb_map_sin_dsin_f32(const float* x, float* y, float* dy, int64_t n,
                          void* stream);

/* Generic fused chain out[i] = chain(a[i], b[i], scalars) for any chain of
 * scalar-realisable ops (reference ExprEvaluator, kernel_buffers.cpp:106-178).
 * elem_dtype MLKB_F32 or MLKB_F64 for a, b and out alike; b may be NULL when
 * the chain never reads ElemB. At most 64 expressions (the reference's
 * kMaxTempSlots); the scalar table may be any size, and a ScalarParam past
 * its end reads 0 as in the reference (kernel_buffers.cpp:114-117).
 * poly7_sin != 0 evaluates Sin with the reference's "poly7" family,
 * families::polySin (compiler/include/mlk/support/math_families.h:81-90),
 * bit-identical to it in f64; other ops keep the libm family
 * (kernel_buffers.cpp:42-51).
 * The first call for a chain STRUCTURE (ops, operand kinds and temp indices,
 * poly7, dtype, whether b is read) compiles a straight-line kernel for it
 * with NVRTC, in-process, and caches it; constants and scalars are kernel
 * parameters, so other values reuse it. Where NVRTC cannot be loaded
 * (MLKB_NVRTC_LIB names the library, default libnvrtc.so.12), or
 * compilation is off (mlkb_chain_compile), an interpreter kernel runs the
 * chain instead, with identical results. */
int mlkb_map_chain(const mlkb_expr* exprs, int32_t n_exprs, int32_t poly7_sin,
                   const void* a, const void* b, void* out, int32_t elem_dtype,
                   int64_t n, const double* scalars, int64_t n_scalars,
                   void* stream);

/* Run-time compilation of chains. mode 1 compiles chains on first use (the
 * default; MLKB_CHAIN_JIT=0 in the environment starts the process at 0),
 * 0 runs every chain on the interpreter, any other value changes nothing.
 * With MLKB_CACHE_DIR set, compiled chains are also stored in that directory
 * and later processes load them instead of compiling (nothing is written
 * unless it is set; a stored file is used only when its recorded source
 * equals the one wanted).
 * Returns 1 when chains will be compiled (mode 1 and NVRTC loadable), else 0;
 * *compiled and *launched (either may be NULL) receive how many chain
 * kernels this process has compiled and launched. No counterpart in the
 * reference (its chains are compiled by an out-of-process nvcc). */
int32_t mlkb_chain_compile(int32_t mode, int64_t* compiled, int64_t* launched);

/* Compiles and caches the kernel mlkb_map_chain would use for this chain
 * structure without launching anything (no GPU needed): MLKB_OK, or
 * MLKB_ERR_UNSUPPORTED with the NVRTC log's head in mlkb_last_error() when
 * it cannot be compiled (the interpreter then runs the chain). has_b: the
 * call will pass a b buffer. */
int mlkb_chain_build(const mlkb_expr* exprs, int32_t n_exprs, int32_t poly7_sin,
                     int32_t elem_dtype, int32_t has_b);

/* Row softmax Y[m,:] = softmax(X[m,:]) over a row-major [rows, cols] matrix
 * (reference execSoftmaxCall, kernel_buffers.cpp:290-340). */
int mlkb_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols,
                     void* stream);
int mlkb_softmax_f64(const double* x, double* y, int64_t rows, int64_t cols,
                     void* stream);

/*
 * The row softmax of mlkb_softmax_f32 for callers that cannot allocate device
 * memory: a process whose device memory is all handed out by its own pool
 * allocator, a plugin host whose execute callback must not call cudaMalloc,
 * or code that may not pay the device-wide synchronisation cudaMalloc implies.
 * mlkb_softmax_f32 obtains its kernel's status word with cudaMalloc on its
 * first call on each device; this entry keeps that scratch in a fixed 256-byte
 * array of the library instead (each GPU that loads the library holds one
 * until the process exits) and calls no cudaMalloc, cudaFree or other
 * allocating routine. No counterpart in the reference (its emitted artifacts
 * allocate and free on every call).
 *   rows, cols   at most 8192 columns, a multiple of 4, x and y 16-byte
 *                aligned; anything else returns MLKB_ERR_INVALID (use
 *                mlkb_softmax_f32 for it). The kernel needs 4 bytes of the
 *                scratch whatever the shape.
 *   wait         0: returns once the kernel is queued on `stream`, and a
 *                bounded device wait that gives up is not reported; nonzero:
 *                synchronises `stream` and returns the kernel's device status
 *                (MLKB_ERR_TIMEOUT if one of its waits gave up).
 * The first call on each device looks up the scratch's device address with
 * that device current (no allocation); make that first call before any
 * stream capture. All calls on a device share the one array: each call clears
 * the status word before its kernel, so calls that overlap on the GPU (other
 * streams or threads) race on it.
 */
int mlkb_softmax_f32_noalloc(const float* x, float* y, int64_t rows, int64_t cols,
                             int32_t wait, void* stream);

/* Row sums Y[m] = sum_k X[m,k] (reference execReduceSumCall,
 * kernel_buffers.cpp:237-277). */
int mlkb_reducesum_f32(const float* x, float* y, int64_t rows, int64_t cols,
                       void* stream);
int mlkb_reducesum_f64(const double* x, double* y, int64_t rows, int64_t cols,
                       void* stream);

/* C[M,N] (+)= A[M,K] * B[K,N], all row-major (reference gemmRowBlock,
 * kernel_buffers.cpp:406-432; accumulate != 0 gives the reference's C += A*B).
 * f16 inputs, f32 accumulation and output, on the tcgen05 tensor cores. */
int mlkb_gemm_f16_f32(const void* a, const void* b, float* c, int64_t m,
                      int64_t n, int64_t k, int32_t accumulate, void* stream);
/* Same contraction with f32 inputs, f32 FMA accumulation (no TF32). */
int mlkb_gemm_f32(const float* a, const float* b, float* c, int64_t m,
                  int64_t n, int64_t k, int32_t accumulate, void* stream);
/* Same contraction in f64 with the reference's per-element order
 * (ascending k, zero-a terms skipped, no contraction into FMA). */
int mlkb_gemm_f64(const double* a, const double* b, double* c, int64_t m,
                  int64_t n, int64_t k, int32_t accumulate, void* stream);

/* Batched Y[b] = softmax_rows(scale * Q[b] * K[b]^T), Q and K f16
 * [batch, s, d] row-major, Y f32 [batch, s, s]: the reference composite
 * Call(MatMul) -> scale map -> Call(Softmax) (kernel_buffers.cpp:1001-1085,
 * :342-402, :290-340) fused into one kernel. */
int mlkb_qk_softmax_f16(const void* q, const void* k, float* y, int64_t batch,
                        int64_t s, int64_t d, double scale, void* stream);

/* The same composite with K given as the reference's MatMul B operand:
 * Q f16 [batch, m, d], Kt f16 [batch, d, s] ([K, N] row-major per batch,
 * reference kernel_buffers.cpp:1030-1036), Y f32 [batch, m, s]. Kt is read
 * in place as the tensor cores' MN-major operand; nothing is transposed. */
int mlkb_qk_softmax_kt_f16(const void* q, const void* kt, float* y, int64_t batch,
                           int64_t m, int64_t s, int64_t d, double scale, void* stream);

/* Deterministic synthetic inputs, generated on the device: a counter-based
 * SplitMix64 stream of (seed, stream_id, element index).
 *   dist 0: uniform  lo + (hi-lo) * k * 2^-24, k = top 24 bits
 *   dist 1: normal   Box-Muller, mean lo, standard deviation hi */
int mlkb_fill_f32(float* out, int64_t n, uint64_t seed, uint32_t stream_id,
                  int32_t dist, double lo, double hi, void* stream);
int mlkb_fill_f16(void* out, int64_t n, uint64_t seed, uint32_t stream_id,
                  int32_t dist, double lo, double hi, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLKB200_H */
