/*
 * ggemm_vark.h - C ABI of the B200 (sm_100a) variable-K grouped FP8 GEMM.
 *
 * The path computed by every entry point, for each group (expert) g in [0, G):
 *
 *     C[g][i][j] = bf16_rne( sL * sR * sum_{t in [off_g, off_{g+1})} LHS[t][i] * RHS[t][j] )
 *
 * LHS is [M_total, OUT_M] float8 e4m3fn, RHS is [M_total, OUT_N] float8 e5m2, both token-major
 * (row t holds one token). C is [G, OUT_M, OUT_N] bf16. Products are accumulated in fp32.
 * group_offs is a device int64 array of G+1 prefix sums (off_0 = 0, off_G = M_total); a group
 * with off_{g+1} == off_g is empty and its C[g] is overwritten with zeros.
 *
 * Reference interface replaced: the 14 runtime kernel arguments of
 * `_grouped_variable_k_gemm_kernel` (ggemm-asm README.md:88-95, launcher.cpp:16-33,
 * bench.py:364-413): LHS, RHS, C, LHS_scale, RHS_scale, group_offs, G, OUT_M, OUT_N,
 * stride_lhs_m, stride_rhs_m, stride_cg, stride_cm, stride_cn.  The reference's two trailing
 * Triton scratch pointers (global_scratch, profile_scratch; always NULL there, bench.py:383-384)
 * are dropped; the stream the reference passes as NULL (bench.py:343) is explicit here.
 *
 * Conventions shared by all entry points:
 *  - every buffer is device memory owned by the caller; strides are in ELEMENTS (int32),
 *    exactly as the reference packs them (bench.py:370-374);
 *  - lhs_scale / rhs_scale point to device fp32 values;
 *  - calls are asynchronous on `stream` (a cudaStream_t passed as void*, NULL = legacy default
 *    stream); no host synchronisation and no device-to-host copy of group_offs happens;
 *  - C is always fully overwritten (no accumulate-into-C);
 *  - the return value is 0 on success or a GGEMM_VARK_E* code (nothing is launched on error);
 *  - entry points may be called from several host threads on distinct streams. A call given no
 *    status block records its device-side status in the library's one block for the current
 *    device, which every such call on that device shares: a bit found there cannot be traced to
 *    one call. Give each stream its own block (the `status` argument of the _ex entry points)
 *    to keep them apart. ggemm_vark_read_status synchronises the whole device;
 *    ggemm_vark_read_status_stream waits for one stream only.
 */
#ifndef GGEMM_VARK_H_
#define GGEMM_VARK_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GGEMM_VARK_API __attribute__((visibility("default")))
#else
#define GGEMM_VARK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------ */
#define GGEMM_VARK_OK                 0
#define GGEMM_VARK_EINVAL_PTR         1  /* a required pointer is NULL */
#define GGEMM_VARK_EINVAL_SHAPE       2  /* G <= 0, OUT_M <= 0 or OUT_N <= 0 */
#define GGEMM_VARK_EINVAL_STRIDE      3  /* a stride is not positive or makes rows overlap */
#define GGEMM_VARK_EINVAL_ARG         4  /* another argument is out of its documented range */
#define GGEMM_VARK_ENO_DEVICE         5  /* no CUDA device, or the current device is not sm_100 */
#define GGEMM_VARK_ECUDA              6  /* a CUDA runtime/driver call failed */
#define GGEMM_VARK_ELAYOUT            7  /* layout not expressible for the forced tensor-core path */
#define GGEMM_VARK_ETOO_LARGE         8  /* a size exceeds the documented maximum */

/* ---- device-side status bits (read with ggemm_vark_read_status) -------------------------- */
#define GGEMM_VARK_DEV_BAD_OFFS   0x1u   /* group_offs not monotone, negative, or past m_total
                                            (past group_offs[G] when m_total is not given) */
#define GGEMM_VARK_DEV_TIMEOUT    0x2u   /* a pipeline wait exceeded its limit; the CTA stopped */

/* ---- status block layout (32-bit words; a caller's block is >= 256 bytes, 16-byte aligned) -
 *  word 0  GGEMM_VARK_DEV_* bits, or-ed by every launch
 *  word 1  where a wait expired (GGEMM_VARK_DEV_TIMEOUT), for diagnosis
 *  word 3  the failure-detection test hook (GGEMM_VARK_TEST_STALL_MAGIC); never written
 *  word 4  wgrad: the end (exclusive) of the highest LHS token row any load of the tensor-core
 *          kernels could read, maximum over launches; fixed-K GEMM: the same for A's rows
 *  word 5  wgrad: the same for RHS
 * A load past M_total when m_total is given is clipped by the hardware without reading memory,
 * so words 4 and 5 never exceed m_total; without m_total they never exceed group_offs[G]. */
#define GGEMM_VARK_STATUS_WORD_BITS      0
#define GGEMM_VARK_STATUS_WORD_SITE      1
#define GGEMM_VARK_STATUS_WORD_LHS_ROWS  4
#define GGEMM_VARK_STATUS_WORD_RHS_ROWS  5

/* ---- test hook for failure detection ------------------------------------------------------
 * If word 3 of a caller-provided status block (ggemm_vark_fp8_wgrad_ex's `status`) holds this
 * value, the tensor-core kernels withhold their first pipeline stage, so the MMA warp's bounded
 * wait expires after `timeout_ns`: every CTA stops, and the call reports GGEMM_VARK_DEV_TIMEOUT
 * in word 0 (C is left incomplete). Nothing faults or hangs; the context stays usable. Only the
 * failure-detection tests set it. */
#define GGEMM_VARK_TEST_STALL_MAGIC 0x5374616cu

/* ---- path selection flags for ggemm_vark_fp8_wgrad_ex ------------------------------------ */
#define GGEMM_VARK_PATH_AUTO      0      /* tensor-core path when the layout allows, else SIMT */
#define GGEMM_VARK_PATH_TCGEN05   1      /* force the tcgen05 CTA-pair path (ELAYOUT if not expressible) */
#define GGEMM_VARK_PATH_SIMT      2      /* force the CUDA-core path (any strides) */
#define GGEMM_VARK_PATH_TCGEN05_1SM 3    /* force the single-CTA tcgen05 path (same layout rules) */

/*
 * ggemm_vark_fp8_wgrad - the drop-in for `_grouped_variable_k_gemm_kernel`.
 *
 * Replaces the launch in bench.py:364-413 (prepare_variable_k_args / launch_variable_k_kernel)
 * and launcher.cpp:123-168 (KernelArgs + hipModuleLaunchKernel); argument order and meaning are
 * the reference's (README.md:88-95). Per-tensor scales (one fp32 each). The token count
 * M_total is not an argument, exactly as in the reference: group_offs[G] is taken as M_total.
 * No load reads a token row at or past it (the kernel reads group_offs[G] on the device and
 * moves the boxes that would cross it), so LHS and RHS allocations of exactly group_offs[G] rows
 * are safe; offsets past group_offs[G] are reported (GGEMM_VARK_DEV_BAD_OFFS) and their groups
 * written as zeros. The first call on a device makes the library's one allocation for that
 * device (cudaMalloc of the 4 KiB status block); make the first call before any stream capture.
 */
GGEMM_VARK_API int ggemm_vark_fp8_wgrad(const void* lhs, const void* rhs, void* c,
                         const float* lhs_scale, const float* rhs_scale,
                         const int64_t* group_offs,
                         int32_t G, int32_t OUT_M, int32_t OUT_N,
                         int32_t stride_lhs_m, int32_t stride_rhs_m,
                         int32_t stride_cg, int32_t stride_cm, int32_t stride_cn,
                         void* stream);

/*
 * ggemm_vark_fp8_wgrad_ex - the same computation with the extensions the reference ABI lacks.
 *
 *  m_total       rows allocated in LHS/RHS, or -1 if unknown. When known, group offsets past
 *                m_total are reported (GGEMM_VARK_DEV_BAD_OFFS) and such groups are written
 *                as zeros instead of being read. With m_total == 0, lhs and rhs may be NULL
 *                (every group is empty and C is zeroed). Unknown (-1): group_offs[G] takes
 *                m_total's place, as in ggemm_vark_fp8_wgrad, and no load reaches past it.
 *  scale_stride  0: lhs_scale/rhs_scale are single values (the reference's tensorwise scales,
 *                bench.py:266-267); 1: they are arrays of G per-group values.
 *  path          GGEMM_VARK_PATH_* selector.
 *  status        device pointer to a 256-byte, 16-byte aligned status block (see
 *                ggemm_vark_read_status), or NULL to use the library's per-device block.
 *  timeout_ns    limit on any single pipeline wait inside the kernel (0 = default, 2 s).
 */
GGEMM_VARK_API int ggemm_vark_fp8_wgrad_ex(const void* lhs, const void* rhs, void* c,
                            const float* lhs_scale, const float* rhs_scale,
                            const int64_t* group_offs,
                            int32_t G, int32_t OUT_M, int32_t OUT_N,
                            int32_t stride_lhs_m, int32_t stride_rhs_m,
                            int32_t stride_cg, int32_t stride_cm, int32_t stride_cn,
                            int64_t m_total, int32_t scale_stride, int32_t path,
                            void* status, uint64_t timeout_ns,
                            void* stream);

/*
 * ggemm_vark_read_status - synchronously read (and optionally clear) the device status bits
 * (GGEMM_VARK_DEV_*) written by earlier launches. `status` is the block given to _ex, or NULL
 * for the current device's library block. Synchronises the device. Returns a GGEMM_VARK_E code.
 */
GGEMM_VARK_API int ggemm_vark_read_status(void* status, int clear, uint32_t* bits_out);

/*
 * ggemm_vark_read_status_stream - read the first `nwords` (1..8) words of a status block in
 * the order of `stream`: the copy is queued behind the stream's earlier work and only that
 * stream is waited for, so other streams keep running. `clear` then queues, on the same stream,
 * the zeroing of words 0, 1, 4 and 5. `status` NULL = the current device's library block.
 */
GGEMM_VARK_API int ggemm_vark_read_status_stream(void* status, int clear, uint32_t* words_out,
                                                 int32_t nwords, void* stream);

/*
 * ggemm_vark_device_bytes - device memory this library has allocated on `device`: 0 until the
 * first call of an entry point that uses the library's block there, then the 4 KiB status
 * block. The static array of ggemm_vark_fp8_wgrad_noalloc is not an allocation and is not
 * counted. Touches no device.
 */
GGEMM_VARK_API int ggemm_vark_device_bytes(int32_t device, uint64_t* bytes_out);

/* ggemm_vark_tc_supported - 1 if `path` AUTO would take the tcgen05 path for this layout. */
GGEMM_VARK_API int ggemm_vark_tc_supported(const void* lhs, const void* rhs, void* c,
                            int32_t OUT_M, int32_t OUT_N,
                            int32_t stride_lhs_m, int32_t stride_rhs_m,
                            int32_t stride_cg, int32_t stride_cm, int32_t stride_cn);

/*
 * ggemm_vark_fp8_wgrad_noalloc - the same computation for callers that must not let a library
 * allocate device memory. No counterpart in the reference: its kernel takes two scratch
 * pointers (always NULL there) and this library otherwise makes one cudaMalloc per device.
 *
 * Callers that cannot allocate: code running inside a framework-owned memory pool or arena
 * (every device byte must come from the pool), allocators with strict accounting, processes that
 * fixed their device footprint up front, and latency-critical paths that must not hit the
 * implicit synchronisation of cudaMalloc/cudaFree. This entry point runs the tensor-core (CTA
 * pair) kernel with its scratch - the status words - taken from a file-scope device array of
 * GGEMM_VARK_NOALLOC_SCRATCH_BYTES (4 KiB) that every GPU loading this library holds until the
 * process exits. It never calls cudaMalloc or cudaFree.
 *
 *  - Arguments as ggemm_vark_fp8_wgrad_ex (m_total -1 = unknown: loads stay below
 *    group_offs[G]); only tensor-core layouts are accepted (16-byte
 *    aligned bases and row pitches, stride_cn == 1, OUT_N a multiple of 8), anything else
 *    returns GGEMM_VARK_ELAYOUT.
 *  - `status`: a caller-owned 16-byte aligned device buffer of >= 256 bytes for the status
 *    words, or NULL to record them in the shared array (cleared at the start of every call, not
 *    readable). Only a caller-owned block lets the caller see a bad group_offs or an expired
 *    wait; waits are limited to 2 s.
 *  - lhs and rhs may be NULL when m_total == 0, as for ggemm_vark_fp8_wgrad_ex.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress) and
 *    sets kernel attributes; make that first call before any stream capture.
 *  - All calls on a device share the array and it keeps the last call's contents; calls that
 *    overlap on the GPU (different streams without ordering) race on its status words.
 */
#define GGEMM_VARK_NOALLOC_SCRATCH_BYTES 4096u
GGEMM_VARK_API int ggemm_vark_fp8_wgrad_noalloc(const void* lhs, const void* rhs, void* c,
                            const float* lhs_scale, const float* rhs_scale,
                            const int64_t* group_offs,
                            int32_t G, int32_t OUT_M, int32_t OUT_N,
                            int32_t stride_lhs_m, int32_t stride_rhs_m,
                            int32_t stride_cg, int32_t stride_cm, int32_t stride_cn,
                            int64_t m_total, int32_t scale_stride,
                            void* status, void* stream);

/*
 * ggemm_vark_grouped_fp8_fwd - the fixed-K grouped FP8 GEMM of the MoE forward and data-gradient
 * sites (the harness's "persistent" kernel type, ggemm-asm bench.py:154-181, launched with the
 * argument layout of bench.py:312-338; the reference ships no kernel for it, its harness runs
 * Primus-Turbo's grouped_gemm_fp8_tensorwise_triton_kernel, bench.py:241-260):
 *
 *     C[t, n] = a_scale * b_scale * sum_k A[t, k] * B[g, n, k]   for off_g <= t < off_{g+1}
 *
 *  A          [rows, K] float8 e4m3fn (this entry point) with row pitch stride_am (elements =
 *             bytes); K contiguous
 *  B          [G, N, K] float8 e4m3fn ("trans_b"): expert stride stride_bg, row stride stride_bn
 *  C          [rows, N] bf16, row pitch stride_cm, stride_cn == 1; rows of every expert are
 *             overwritten, other rows are not touched
 *  scales     device fp32 scalars; group_offs device int64 [G + 1]
 * Tensor-core layout rules: 16-byte aligned bases; stride_am, stride_bn, stride_bg and
 * 2 * stride_cm multiples of 16; stride_cn == 1 (GGEMM_VARK_ELAYOUT otherwise). Like the
 * 14-argument wgrad entry point it takes group_offs[G] as the row count of A and C: no load or
 * store touches a row at or past it, and offsets past it are reported and their expert skipped.
 */
GGEMM_VARK_API int ggemm_vark_grouped_fp8_fwd(const void* a, const void* b, void* c,
                            const float* a_scale, const float* b_scale,
                            const int64_t* group_offs, int32_t G, int32_t N, int32_t K,
                            int32_t stride_am, int32_t stride_bg, int32_t stride_bn,
                            int32_t stride_cm, int32_t stride_cn, void* stream);

/*
 * ggemm_vark_grouped_fp8_fwd_ex - the same with the A format and B layout selectable and the
 * extensions of ggemm_vark_fp8_wgrad_ex:
 *  m_total       rows allocated in A and C, or -1; offsets past it are reported and their
 *                expert skipped; 0 allows NULL a, b, c
 *  a_fmt         0: e4m3fn (forward sites), 1: e5m2 (data-gradient sites); B stays e4m3fn
 *  scale_stride  0: a_scale and b_scale are single values; 1: both hold G per-expert values
 *  b_layout      0: B [G, N, K] with K contiguous ("trans_b", the harness's layout): element
 *                (g, n, k) at b + g*stride_bg + n*stride_bn + k; 1: B [G, K, N] with N
 *                contiguous: element (g, k, n) at b + g*stride_bg + k*stride_bn + n
 *  status, timeout_ns  as ggemm_vark_fp8_wgrad_ex
 */
GGEMM_VARK_API int ggemm_vark_grouped_fp8_fwd_ex(const void* a, const void* b, void* c,
                            const float* a_scale, const float* b_scale,
                            const int64_t* group_offs, int32_t G, int32_t N, int32_t K,
                            int32_t stride_am, int32_t stride_bg, int32_t stride_bn,
                            int32_t stride_cm, int32_t stride_cn, int64_t m_total,
                            int32_t a_fmt, int32_t scale_stride, int32_t b_layout,
                            void* status, uint64_t timeout_ns, void* stream);

/*
 * ggemm_vark_quantize_fp8 - per-expert (or per-tensor) amax scaling and FP8 quantisation of a
 * token-major bf16 operand: the producer step in front of ggemm_vark_fp8_wgrad (x -> e4m3 LHS,
 * dy -> e5m2 RHS). No kernel counterpart in the reference: its harness makes the fp8 operands on
 * the host side (bench.py:221-223, scales fixed by bench.py:266-267).
 *
 *  x          bf16 [rows, F], row pitch stride_x elements (2-byte aligned)
 *  q          fp8 [rows, F], row pitch stride_q bytes; fmt 0: e4m3fn (FMAX 448), 1: e5m2 (57344)
 *  scales     fp32 [G] (per_group = 1) or [1] (per_group = 0), written by the call
 *  group_offs device int64 [G + 1]; unit g is rows [off_g, off_{g+1}); per tensor, one unit of
 *             rows [off_0, off_G)
 *  m_total    rows allocated in x and q, or -1 if unknown; offsets past it are reported
 *             (GGEMM_VARK_DEV_BAD_OFFS) and their unit is left unwritten with scale 1.0. With
 *             m_total == 0, x and q may be NULL.
 *  workspace  device buffer of ggemm_vark_quantize_workspace_bytes(G) bytes, 16-byte aligned;
 *             the call clears it on `stream` before the kernel runs (no allocation here)
 *  status     16-byte aligned status block, or NULL for the library's per-device block
 *  timeout_ns limit on any single wait of one CTA for the others (0 = default, 2 s)
 *
 * Per unit: s = amax/FMAX (fp32 IEEE division; 1.0 for an empty unit or amax == 0; NaN if the
 * unit holds a NaN), q = fp8(x / s) rounded to nearest even and saturated to +-FMAX. Rows
 * outside every unit are not written. The kernel is a cooperative launch of one co-resident
 * grid; calls on different streams must not share a workspace.
 */
GGEMM_VARK_API size_t ggemm_vark_quantize_workspace_bytes(int32_t G);
GGEMM_VARK_API int ggemm_vark_quantize_fp8(const void* x, void* q, float* scales,
                            const int64_t* group_offs, int32_t G, int32_t F,
                            int32_t stride_x, int32_t stride_q, int32_t fmt, int32_t per_group,
                            int64_t m_total, void* workspace, void* status,
                            uint64_t timeout_ns, void* stream);

/* ggemm_vark_strerror - static description of a GGEMM_VARK_E* code. */
GGEMM_VARK_API const char* ggemm_vark_strerror(int code);

/* ggemm_vark_last_cuda_error - the CUDA error number behind the last GGEMM_VARK_ECUDA on this
 * host thread (0 if none). */
GGEMM_VARK_API int ggemm_vark_last_cuda_error(void);

/* ggemm_vark_version - library version, e.g. 0x000100 for 0.1.0. */
GGEMM_VARK_API int ggemm_vark_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GGEMM_VARK_H_ */
