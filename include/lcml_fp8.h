/*
 * lcml_fp8.h — C ABI of the B200 (sm_100a) FP8 e4m3 operator path.
 *
 * A thin shim over hand-written CUDA kernels. Every entry point:
 *   - takes device pointers, 64-bit sizes and a CUDA stream (lcml_stream_t is
 *     layout-identical to cudaStream_t; NULL is the legacy default stream);
 *   - enqueues work asynchronously and never synchronises the stream;
 *   - never allocates device memory on the hot path (callers pass workspace);
 *   - returns an lcml_status; a nonzero status leaves a message for
 *     lcml_last_error() (thread-local). No exceptions cross the ABI and no
 *     kernel traps: a kernel that gives up on a bounded wait records a code
 *     readable with lcml_device_error().
 *
 * The operators of the ONNX graph executor (include/lcml_onnx.h) call these
 * functions from Operator::forward. Reference interfaces each entry point
 * stands in for are cited beside it (paths inside the LuisaML tree).
 */
#ifndef LCML_FP8_H
#define LCML_FP8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *lcml_stream_t;
typedef struct CUevent_st *lcml_event_t;

/* Status codes. */
typedef enum lcml_status {
    LCML_OK = 0,
    LCML_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, misaligned pointer */
    LCML_ERR_UNSUPPORTED = 2,      /* a valid request this build does not implement */
    LCML_ERR_CUDA = 3,             /* a CUDA runtime call failed; message has the detail */
    LCML_ERR_NO_DEVICE = 4,        /* no sm_100 device visible */
    LCML_ERR_DEVICE_TIMEOUT = 5    /* a kernel abandoned a bounded wait (lcml_device_error) */
} lcml_status;

/* Element types: the ONNX TensorProto.DataType numbers (include/onnx/onnx.h:31-60). */
typedef enum lcml_dtype {
    LCML_DTYPE_FLOAT = 1,
    LCML_DTYPE_FLOAT16 = 10,
    LCML_DTYPE_BFLOAT16 = 16,
    LCML_DTYPE_FLOAT8E4M3FN = 17,
    LCML_DTYPE_FLOAT8E5M2 = 19,
    LCML_DTYPE_FLOAT4E2M1 = 23  /* two codes per byte, element 2i in the low nibble of byte i */
} lcml_dtype;

/* Scale layouts. TENSOR: one fp32 scale. AXIS: one per index of the quantized
 * axis. For 2-D GEMM operands ROW ([M] for A) and COL ([N] for B) are AXIS
 * along dim 0 and the N dimension respectively. */
typedef enum lcml_scale_mode {
    LCML_SCALE_TENSOR = 0,
    LCML_SCALE_AXIS = 1,
    LCML_SCALE_ROW = 1,
    LCML_SCALE_COL = 2
} lcml_scale_mode;

/* GEMM epilogues (the activation nodes fused behind Gemm/MatMul/Conv). */
typedef enum lcml_epilogue {
    LCML_EPI_NONE = 0,
    LCML_EPI_RELU = 1,     /* Relu, src/onnx/operators/unary.cpp:85 */
    LCML_EPI_SILU_MUL = 2  /* SiLU(gate) * up: Sigmoid+Mul+Mul (unary.cpp:86-87, binary.cpp:347).
                              B holds gate/up rows interleaved in groups of 128:
                              [gate 0..127; up 0..127; gate 128..255; up 128..255; ...],
                              Y has N/2 columns. */
} lcml_epilogue;

/* Library / device state. */
const char *lcml_last_error(void);
int lcml_abi_version(void);
/* 0 when an sm_100 device is current; LCML_ERR_NO_DEVICE otherwise. */
int lcml_device_check(void);
/* Reads and clears the device error word (synchronises the device). *code = 0: none. */
int lcml_device_error(int *code);
/* Number of kernels this library has launched in this process (all streams). */
uint64_t lcml_launch_count(void);

/* CUDA IPC for the fused all-gather: export a buffer allocated with
 * lcml_device_alloc as an opaque handle (LCML_IPC_HANDLE_BYTES), map a peer
 * process's handle into this process, and unmap it. */
#define LCML_IPC_HANDLE_BYTES 64
int lcml_ipc_get_handle(void *device_ptr, void *handle_out);
int lcml_ipc_open(const void *handle, void **device_ptr);
int lcml_ipc_close(void *device_ptr);
/* Enables peer access from the current device to `peer_device` (no-op if already on). */
int lcml_enable_peer_access(int peer_device);

/* Max of one float over the `world` ranks of a peer group, and a barrier
 * (value = NULL): one single-warp kernel per rank instead of a one-float
 * collective. No counterpart in the reference (single device). Rank `rank`
 * stores (epoch, *value) into its slot of every rank's slot array with one
 * 64-bit release store over NVLink, then waits until every slot of its own
 * array carries `epoch` and writes the max of the ranks' values to *out.
 * slots: this rank's array of LCML_PEER_SLOTS_BYTES, zeroed once before the
 * first call and mapped into every other rank (lcml_ipc_get_handle /
 * lcml_ipc_open); peer_slots: device array of the other ranks' mapped
 * arrays in rank order (world - 1 pointers, this rank skipped). Every rank
 * calls it with the same epoch sequence 1, 2, 3, ... (never 0). The wait is
 * bounded by timeout_us; a rank that gives up leaves *out unchanged and
 * records device error 5 (lcml_device_error). The stream's earlier peer
 * stores are ordered before this rank's slot store. world <= 32. */
#define LCML_PEER_SLOTS_BYTES 512
int lcml_peer_exchange_max(const float *value, float *out, uint64_t *slots, uint64_t *const *peer_slots, int rank,
                           int world, uint32_t epoch, uint32_t timeout_us, lcml_stream_t stream);

/* Device memory and copies for hosts that have no CUDA runtime of their own
 * (the C++ executor allocates intermediates once, at prepare time, through
 * these; the reference gets its buffers from LuisaCompute's Device).
 * kind: 1 host->device, 2 device->host, 3 device->device. */
int lcml_device_alloc(size_t bytes, void **ptr);
int lcml_device_free(void *ptr);
int lcml_memcpy_async(void *dst, const void *src, size_t bytes, int kind, lcml_stream_t stream);
int lcml_memset_async(void *dst, int value, size_t bytes, lcml_stream_t stream);
int lcml_stream_synchronize(lcml_stream_t stream);

/* Streams and events for hosts without a CUDA runtime of their own (the
 * executor's host-staged inputs copy on a second stream; the reference has
 * LuisaCompute's Stream / Event). lcml_stream_create makes a non-blocking
 * stream; events carry no timing. */
int lcml_stream_create(lcml_stream_t *stream);
int lcml_stream_destroy(lcml_stream_t stream);
int lcml_event_create(lcml_event_t *event);
int lcml_event_destroy(lcml_event_t event);
int lcml_event_record(lcml_event_t event, lcml_stream_t stream);
int lcml_stream_wait_event(lcml_stream_t stream, lcml_event_t event);

/*
 * QuantizeLinear to float8e4m3fn, zero point 0, saturate = 1 (ONNX opset 19+):
 *   y[i] = e4m3(x[i] / s), x / s an IEEE fp32 divide, e4m3() bit-identical to
 *   FP8E4M3FN::from_float (include/onnx/fp_quantized.h:149-223).
 * The reference registers no QuantizeLinear (its loader asserts at
 * src/onnx/onnx.cpp:228-229); its FP8 conversion is Cast (src/onnx/operators/cast.cpp:63-67).
 * x (fp32) is viewed as [outer, axis_len, inner]; TENSOR uses scale[0], AXIS
 * uses scale[(i / inner) % axis_len].
 */
int lcml_fp8_quantize(const float *x, int64_t outer, int64_t axis_len, int64_t inner, const float *scale,
                      int scale_mode, uint8_t *y, lcml_stream_t stream);

/* Same, with the scale derived on the device from a per-axis amax:
 * s[a] = amax[a] / 448 (1 when amax is 0); s is also written to scale_out
 * when not NULL. Used after a GEMM epilogue that produced row maxima. */
int lcml_fp8_quantize_from_amax(const float *x, int64_t outer, int64_t axis_len, int64_t inner,
                                const float *amax, float *scale_out, uint8_t *y, lcml_stream_t stream);

/* Dynamic per-row (per-token) quantization of x [rows, cols] (row stride ldx
 * elements): s[r] = max|x[r,:]| / 448 (1 for an all-zero row; NaN ignored),
 * y[r,c] = e4m3(x[r,c] / s[r]). The Abs -> ReduceMax -> Div -> QuantizeLinear
 * chain (unary.cpp:110, reduce.cpp:431, binary.cpp:350) as one pass. */
int lcml_fp8_quantize_rows_dynamic(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *scale_out,
                                   uint8_t *y, lcml_stream_t stream);

/* max |x| over n fp32 values (NaN ignored) into *amax_out (device). */
int lcml_amax(const float *x, int64_t n, float *amax_out, lcml_stream_t stream);

/* Dynamic per-tensor quantization: s = max|x| / 448 (1 for an all-zero
 * tensor; NaN ignored), y = e4m3(x / s). workspace: caller-owned device
 * scratch of at least LCML_FP8_TENSOR_DYNAMIC_WORKSPACE_BYTES (per-block
 * partial maxima; its contents on entry do not matter). scale_out (device,
 * 1 float) receives s. Two kernels: the partial maxima front to back, then
 * the reduction and the quantization back to front, so the part of x still in
 * the L2 is read first. */
#define LCML_FP8_TENSOR_DYNAMIC_WORKSPACE_BYTES 4096
int lcml_fp8_quantize_tensor_dynamic(const float *x, int64_t n, float *scale_out, uint8_t *y, float *workspace,
                                     lcml_stream_t stream);

/* DequantizeLinear: y = to_float(q) * s (fp32 multiply), output fp32 or bf16.
 * to_float() is FP8E4M3FN::to_float (include/onnx/fp_quantized.h:226-249). */
int lcml_fp8_dequantize(const uint8_t *q, int64_t outer, int64_t axis_len, int64_t inner, const float *scale,
                        int scale_mode, void *y, int y_dtype, lcml_stream_t stream);

/* e4m3 matrix transpose: src [rows, cols] -> dst [cols, rows] (row-major).
 * Converts MatMul's [K,N] weights into the K-major layout the tensor-core
 * GEMM reads. */
int lcml_fp8_transpose(const uint8_t *src, int64_t rows, int64_t cols, uint8_t *dst, lcml_stream_t stream);

/*
 * Fused FP8 GEMM: the DequantizeLinear -> Gemm/MatMul -> (Relu | Sigmoid*Mul)
 * -> (QuantizeLinear) node group of a QDQ graph in one kernel.
 *   acc[m,n] = sum_k A[m,k] * B[k,n]   (e4m3 x e4m3, exact products, fp32 accumulate)
 *   v = acc * (alpha * sa * sb) + beta * C     sa: [1] or [M]; sb: [1] or [N]
 *   v = act(v)                                 (epilogue)
 *   Y = v (f32 / bf16) or e4m3(v / y_scale)
 * Stands in for Gemm::apply (src/onnx/operators/gemm.cpp:28-325) and MatMul
 * (src/onnx/operators/mat_mul.cpp:51-186) fed by DequantizeLinear, which the
 * reference cannot express (Gemm excludes FP8, gemm.cpp:11-16).
 */
typedef struct lcml_fp8_gemm_desc {
    int64_t M, N, K;
    const uint8_t *A; /* [M, K] e4m3, row stride lda bytes (K-major) */
    int64_t lda;
    const uint8_t *B; /* b_kmajor=1: [N, K], row stride ldb (Gemm transB=1)  */
    int64_t ldb;      /* b_kmajor=0: [K, N], row stride ldb (MatMul layout)   */
    int b_kmajor;
    const float *scale_a; /* device */
    int scale_a_mode;     /* LCML_SCALE_TENSOR or LCML_SCALE_ROW */
    const float *scale_b; /* device */
    int scale_b_mode;     /* LCML_SCALE_TENSOR or LCML_SCALE_COL */
    float alpha;
    float beta;
    const float *c_vec;   /* optional fp32 C broadcast: [N] (COL), [M] (ROW) or [1] (TENSOR) */
    int c_vec_mode;
    const void *c_mat;    /* optional full C [M, N] (e.g. the FFN residual), row stride ldc elements */
    int c_mat_dtype;      /* LCML_DTYPE_FLOAT, LCML_DTYPE_BFLOAT16 or LCML_DTYPE_FLOAT8E4M3FN (see c_mat_scale) */
    int64_t ldc;
    int epilogue;         /* lcml_epilogue */
    void *Y;              /* [M, N] (N/2 for SILU_MUL), row stride ldy elements */
    int y_dtype;          /* FLOAT, BFLOAT16 or FLOAT8E4M3FN */
    int64_t ldy;
    const float *y_scale; /* device, per-tensor output scale when y_dtype is e4m3 */
    float *row_amax;      /* optional device [M]: max |v| per row (atomic; zero it first) */
    /* Output placement for a column shard of a larger matrix, and the fused
     * all-gather of tensor-parallel GEMMs: every output element (row, col) is
     * stored at Y[row * ldy + y_col_offset + col] and at the same offset of
     * each of the y_num_peers buffers in y_peers (other GPUs' outputs mapped
     * with lcml_ipc_open), so the shard reaches every rank while the GEMM
     * runs. Zero-initialise these fields when unused. */
    int64_t y_col_offset;
    void *const *y_peers; /* device array of y_num_peers device pointers */
    int y_num_peers;
    const float *c_mat_scale; /* device [1]: DequantizeLinear scale of an e4m3 c_mat (a quantized residual) */
    /* Kernel choice, per call (0 = automatic; results agree up to the fp32
     * summation order). Bits 0-1: 1 single-CTA tiles, 2 CTA-pair tiles, 3
     * split-K wherever the tile count allows it (also M > 128); bit 2: plain
     * global stores instead of TMA stores. For cross-checking and tuning. */
    int variant;
} lcml_fp8_gemm_desc;

int lcml_fp8_gemm(const lcml_fp8_gemm_desc *desc, lcml_stream_t stream);

/*
 * Gemm (+ epilogue) followed by dynamic per-row QuantizeLinear of its output:
 * the Gemm -> [Sigmoid*Mul] -> Abs -> ReduceMax(axis=-1) -> Div(448) ->
 * QuantizeLinear chain that feeds the next FP8 Gemm (the FFN's h), as two
 * kernels. desc->Y (fp32, dense: ldy == output columns) receives the
 * unquantized output; the GEMM epilogue accumulates each row's max |v| into
 * `workspace`; then q[r, c] = e4m3(Y[r, c] / s[r]), s[r] = amax[r] / 448
 * (1 for an all-zero row), written to q (dense) and q_scale [M].
 * workspace: caller-owned device scratch of at least M floats; it is zeroed
 * here, so its contents on entry do not matter. desc->row_amax must be NULL.
 * Reference pieces: unary.cpp:110 (Abs), reduce.cpp:431 (ReduceMax),
 * binary.cpp:350 (Div), fp_quantized.h:149-223 (the e4m3 encoder).
 */
int lcml_fp8_gemm_rowquant(const lcml_fp8_gemm_desc *desc, uint8_t *q, float *q_scale, float *workspace,
                           lcml_stream_t stream);

/*
 * QuantizeLinear of an fp32 activation with a dynamic per-tensor scale
 * followed by the GEMM that consumes it (the DynamicQuantizeLinear /
 * Abs -> ReduceMax -> Div -> QuantizeLinear -> DequantizeLinear -> Gemm
 * chain of a decode step; no counterpart in the reference, which has no
 * QuantizeLinear): s = max|A| / 448 (1 for an all-zero A, NaN ignored),
 * aq = e4m3(A / s) bit-exact as lcml_fp8_quantize, then lcml_fp8_gemm on
 * (aq, s) with desc's B, scales, epilogue and output; desc->A, lda,
 * scale_a and scale_a_mode are ignored. a: [M, K] fp32, row stride lda
 * elements. scale_a_out receives s. For M <= 4 on the GEMV path (desc
 * variant 0, no peers, not SILU_MUL) it is one kernel: every CTA derives s
 * from all of A and quantizes A while staging it; aq may then be NULL
 * (written when given) and workspace is unused. Otherwise A must be dense
 * (lda == K) and it runs lcml_fp8_quantize_tensor_dynamic into aq (M*K
 * bytes) with workspace (LCML_FP8_TENSOR_DYNAMIC_WORKSPACE_BYTES), then the
 * GEMM.
 */
int lcml_fp8_gemm_quantize_a(const lcml_fp8_gemm_desc *desc, const float *a, int64_t lda, uint8_t *aq,
                             float *scale_a_out, float *workspace, lcml_stream_t stream);

/*
 * lcml_fp8_gemm_rowquant for callers that cannot allocate device memory.
 * No counterpart in the reference: it exists for hosts that own every byte
 * of device memory through their own buffer abstraction and have no way to
 * hand this library a temporary buffer, or that reserve the whole HBM up
 * front and must not call cudaMalloc (which also synchronises the device)
 * while serving. Same inputs, outputs and results as lcml_fp8_gemm_rowquant;
 * the M-float row-max scratch is instead a static device array inside the
 * library (256 KiB per GPU that loads it, held until the process exits).
 * Limit: M <= 65536 rows; larger M is rejected with LCML_ERR_INVALID_ARGUMENT
 * before any work is enqueued. It calls no cudaMalloc / cudaFree.
 * Each call looks up the array's device address (cudaGetSymbolAddress), so
 * the address follows a module reload after cudaDeviceReset; the first call
 * on a device may load the module, so make it before any stream capture.
 * The library's other per-device state (its device error word) is kept for
 * the life of the process: do not cudaDeviceReset a device while this
 * library is in use on it.
 * All calls share the array and each call zeroes the rows it uses, so calls
 * that overlap on the GPU (e.g. on two streams) race and must be serialised.
 */
int lcml_fp8_gemm_rowquant_noalloc(const lcml_fp8_gemm_desc *desc, uint8_t *q, float *q_scale,
                                   lcml_stream_t stream);

/*
 * Plain fp32 Gemm, Y = alpha * op(A) * op(B) + beta * C, for graphs without
 * QDQ nodes (e.g. the reference's fp32 MLP fixture). Follows Gemm::apply
 * (src/onnx/operators/gemm.cpp:28-325): transA/transB, C broadcast from a
 * scalar, [N], [M], [1,N], [M,1] or [M,N] (c_ndim < 0: no C), fp32 fma
 * accumulation. CUDA-core kernel; the FP8 path is lcml_fp8_gemm.
 */
int lcml_gemm_f32(const float *A, const float *B, const float *C, int64_t M, int64_t N, int64_t K, int transA,
                  int transB, float alpha, float beta, int c_ndim, int64_t c_d0, int64_t c_d1, float *Y,
                  lcml_stream_t stream);
/* The same Gemm followed by Relu (Y = Y > 0 ? Y : 0, as the Relu operator) in one
 * kernel: the executor's fusion of an fp32 Gemm whose only reader is a Relu. */
int lcml_gemm_f32_relu(const float *A, const float *B, const float *C, int64_t M, int64_t N, int64_t K, int transA,
                       int transB, float alpha, float beta, int c_ndim, int64_t c_d0, int64_t c_d1, float *Y,
                       lcml_stream_t stream);

/*
 * FP8 2-D convolution on the tensor cores (the DequantizeLinear -> Conv ->
 * (Add residual) -> (Relu) -> (QuantizeLinear) node group of a QDQ graph).
 * Stands in for Conv::forward (src/onnx/operators/conv.cpp:35-255), which
 * accumulates FP8 inputs in half precision; here products are exact and
 * accumulate in fp32. Lowering: output pixels are GEMM rows, output channels
 * GEMM columns, K = (kh, kw, c) with c over Cp channels per tap: Cp = C
 * when C is a multiple of 16, else C padded to 4, 8 or the next multiple of
 * 16 (so each tap is one 4-, 8- or 16-byte vector). A 1x1 / stride-1 /
 * unpadded conv on an NHWC input reads X as the GEMM's A directly. A conv on
 * an NHWC input with C a multiple of 64 (X 16-byte aligned; pads <= 128,
 * strides <= 8, (k - 1) * dilation <= 255) runs as an implicit GEMM: the
 * kernel loads each K-block of patches from X with a TMA im2col copy (zero
 * outside the image), so it needs no workspace. Every other conv gathers its
 * patches (im2col, e4m3, zero padding) into `workspace` (after copying X into
 * a channel-padded NHWC layout there when X is NCHW or C is not a multiple of
 * 16) and runs the TMA-fed GEMM on them.
 * X: e4m3, NHWC (x_nhwc = 1) or NCHW (x_nhwc = 0), per-tensor scale.
 * Wp: weights packed by lcml_fp8_conv_pack_weight, per-tensor or per-output-
 * channel scales. Y: NHWC [N, oH, oW, M] (the GEMM's row-major output),
 * fp32 / bf16 / e4m3 (with y_scale). residual: same layout as Y, fp32 or e4m3
 * (with residual_scale), added before the activation. Pads are the begin
 * pads (conv.cpp:119-121). group > 1 (grouped and depthwise convs, conv.cpp:
 * 62-63, :122-139: input channels [g*C/group, (g+1)*C/group) feed output
 * channels [g*M/group, (g+1)*M/group)) runs a direct kernel on the CUDA cores
 * (little reuse per output: memory-bound), with weights packed for C/group
 * channels and the same epilogue; it needs no workspace.
 */
typedef struct lcml_fp8_conv_desc {
    int64_t N, C, H, W;     /* input */
    int64_t M, kH, kW;      /* output channels, kernel */
    int64_t oH, oW;         /* output spatial */
    int sH, sW, pH, pW, dH, dW, group;
    const uint8_t *X;
    int x_nhwc;
    const float *scale_x;   /* device [1] */
    const uint8_t *Wp;      /* packed weights [M, Kp] */
    const float *scale_w;   /* device [1] or [M] */
    int scale_w_mode;       /* LCML_SCALE_TENSOR or LCML_SCALE_AXIS (per output channel) */
    const float *bias;      /* optional fp32 [M] */
    const void *residual;   /* optional, NHWC like Y */
    int residual_dtype;     /* LCML_DTYPE_FLOAT or LCML_DTYPE_FLOAT8E4M3FN */
    const float *residual_scale;
    int epilogue;           /* LCML_EPI_NONE or LCML_EPI_RELU */
    void *Y;
    int y_dtype;            /* FLOAT, BFLOAT16 or FLOAT8E4M3FN */
    const float *y_scale;   /* per-tensor output scale when y_dtype is e4m3 */
    void *workspace;        /* lcml_fp8_conv_workspace_size() bytes, 256-byte aligned */
    /* Lowering choice, per call (0 = automatic). Bit 0: gather the patches
     * (im2col into the workspace) even where the implicit GEMM applies;
     * bits 8-10: the GEMM's lcml_fp8_gemm_desc.variant. */
    int variant;
} lcml_fp8_conv_desc;

/* Packed K: kH * kW * Cp (Cp: C padded as above) rounded up to a multiple of 16. */
int64_t lcml_fp8_conv_packed_k(int64_t Cg, int64_t kH, int64_t kW);
/* Bytes of scratch `desc` needs (0 for the direct 1x1 and the implicit-GEMM paths, -1 on a bad desc). */
int64_t lcml_fp8_conv_workspace_size(const lcml_fp8_conv_desc *desc);
/* Packs e4m3 W [M, Cg, kH, kW] (ONNX layout) into Wp [M, Kp], K order (kh, kw, c) over Cp channels,
 * zero in the padding channels and past kH * kW * Cp. */
int lcml_fp8_conv_pack_weight(const uint8_t *W, int64_t M, int64_t Cg, int64_t kH, int64_t kW, uint8_t *Wp,
                              lcml_stream_t stream);
int lcml_fp8_conv(const lcml_fp8_conv_desc *desc, lcml_stream_t stream);

/*
 * fp32 Conv (src/onnx/operators/conv.cpp:115-207) for graphs without QDQ:
 * X NCHW [N, C, H, W], W [M, C/group, kH, kW], optional bias B [M], begin
 * pads, strides, dilations, group; Y NCHW [N, M, oH, oW]. The sum order is the
 * reference's: taps in (kh, kw) order, within a tap four lane sums over the
 * group's channels (fma) added as ((x + y) + z) + w, the remaining C/group % 4
 * channels by fma, then + bias. A 1-D conv is H = kH = oH = 1.
 */
int lcml_conv2d_f32(const float *X, const float *W, const float *B, int64_t N, int64_t C, int64_t H, int64_t Wd,
                    int64_t M, int64_t kH, int64_t kW, int64_t oH, int64_t oW, int sH, int sW, int pH, int pW, int dH,
                    int dW, int group, float *Y, lcml_stream_t stream);
/* fp32 ConvTranspose (src/onnx/operators/conv_transpose.cpp): X NCHW
 * [N, C, H, W], W [C, M/group, kH, kW], optional bias [M], Y NCHW
 * [N, M, oH, oW] (oH / oW as the graph declares them, output_padding
 * included). Gather form: Y[n, m, oh, ow] sums X[n, c, ih, iw] *
 * W[c, m % (M/group), kh, kw] over the channels c of m's group and the taps
 * with oh + pH - kh * dH = ih * sH (likewise ow), in the reference's order
 * (taps, then four lane sums over c), then + bias. */
int lcml_conv_transpose2d_f32(const float *X, const float *W, const float *B, int64_t N, int64_t C, int64_t H,
                              int64_t Wd, int64_t M, int64_t kH, int64_t kW, int64_t oH, int64_t oW, int sH, int sW,
                              int pH, int pW, int dH, int dW, int group, float *Y, lcml_stream_t stream);

/*
 * Memory-bound operators around the GEMMs (fp32 unless stated).
 */
/* Relu (unary.cpp:85) / Sigmoid (unary.cpp:86-87) / Abs (unary.cpp:110). op: 0 relu, 1 sigmoid, 2 abs */
int lcml_unary_f32(int op, const float *x, float *y, int64_t n, lcml_stream_t stream);
/* Add/Sub/Mul/Div (binary.cpp:341-350) with NumPy broadcast of b over a's
 * trailing dims: b has b_n elements and b_n divides n (scalar, row or same shape).
 * op: 0 add, 1 sub, 2 mul, 3 div. */
int lcml_binary_f32(int op, const float *a, const float *b, int64_t n, int64_t b_n, float *y,
                    lcml_stream_t stream);
/* ReduceMax over the last axis (reduce.cpp:431): x [rows, cols] -> y [rows]. abs_first applies Abs. */
int lcml_reduce_max_rows(const float *x, int64_t rows, int64_t cols, int abs_first, float *y,
                         lcml_stream_t stream);
/* Softmax over the last axis (softmax.cpp:216-443): x, y [rows, cols]. */
int lcml_softmax_rows(const float *x, int64_t rows, int64_t cols, float *y, lcml_stream_t stream);
/* Add/Sub/Mul/Div of FP8-typed tensors (FLOAT8E4M3FN or FLOAT8E5M2 values,
 * no scale), the reference's quantized Binary path (binary.cpp:185-283):
 * both operands decoded to half, the op in IEEE half arithmetic, the half
 * result encoded with the fp_quantized.h codec. Broadcast of b as in
 * lcml_binary_f32. op: 0 add, 1 sub, 2 mul, 3 div. */
int lcml_binary_fp8(int op, const uint8_t *a, const uint8_t *b, int64_t n, int64_t b_n, uint8_t *y, int dtype,
                    lcml_stream_t stream);
/* Softmax over the last axis of an FP8-typed tensor (softmax.cpp:245-280:
 * decode, softmax, encode). The softmax runs in fp32 (the reference's half
 * arithmetic and half exp are not reproduced); its result is rounded to half
 * and encoded with the codec. */
int lcml_softmax_rows_fp8(const uint8_t *x, int64_t rows, int64_t cols, uint8_t *y, int dtype,
                          lcml_stream_t stream);
/* MaxPool 2-D (max_pool.cpp:20-300), NCHW fp32 or e4m3 (elem_dtype), begin pads. */
int lcml_maxpool2d(const void *x, int elem_dtype, int64_t NC, int64_t H, int64_t W, int kH, int kW, int sH,
                   int sW, int pH, int pW, int64_t oH, int64_t oW, void *y, int x_nhwc, int64_t C,
                   lcml_stream_t stream);
/* GlobalAveragePool (global_average_pool.cpp:12-154): x [N, C, H*W] (or NHWC) -> y [N, C] fp32.
 * x may be e4m3 with a per-tensor scale (x_scale) or fp32/bf16. */
int lcml_global_avgpool(const void *x, int elem_dtype, const float *x_scale, int64_t N, int64_t C, int64_t HW,
                        int x_nhwc, float *y, lcml_stream_t stream);
/* Cast (src/onnx/operators/cast.cpp:10-162) of n elements between FLOAT,
 * FLOAT16, BFLOAT16, FLOAT8E4M3FN, FLOAT8E5M2 and FLOAT4E2M1 (packed). As the
 * reference: to FP8 / FP4 the value is rounded to half first and then
 * encoded (cast.cpp:63-67, from_float(half(x)) with the fp_quantized.h
 * encoders: e4m3 and e2m1 saturate, e5m2 overflows to inf); from FP8 / FP4 it
 * is decoded exactly (cast.cpp:44-48); fp32 / fp16 / bf16 convert with one
 * round-to-nearest-even. Source and destination types must differ; x and y
 * must be aligned to their element size (LCML_ERR_INVALID_ARGUMENT otherwise). */
int lcml_cast(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, lcml_stream_t stream);

#ifdef __cplusplus
}/* extern "C" */
#endif

#endif /* LCML_FP8_H */
