/* C ABI of the B200 (sm_100a) geo-biased station attention library, libgeoattn.so.
 *
 * The reference implements this path in Python: the operator is
 *   MultiHeadAttention.scaled_dot_product_attention        fore_swe/custom_encoder_model.py:25-39
 * its fused replacement is
 *   FusedGeoAttentionV2.forward / .backward                 foreswe_bench/geo_attention_v2.py:401-461
 *   fused_geo_attention_v2(q, k, v, dist, ang, a, b, g)     foreswe_bench/geo_attention_v2.py:464-465
 * and the bias construction is
 *   DataLoader.getDistanceAndAngularity (+ helpers)         fore_swe/extended_dl_forecasting.py:305-352
 * A Python (ctypes) binding of every entry point below lives in foreswe_gpu_optimization_b200/_lib.py.
 *
 * Conventions: all data pointers are memory of the current device (cudaGetDevice) or managed memory, and
 * `stream` belongs to that device; tensors are [B, H, N, D] with element strides; the
 * library never allocates or frees device memory (callers pass outputs and workspaces sized by the *_bytes
 * functions); every call is asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream), performs no
 * host synchronisation and is safe to capture in a CUDA graph. Every entry point returns a GEOATTN_* status code.
 */
#ifndef GEOATTN_H_
#define GEOATTN_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GEOATTN_VERSION 2

enum {
  GEOATTN_OK = 0,
  GEOATTN_ERR_INVALID = 1,     /* null, host or other-device pointer, non-positive size, bad enum */
  GEOATTN_ERR_UNSUPPORTED = 2, /* head_dim / dtype combination without a kernel */
  GEOATTN_ERR_ALIGNMENT = 3,   /* tensor base or stride not 16-byte aligned, or head dim not contiguous */
  GEOATTN_ERR_TMA = 4,         /* TMA descriptor encoding failed */
  GEOATTN_ERR_LAUNCH = 5,      /* CUDA launch error */
  GEOATTN_ERR_DEVICE = 6,      /* a kernel's bounded wait expired (reported through geoattn_read_status) */
  GEOATTN_ERR_SCRATCH = 7      /* geoattn_bwd_noalloc: workspace larger than its static buffer */
};

enum { GEOATTN_DTYPE_BF16 = 0, GEOATTN_DTYPE_FP32 = 1 };

/* Problem shape. dtype is the storage type of q, k, v, o, dO, dQ, dK, dV:
 *   BF16 -> bf16 tensor-core path (kind::f16), geo prior kept as fp16 pairs;
 *   FP32 -> TF32 tensor-core path (kind::tf32) with 3-term split products for QK^T and dO V^T
 *           (round-to-nearest hi/lo operands), 1-term for the rest; geo prior kept in fp32.
 * Supported head_dim: 1..192 (BF16 and FP32). n >= 1 (any size).                                          */
typedef struct {
  int batch, heads, n, head_dim;
  int dtype;
  int per_head; /* alpha/beta/gamma hold `heads` values each (else 1): reference parameters are scalars
                   (custom_encoder_model.py:16-18) */
} GeoAttnShape;

typedef struct {
  const void* data;
  long long stride[4]; /* element strides of [B, H, N, D]; stride[3] must be 1 */
} GeoAttnTensor;

/* ---- geometry: station coordinates -> geo prior (replaces the host float64 construction) ---------------- */
size_t geoattn_prior_bytes(const GeoAttnShape* shape);

/* Prior from dense [n, n] fp32 distance (km) and angle (degrees) matrices (row strides ld_*), i.e. the
 * reference's (distances, angularities) arguments: Dp = 1/(1+dist), Ap = 1/(1+ang) (custom_encoder_model.py:32-33).
 * Requires dist, ang >= 0.                                                                                  */
int geoattn_prior_from_dense(const GeoAttnShape* shape, const float* dist, long long ld_dist, const float* ang,
                             long long ld_ang, void* prior, void* stream);

/* Prior straight from per-station coordinates (float64 degrees, elevation in feet): great-circle distance on
 * the 6371 km sphere and Kahan's 2*atan2 angle between the reference's station vectors
 * (extended_dl_forecasting.py:20-30, :305-344), evaluated in float64 on the device and rounded to fp32 like the
 * reference's fp32 copies; no [n, n] matrix is produced. dist_out / ang_out (may be NULL) receive the
 * fp32 matrices with row stride n.                                                                          */
int geoattn_prior_from_coords(const GeoAttnShape* shape, const double* lat_deg, const double* lon_deg,
                              const double* elev_ft, void* prior, float* dist_out, float* ang_out, void* stream);

/* ---- forward ------------------------------------------------------------------------------------------- */
size_t geoattn_stats_bytes(const GeoAttnShape* shape);          /* row statistics kept for the backward */
size_t geoattn_fwd_workspace_bytes(const GeoAttnShape* shape);

typedef struct {
  GeoAttnShape shape;
  GeoAttnTensor q, k, v;
  const float* abg;   /* device fp32 [3 * nabg]: alpha..., beta..., gamma... (nabg = per_head ? heads : 1) */
  const void* prior;  /* from geoattn_prior_* for the same n and dtype */
  void* o;            /* output, dtype of the inputs */
  long long o_stride[4];
  float* stats;       /* geoattn_stats_bytes */
  void* workspace;    /* geoattn_fwd_workspace_bytes, 256-byte aligned */
  void* const* events; /* optional (NULL = none): 2 cudaEvent_t recorded on `stream` around the attention
                          kernel, for per-kernel timing */
} GeoAttnFwdArgs;

/* O = softmax(alpha*softmax(QK^T/sqrt(d)) + beta*Dp + gamma*Ap) V; replaces FusedGeoAttentionV2.forward
 * (geo_attention_v2.py:402-425). */
int geoattn_fwd(const GeoAttnFwdArgs* args, void* stream);

/* ---- backward ------------------------------------------------------------------------------------------ */
size_t geoattn_bwd_workspace_bytes(const GeoAttnShape* shape);

typedef struct {
  GeoAttnShape shape;
  GeoAttnTensor q, k, v, o, dout; /* o: the forward output; checked, not read (delta2 comes from the tiles) */
  const float* abg;
  const void* prior;
  const float* stats; /* written by geoattn_fwd for the same inputs */
  void* dq;
  long long dq_stride[4];
  void* dk;
  long long dk_stride[4];
  void* dv;
  long long dv_stride[4];
  float* dabg;        /* fp32 [3 * nabg]: d alpha..., d beta..., d gamma... (summed over batch, rows) */
  void* workspace;    /* geoattn_bwd_workspace_bytes, 256-byte aligned */
  void* const* events; /* optional (NULL = none): 4 cudaEvent_t recorded on `stream` before the row-pass kernel,
                          between the row-pass and key-pass kernels, after the key-pass kernel and after the dQ
                          GEMM (the last two coincide when dQ comes from the row pass) */
} GeoAttnBwdArgs;

/* dQ, dK, dV and the bias-parameter gradients; replaces FusedGeoAttentionV2.backward
 * (geo_attention_v2.py:428-461). Deterministic: no atomics, fixed reduction order. BF16: the workspace holds a
 * bf16 dS scratch of B*H*N_pad^2 elements (N_pad = N rounded up to 128), which the key pass writes and a dQ GEMM
 * reads; FP32: the same with an fp32 scratch of B*H*N_pad^2 elements and a TF32 dQ GEMM (above head_dim 64 the GEMM
 * transposes each dS tile in shared memory). */
int geoattn_bwd(const GeoAttnBwdArgs* args, void* stream);

/* Allocation-free backward (no counterpart in the reference, which always allocates through PyTorch).
 * For callers that cannot allocate device memory themselves -- plugin/custom-op hosts that own every device buffer
 * and give an operator only its inputs and outputs, or code with a fixed memory plan where an allocation would
 * synchronise the device. Same arguments and results as geoattn_bwd, except that args->workspace is ignored: the
 * scratch comes from a static 16 MiB device array that the library holds on every device that loads it until the
 * process exits. Limits: BF16 only (GEOATTN_ERR_UNSUPPORTED for FP32). The scratch it needs is
 *   256 + align256(B*H*N_pad*16) + align256(B*H*ceil(N/128)*24) bytes,  N_pad = N rounded up to 128
 * (row records and bias-gradient partials; it forms dQ in a second row-pass sweep and keeps no dS scratch, so this
 * is not geoattn_bwd_workspace_bytes), and must be <= 16 MiB, else GEOATTN_ERR_SCRATCH before any launch: at
 * N = 512 that is B*H <= 2024 (e.g. 64 issue dates x 16 heads; 128 x 16 is rejected), about 1M query rows.
 * All calls share the array, so calls that overlap on the GPU race. The first call on a device looks up the
 * array's address (cudaGetSymbolAddress); make it before any stream capture. A bounded wait that expires inside
 * the call is reported through geoattn_read_status(NULL, ...) (below), not by the return code.
 * It allocates nothing (no cudaMalloc/cudaFree, no allocating library call).                                  */
int geoattn_bwd_noalloc(const GeoAttnBwdArgs* args, void* stream);

/* ---- diagnostics --------------------------------------------------------------------------------------- */
/* Copies the device status word of a workspace (0 = ok, 1 = a bounded wait expired, 2 = a kernel found its shared
 * memory misaligned and did nothing) to *status. workspace = NULL reads the status word of the last
 * geoattn_bwd_noalloc call on the current device (its static scratch). Synchronises the stream; for tests and
 * debugging only. */
int geoattn_read_status(const void* workspace, int* status, void* stream);
/* Self-test of the kernels' bounded waits: launches one thread that waits on a barrier nothing completes. After the
 * wait limit (about 2 s) the wait gives up, the kernel sets the 4-byte device word `status_word` to 1 (as a timed-out
 * attention kernel sets its workspace's status word) and returns; the context stays usable. Asynchronous on
 * `stream`; for tests only. */
int geoattn_wait_selftest(void* status_word, void* stream);
const char* geoattn_error_string(int code);
int geoattn_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GEOATTN_H_ */
