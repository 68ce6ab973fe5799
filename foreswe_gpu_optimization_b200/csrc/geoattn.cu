// libgeoattn.so: host launchers behind the C ABI in include/geoattn.h, plus the small auxiliary kernels
// (geometry prologue, TF32 operand split, deterministic bias-gradient reduction).
#include <cuda_fp16.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/geoattn.h"
#include "geoattn_kernels.cuh"
#include "tma_host.h"

namespace geoattn {

// ---------------------------------------------------------------------------------------------------------------
// Geometry prologue
// ---------------------------------------------------------------------------------------------------------------
template <bool F16>
struct PairT;
template <>
struct PairT<true> {
  using type = __half2;
  __device__ static type make(float a, float b) { return __floats2half2_rn(a, b); }
};
template <>
struct PairT<false> {
  using type = float2;
  __device__ static type make(float a, float b) { return make_float2(a, b); }
};

// Reciprocal prior exactly as the reference's fp32 elementwise ops: 1 / (1 + x), both correctly rounded.
__device__ __forceinline__ float recip1p(float x) { return __frcp_rn(__fadd_rn(1.0f, x)); }

template <bool F16>
__global__ void prior_dense_kernel(const float* __restrict__ dist, long long ldd, const float* __restrict__ ang,
                                   long long lda, int N, int np, void* prior, void* priorT) {
  using P = PairT<F16>;
  using V = typename P::type;
  __shared__ V tile[32][33];
  const int i0 = blockIdx.y * 32, j0 = blockIdx.x * 32, tx = threadIdx.x;
  V* pr = reinterpret_cast<V*>(prior);
  V* pt = reinterpret_cast<V*>(priorT);
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int i = i0 + k, j = j0 + tx;
    float a = 0.f, b = 0.f;
    if (i < N && j < N) {
      a = recip1p(dist[(long long)i * ldd + j]);
      b = recip1p(ang[(long long)i * lda + j]);
    }
    const V v = P::make(a, b);
    pr[(size_t)i * np + j] = v;
    tile[k][tx] = v;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) pt[(size_t)(j0 + k) * np + (i0 + tx)] = tile[tx][k];
}

// float64 station geometry, operation order of the reference's numpy code (no FMA contraction):
//   haversine: 2*asin(sqrt(sin^2((lat_i-lat_j)/2) + cos(lat_i)cos(lat_j) sin^2((lon_i-lon_j)/2))) * 6371
//   vectors:   R = 6371 + elev_ft*0.3048; x = R cos(lat) cos(lon); y = R cos(lat) sin(lon); v = (x, y, x)
//   angle:     2*atan2(|n_i v_j - n_j v_i|, |n_i v_j + n_j v_i|) in degrees
__device__ __forceinline__ void station_vec(double lat, double lon, double elev_ft, double& x, double& y, double& n) {
  const double d2r = 0.017453292519943295;  // pi / 180
  const double r = __dadd_rn(6371.0, __dmul_rn(elev_ft, 0.3048));
  const double cl = cos(__dmul_rn(lat, d2r));
  x = __dmul_rn(__dmul_rn(r, cl), cos(__dmul_rn(lon, d2r)));
  y = __dmul_rn(__dmul_rn(r, cl), sin(__dmul_rn(lon, d2r)));
  n = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)), __dmul_rn(x, x)));
}

__device__ __forceinline__ void pair_geometry(const double* lat, const double* lon, const double* elev, int i, int j,
                                              float& dist_km, float& ang_deg) {
  const double d2r = 0.017453292519943295;
  const double li = __dmul_rn(lat[i], d2r), lj = __dmul_rn(lat[j], d2r);
  const double oi = __dmul_rn(lon[i], d2r), oj = __dmul_rn(lon[j], d2r);
  const double s1 = sin(__dmul_rn(0.5, __dsub_rn(li, lj)));
  const double s2 = sin(__dmul_rn(0.5, __dsub_rn(oi, oj)));
  const double h = __dadd_rn(__dmul_rn(s1, s1), __dmul_rn(__dmul_rn(__dmul_rn(cos(li), cos(lj)), s2), s2));
  dist_km = (float)__dmul_rn(__dmul_rn(2.0, asin(sqrt(h))), 6371.0);
  double xi, yi, ni, xj, yj, nj;
  station_vec(lat[i], lon[i], elev[i], xi, yi, ni);
  station_vec(lat[j], lon[j], elev[j], xj, yj, nj);
  // u_norm_v = n_i * v_j, v_norm_u = n_j * v_i (components x, y, x)
  const double ax = __dsub_rn(__dmul_rn(ni, xj), __dmul_rn(nj, xi));
  const double ay = __dsub_rn(__dmul_rn(ni, yj), __dmul_rn(nj, yi));
  const double sx = __dadd_rn(__dmul_rn(ni, xj), __dmul_rn(nj, xi));
  const double sy = __dadd_rn(__dmul_rn(ni, yj), __dmul_rn(nj, yi));
  const double na = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(ax, ax), __dmul_rn(ay, ay)), __dmul_rn(ax, ax)));
  const double ns = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(sx, sx), __dmul_rn(sy, sy)), __dmul_rn(sx, sx)));
  ang_deg = (float)__dmul_rn(__dmul_rn(2.0, atan2(na, ns)), 57.29577951308232);  // 180 / pi
}

template <bool F16>
__global__ void prior_coords_kernel(const double* __restrict__ lat, const double* __restrict__ lon,
                                    const double* __restrict__ elev, int N, int np, void* prior, void* priorT,
                                    float* dist_out, float* ang_out) {
  using P = PairT<F16>;
  using V = typename P::type;
  __shared__ V tile[32][33];
  const int i0 = blockIdx.y * 32, j0 = blockIdx.x * 32, tx = threadIdx.x;
  V* pr = reinterpret_cast<V*>(prior);
  V* pt = reinterpret_cast<V*>(priorT);
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int i = i0 + k, j = j0 + tx;
    float a = 0.f, b = 0.f;
    if (i < N && j < N) {
      float dk, ad;
      pair_geometry(lat, lon, elev, i, j, dk, ad);
      if (dist_out) dist_out[(size_t)i * N + j] = dk;
      if (ang_out) ang_out[(size_t)i * N + j] = ad;
      a = recip1p(dk);
      b = recip1p(ad);
    }
    const V v = P::make(a, b);
    if (pr) pr[(size_t)i * np + j] = v;
    tile[k][tx] = v;
  }
  __syncthreads();
  if (pt)
    for (int k = threadIdx.y; k < 32; k += 8) pt[(size_t)(j0 + k) * np + (i0 + tx)] = tile[tx][k];
}

// ---------------------------------------------------------------------------------------------------------------
// TF32 operand split: x = hi + lo, hi = tf32_rn(x), lo = tf32_rn(x - hi).
//   natural planes: [2][B][H][N][DP] (hi then lo), transposed hi plane: [B][H][DP][NP]; zero padded.
// ---------------------------------------------------------------------------------------------------------------
__global__ void split_tf32_kernel(const float* __restrict__ x, long long s0, long long s1, long long s2, long long s3,
                                  int B, int H, int N, int D, int DP, int NP, float* nat, float* tr) {
  __shared__ float tile[32][33];
  const int bh = blockIdx.z, b = bh / H, h = bh % H;
  const int n0 = blockIdx.x * 32, d0 = blockIdx.y * 32, tx = threadIdx.x;
  const size_t plane = (size_t)B * H * N * DP;
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int n = n0 + k, d = d0 + tx;
    float v = 0.f;
    if (n < N && d < D) v = x[b * s0 + h * s1 + (long long)n * s2 + (long long)d * s3];
    const float hi = round_tf32(v);
    const float lo = round_tf32(v - hi);
    if (nat && n < N) {
      const size_t o = ((size_t)bh * N + n) * DP + d;
      nat[o] = hi;
      nat[plane + o] = lo;
    }
    tile[k][tx] = hi;
  }
  if (!tr) return;
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) tr[((size_t)bh * DP + d0 + k) * NP + n0 + tx] = tile[tx][k];
}

// The same split with 16-byte accesses, for a tensor whose head dim is contiguous (stride 1) and whose other strides,
// base address and D are multiples of 4 elements (every operand of a torch-allocated fp32 tensor with D % 4 == 0).
// Thread t of 256 loads 4 consecutive d of one row (tile 32 rows x 32 d), writes both natural planes as float4, and
// the transposed hi plane leaves through a [d][n] shared-memory tile as float4 along n.
__global__ void __launch_bounds__(256) split_tf32_vec_kernel(const float* __restrict__ x, long long s0, long long s1,
                                                             long long s2, int B, int H, int N, int D, int DP, int NP,
                                                             float* nat, float* tr) {
  __shared__ float tile[32][33];
  const int bh = blockIdx.z, b = bh / H, h = bh % H;
  const int n0 = blockIdx.x * 32, d0 = blockIdx.y * 32, t = threadIdx.x;
  const int r = t >> 3, d = d0 + 4 * (t & 7), n = n0 + r;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (n < N && d < D) v = *reinterpret_cast<const float4*>(x + b * s0 + h * s1 + (long long)n * s2 + d);
  const float4 hi = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
  if (nat && n < N) {
    const size_t o = ((size_t)bh * N + n) * DP + d;
    const float4 lo = make_float4(round_tf32(v.x - hi.x), round_tf32(v.y - hi.y), round_tf32(v.z - hi.z),
                                  round_tf32(v.w - hi.w));
    *reinterpret_cast<float4*>(nat + o) = hi;
    *reinterpret_cast<float4*>(nat + (size_t)B * H * N * DP + o) = lo;
  }
  if (!tr) return;
  const int dl = d - d0;
  tile[dl][r] = hi.x;
  tile[dl + 1][r] = hi.y;
  tile[dl + 2][r] = hi.z;
  tile[dl + 3][r] = hi.w;
  __syncthreads();
  const int dd = t >> 3, nq = 4 * (t & 7);
  *reinterpret_cast<float4*>(tr + ((size_t)bh * DP + d0 + dd) * NP + n0 + nq) =
      make_float4(tile[dd][nq], tile[dd][nq + 1], tile[dd][nq + 2], tile[dd][nq + 3]);
}

// ---------------------------------------------------------------------------------------------------------------
// d(alpha), d(beta), d(gamma): fixed-order float64 sum of the per-(b*h, row block) partials.
// ---------------------------------------------------------------------------------------------------------------
__global__ void finalize_abg_kernel(const double* __restrict__ part, int B, int H, int nrb, int per_head, float* dabg) {
  __shared__ double red[256];
  const int k = blockIdx.x, hh = blockIdx.y, nabg = per_head ? H : 1;
  const int count = per_head ? B * nrb : B * H * nrb;
  double acc = 0.0;
  for (int idx = threadIdx.x; idx < count; idx += blockDim.x) {
    int bh, rb;
    if (per_head) {
      bh = (idx / nrb) * H + hh;
      rb = idx % nrb;
    } else {
      bh = idx / nrb;
      rb = idx % nrb;
    }
    acc += part[((size_t)bh * nrb + rb) * 3 + k];
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) dabg[k * nabg + hh] = (float)red[0];
}

// ---------------------------------------------------------------------------------------------------------------
// Self-test of the bounded waits every attention kernel uses: one thread waits for the first phase of an mbarrier
// that nothing arrives on. The wait gives up after its limit, records the timeout in the status word (first error
// wins) and the kernel returns, leaving the context usable.
// ---------------------------------------------------------------------------------------------------------------
__global__ void wait_selftest_kernel(int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  abort_flag = 0;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const WaitCtx ctx{&abort_flag, status};
  (void)mbar_wait(&bar, 0, ctx);
}

// ---------------------------------------------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------------------------------------------
namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Dims {
  int B, H, N, D, DP, nrb, np;
  bool bf16;
  int nabg;
};

// The backward keeps a dS scratch and forms dQ by a GEMM (instead of a second row-pass sweep): bf16 stores dS^T
// and reads it MN-major; fp32 at head dim 64 stores dS [query][key] (the pooled key pass has room for the transposed
// tile); fp32 above 64 stores dS^T and its dQ GEMM transposes each tile in shared memory (TF32 operands are K-major).
inline bool uses_ds(const Dims&) { return true; }

// Row records per query row (m1, c2, delta1, delta2; fp32 above head dim 64 also b, for the key pass's d(alpha)).
inline int nrec(const Dims& d) { return (!d.bf16 && d.DP > 64) ? 5 : 4; }

// Every data pointer handed to a kernel must be memory of the current device (or managed memory): the kernels run
// on the current device, which would dereference a host pointer or another device's memory. Checked on the host
// before any launch.
bool dev_ptr(const void* p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error of an unregistered host pointer
    return false;
  }
  if (a.type == cudaMemoryTypeManaged) return true;
  int cur = -1;
  return a.type == cudaMemoryTypeDevice && cudaGetDevice(&cur) == cudaSuccess && a.device == cur;
}

int check_shape(const GeoAttnShape* s, Dims& d) {
  if (!s || s->batch <= 0 || s->heads <= 0 || s->n <= 0 || s->head_dim <= 0) return GEOATTN_ERR_INVALID;
  if (s->dtype != GEOATTN_DTYPE_BF16 && s->dtype != GEOATTN_DTYPE_FP32) return GEOATTN_ERR_INVALID;
  d.B = s->batch;
  d.H = s->heads;
  d.N = s->n;
  d.D = s->head_dim;
  d.bf16 = s->dtype == GEOATTN_DTYPE_BF16;
  d.nrb = (d.N + kBM - 1) / kBM;
  d.np = d.nrb * kBM;
  d.nabg = s->per_head ? d.H : 1;
  if (d.D > 192) return GEOATTN_ERR_UNSUPPORTED;
  d.DP = d.D <= 64 ? 64 : d.D <= 128 ? 128 : 192;
  if ((long long)d.nrb * d.B * d.H > (1ll << 30)) return GEOATTN_ERR_UNSUPPORTED;  // tile index fits an int
  return GEOATTN_OK;
}

size_t prior_table_bytes(const Dims& d) { return (size_t)d.np * d.np * (d.bf16 ? 4 : 8); }

// workspace segments
struct FwdWs {
  int* status;
  float *qn, *kn, *vt;
};
size_t fwd_ws(const Dims& d, uint8_t* base, FwdWs* w) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> uint8_t* {
    uint8_t* p = base ? base + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  FwdWs t{};
  t.status = reinterpret_cast<int*>(take(sizeof(int)));
  if (!d.bf16) {
    const size_t nat = (size_t)2 * d.B * d.H * d.N * d.DP * 4, trn = (size_t)d.B * d.H * d.DP * d.np * 4;
    t.qn = reinterpret_cast<float*>(take(nat));
    t.kn = reinterpret_cast<float*>(take(nat));
    t.vt = reinterpret_cast<float*>(take(trn));
  }
  if (w) *w = t;
  return off;
}

struct BwdWs {
  int* status;
  float* rowrec;
  double* part;
  float *qn, *kn, *vn, *don, *kt, *qt, *dot;
  void* dsT;  // bf16 dS^T scratch [B*H][N_pad keys][N_pad queries] (dS-scratch backward only)
};
// The backward with a caller-provided workspace keeps dS in a scratch (`with_ds`; bf16, and fp32 at head dim 64):
// key pass -> dQ GEMM.
size_t bwd_ws(const Dims& d, uint8_t* base, BwdWs* w, bool with_ds) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> uint8_t* {
    uint8_t* p = base ? base + off : nullptr;
    off += align_up(bytes);
    return p;
  };
  BwdWs t{};
  t.status = reinterpret_cast<int*>(take(sizeof(int)));
  t.rowrec = reinterpret_cast<float*>(take((size_t)d.B * d.H * d.np * nrec(d) * 4));  // [B*H][np/CH][NREC][CH]
  t.part = reinterpret_cast<double*>(take((size_t)d.B * d.H * d.nrb * 3 * 8));
  if (!d.bf16) {
    const size_t nat = (size_t)2 * d.B * d.H * d.N * d.DP * 4, trn = (size_t)d.B * d.H * d.DP * d.np * 4;
    t.qn = reinterpret_cast<float*>(take(nat));
    t.kn = reinterpret_cast<float*>(take(nat));
    t.vn = reinterpret_cast<float*>(take(nat));
    t.don = reinterpret_cast<float*>(take(nat));
    t.kt = reinterpret_cast<float*>(take(trn));
    t.qt = reinterpret_cast<float*>(take(trn));
    t.dot = reinterpret_cast<float*>(take(trn));
  }
  // dS scratch: bf16 dS^T [b*h][key][query]; fp32 at head dim 64 dS [b*h][query][key]; fp32 above dS^T
  if (with_ds && uses_ds(d)) t.dsT = take((size_t)d.B * d.H * d.np * d.np * (d.bf16 ? 2 : 4));
  if (w) *w = t;
  return off;
}

// TMA map over the bf16 dS^T scratch, viewed as 3-D (query, key, b*h); box: 64 queries x `keys` keys.
// TMA map over an fp32 dS scratch, [b*h][query][key] (head dim 64) or [b*h][key][query] (above), viewed as 3-D
// (inner, outer, b*h); box: 32 inner x `queries` outer.
int map_ds_f32(CUtensorMap* m, void* base, const Dims& d, int queries) {
  const uint64_t dims[3] = {(uint64_t)d.np, (uint64_t)d.np, (uint64_t)d.B * d.H};
  const uint64_t str[2] = {(uint64_t)d.np * 4, (uint64_t)d.np * d.np * 4};
  const uint32_t box[3] = {32, (uint32_t)queries, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, str, box) ? GEOATTN_OK : GEOATTN_ERR_TMA;
}

int map_dsT(CUtensorMap* m, void* base, const Dims& d, int keys) {
  const uint64_t dims[3] = {(uint64_t)d.np, (uint64_t)d.np, (uint64_t)d.B * d.H};
  const uint64_t str[2] = {(uint64_t)d.np * 2, (uint64_t)d.np * d.np * 2};
  const uint32_t box[3] = {64, (uint32_t)keys, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, str, box) ? GEOATTN_OK : GEOATTN_ERR_TMA;
}

// TMA map over a user bf16 tensor [B, H, N, D] (box: 64 x rows).
int map_user_bf16(CUtensorMap* m, const GeoAttnTensor& t, const Dims& d, int rows) {
  if (!t.data) return GEOATTN_ERR_INVALID;
  if (t.stride[3] != 1) return GEOATTN_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(t.data) & 15) != 0) return GEOATTN_ERR_ALIGNMENT;
  for (int i = 0; i < 3; ++i)
    if (t.stride[i] <= 0 || ((t.stride[i] * 2) & 15) != 0) return GEOATTN_ERR_ALIGNMENT;
  const uint64_t dims[4] = {(uint64_t)d.D, (uint64_t)d.N, (uint64_t)d.H, (uint64_t)d.B};
  const uint64_t str[3] = {(uint64_t)t.stride[2] * 2, (uint64_t)t.stride[1] * 2, (uint64_t)t.stride[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)rows, 1, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data, dims, str, box) ? GEOATTN_OK : GEOATTN_ERR_TMA;
}

// TMA map over natural fp32 planes [2][B][H][N][DP] viewed as 4-D (DP, N, H, 2B) (box: 32 x rows).
int map_planes(CUtensorMap* m, const float* base, const Dims& d, int rows) {
  const uint64_t dims[4] = {(uint64_t)d.DP, (uint64_t)d.N, (uint64_t)d.H, (uint64_t)(2 * d.B)};
  const uint64_t str[3] = {(uint64_t)d.DP * 4, (uint64_t)d.N * d.DP * 4, (uint64_t)d.H * d.N * d.DP * 4};
  const uint32_t box[4] = {32, (uint32_t)rows, 1, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, str, box) ? GEOATTN_OK : GEOATTN_ERR_TMA;
}

// TMA map over a transposed fp32 plane [B][H][DP][NP] viewed as 4-D (NP, DP, H, B) (box: 32 x DP).
int map_transposed(CUtensorMap* m, const float* base, const Dims& d) {
  const uint64_t dims[4] = {(uint64_t)d.np, (uint64_t)d.DP, (uint64_t)d.H, (uint64_t)d.B};
  const uint64_t str[3] = {(uint64_t)d.np * 4, (uint64_t)d.DP * d.np * 4, (uint64_t)d.H * d.DP * d.np * 4};
  const uint32_t box[4] = {32, (uint32_t)d.DP, 1, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, str, box) ? GEOATTN_OK : GEOATTN_ERR_TMA;
}

// TMA map over a prior table ([np][np] pairs viewed as 32-bit words; box: 32 words x 128 rows).
int map_prior(CUtensorMap* m, const void* table, const Dims& d) {
  const uint64_t words = (uint64_t)d.np * (d.bf16 ? 1 : 2);
  const uint64_t dims[2] = {words, (uint64_t)d.np};
  const uint64_t str[1] = {words * 4};
  const uint32_t box[2] = {32, (uint32_t)kBM};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, table, dims, str, box) ? GEOATTN_OK : GEOATTN_ERR_TMA;
}

int split(const GeoAttnTensor& t, const Dims& d, float* nat, float* tr, cudaStream_t st) {
  if (!t.data) return GEOATTN_ERR_INVALID;
  const bool vec = t.stride[3] == 1 && (reinterpret_cast<uintptr_t>(t.data) & 15) == 0 && d.D % 4 == 0 &&
                   t.stride[0] % 4 == 0 && t.stride[1] % 4 == 0 && t.stride[2] % 4 == 0;
  if (vec) {
    dim3 grid((d.np + 31) / 32, d.DP / 32, d.B * d.H);
    split_tf32_vec_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(t.data), t.stride[0], t.stride[1],
                                                t.stride[2], d.B, d.H, d.N, d.D, d.DP, d.np, nat, tr);
  } else {
    dim3 grid((d.np + 31) / 32, d.DP / 32, d.B * d.H), block(32, 8);
    split_tf32_kernel<<<grid, block, 0, st>>>(reinterpret_cast<const float*>(t.data), t.stride[0], t.stride[1],
                                              t.stride[2], t.stride[3], d.B, d.H, d.N, d.D, d.DP, d.np, nat, tr);
  }
  return cudaGetLastError() == cudaSuccess ? GEOATTN_OK : GEOATTN_ERR_LAUNCH;
}

KParams base_params(const Dims& d, const float* abg, int per_head, const void* prior) {
  KParams p;
  std::memset(&p, 0, sizeof(p));
  p.B = d.B;
  p.H = d.H;
  p.N = d.N;
  p.D = d.D;
  p.nrb = d.nrb;
  p.np = d.np;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)d.D));
  p.inv_sqrt_d = (float)(1.0 / std::sqrt((double)d.D));
  p.abg = abg;
  p.per_head = per_head;
  p.prior = prior;
  p.priorT = reinterpret_cast<const uint8_t*>(prior) + prior_table_bytes(d);
  p.nchp = d.np / (d.bf16 ? 64 : 32);
  return p;
}

// Store map over a bf16 output [B, H, N, D] (box 64 x 128), or false when the tensor is not TMA-compatible (the
// kernels then store rows directly).
bool map_output(CUtensorMap* m, void* data, const long long* stride, const Dims& d) {
  if (!d.bf16) return false;
  GeoAttnTensor t;
  t.data = data;
  for (int i = 0; i < 4; ++i) t.stride[i] = stride[i];
  return map_user_bf16(m, t, d, kBM) == GEOATTN_OK;
}

// Persistent grid: one CTA per SM (every attention kernel holds an SM's tensor memory), at most one per tile.
dim3 persistent_grid(const Dims& d) {
  // SM count per device, looked up once; host threads that race here store the same value
  static std::atomic<int> sms[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cached = dev >= 0 && dev < 64;
  int n = cached ? sms[dev].load(std::memory_order_relaxed) : 0;
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (cached) sms[dev].store(n, std::memory_order_relaxed);
  }
  const long long tiles = (long long)d.nrb * d.B * d.H;
  return dim3((unsigned)(tiles < n ? tiles : n));
}

template <class K>
int launch(K kernel, int smem, int threads, dim3 grid, cudaStream_t st, const TileMaps& maps, const KParams& p) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return GEOATTN_ERR_LAUNCH;
  kernel<<<grid, threads, smem, st>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? GEOATTN_OK : GEOATTN_ERR_LAUNCH;
}

inline void record(void* const* ev, int i, cudaStream_t st) {
  if (ev && ev[i]) cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev[i]), st);
}

template <bool BF16, int DP, bool ONE = false>
int run_fwd(const TileMaps& maps, const KParams& p, const Dims& d, cudaStream_t st, void* const* ev) {
  record(ev, 0, st);
  int rc = launch(geoattn_fwd_kernel<BF16, DP, ONE>, FwdCfg<BF16, DP, ONE>::SMEM, Tile<BF16, DP>::NTHREADS,
                  persistent_grid(d), st, maps, p);
  record(ev, 1, st);
  return rc;
}
// Backward launches. Events (optional): before the row pass, between the row and key passes, after the key pass,
// after the dQ GEMM (equal to the third when there is none).
template <bool BF16, int DP>
int run_bwd(const TileMaps& rmaps, const TileMaps& cmaps, const KParams& prow, const KParams& pcol, const Dims& d,
            cudaStream_t st, void* const* ev) {
  record(ev, 0, st);
  int rc = launch(geoattn_bwd_rows_kernel<BF16, DP, true>, RowsCfg<BF16, DP, true>::SMEM, Tile<BF16, DP>::NTHREADS,
                  persistent_grid(d), st, rmaps, prow);
  if (rc) return rc;
  record(ev, 1, st);
  rc = launch(geoattn_bwd_cols_kernel<BF16, DP, false>, ColsCfg<BF16, DP>::SMEM, Tile<BF16, DP>::NTHREADS,
              persistent_grid(d), st, cmaps, pcol);
  record(ev, 2, st);
  record(ev, 3, st);
  return rc;
}
// BF16 with the dS scratch: row pass (one sweep: records, d(alpha)), key pass (dK, dV, dS^T, d(beta), d(gamma)),
// dQ GEMM.
template <int DP>
int run_bwd_ds(const TileMaps& rmaps, const TileMaps& cmaps, const TileMaps& qmaps, const KParams& prow,
               const KParams& pcol, const KParams& pdq, const Dims& d, cudaStream_t st, void* const* ev) {
  record(ev, 0, st);
  int rc = launch(geoattn_bwd_rows_kernel<true, DP, false>, RowsCfg<true, DP, false>::SMEM,
                  Tile<true, DP>::NTHREADS, persistent_grid(d), st, rmaps, prow);
  if (rc) return rc;
  record(ev, 1, st);
  rc = launch(geoattn_bwd_cols_kernel<true, DP, true>, ColsCfg<true, DP, true>::SMEM, Tile<true, DP>::NTHREADS,
              persistent_grid(d), st, cmaps, pcol);
  if (rc) return rc;
  record(ev, 2, st);
  rc = launch(geoattn_bwd_dq_kernel<DP>, DqCfg<DP>::SMEM, DqCfg<DP>::NTHREADS, persistent_grid(d), st, qmaps, pdq);
  record(ev, 3, st);
  return rc;
}

// fp32 above head dim 64: the wide row pass without its second sweep (records with b), the wide key pass storing the
// fp32 dS^T tiles (and summing d(alpha), d(beta), d(gamma)), the transposing TF32 dQ GEMM.
template <int DP>
int run_bwd_ds_wide(const TileMaps& rmaps, const TileMaps& cmaps, const TileMaps& qmaps, const KParams& prow,
                    const KParams& pcol, const KParams& pdq, const Dims& d, cudaStream_t st, void* const* ev) {
  record(ev, 0, st);
  int rc = launch(geoattn_bwd_rows_kernel<false, DP, false>, RowsCfg<false, DP, false>::SMEM,
                  Tile<false, DP>::NTHREADS, persistent_grid(d), st, rmaps, prow);
  if (rc) return rc;
  record(ev, 1, st);
  rc = launch(geoattn_bwd_cols_kernel<false, DP, true>, ColsCfg<false, DP, true>::SMEM, Tile<false, DP>::NTHREADS,
              persistent_grid(d), st, cmaps, pcol);
  if (rc) return rc;
  record(ev, 2, st);
  rc = launch(geoattn_bwd_dq_tf32t_kernel<DP>, DqTf32tCfg<DP>::SMEM, DqTf32tCfg<DP>::NTHREADS, persistent_grid(d),
              st, qmaps, pdq);
  record(ev, 3, st);
  return rc;
}

// fp32 at head dim 64: the one-sweep row pass, the key pass storing fp32 dS [query][key], the TF32 dQ GEMM.
int run_bwd_ds_f32(const TileMaps& rmaps, const TileMaps& cmaps, const TileMaps& qmaps, const KParams& prow,
                   const KParams& pcol, const KParams& pdq, const Dims& d, cudaStream_t st, void* const* ev) {
  record(ev, 0, st);
  int rc = launch(geoattn_bwd_rows_kernel<false, 64, false>, RowsCfg<false, 64, false>::SMEM,
                  Tile<false, 64>::NTHREADS, persistent_grid(d), st, rmaps, prow);
  if (rc) return rc;
  record(ev, 1, st);
  rc = launch(geoattn_bwd_cols_kernel<false, 64, true>, ColsCfg<false, 64, true>::SMEM, Tile<false, 64>::NTHREADS,
              persistent_grid(d), st, cmaps, pcol);
  if (rc) return rc;
  record(ev, 2, st);
  rc = launch(geoattn_bwd_dq_tf32_kernel<64>, DqTf32Cfg<64>::SMEM, DqTf32Cfg<64>::NTHREADS, persistent_grid(d), st,
              qmaps, pdq);
  record(ev, 3, st);
  return rc;
}

}  // namespace
}  // namespace geoattn

using namespace geoattn;

extern "C" {

int geoattn_version(void) { return GEOATTN_VERSION; }

const char* geoattn_error_string(int code) {
  switch (code) {
    case GEOATTN_OK: return "ok";
    case GEOATTN_ERR_INVALID:
      return "invalid argument (null, host or other-device pointer, non-positive size or unknown enum)";
    case GEOATTN_ERR_UNSUPPORTED: return "unsupported shape/dtype (head_dim <= 192)";
    case GEOATTN_ERR_ALIGNMENT: return "tensor not TMA-compatible (head dim must be contiguous, base and strides 16-byte aligned)";
    case GEOATTN_ERR_TMA: return "TMA descriptor encoding failed";
    case GEOATTN_ERR_LAUNCH: return "CUDA kernel launch failed";
    case GEOATTN_ERR_DEVICE: return "device-side bounded wait expired";
    case GEOATTN_ERR_SCRATCH:
      return "problem needs more backward workspace than geoattn_bwd_noalloc's static 16 MiB device buffer";
  }
  return "unknown geoattn status";
}

size_t geoattn_prior_bytes(const GeoAttnShape* shape) {
  Dims d;
  if (check_shape(shape, d)) return 0;
  return 2 * prior_table_bytes(d);
}

int geoattn_prior_from_dense(const GeoAttnShape* shape, const float* dist, long long ld_dist, const float* ang,
                             long long ld_ang, void* prior, void* stream) {
  Dims d;
  if (int rc = check_shape(shape, d)) return rc;
  if (!dev_ptr(dist) || !dev_ptr(ang) || !dev_ptr(prior) || ld_dist < d.N || ld_ang < d.N) return GEOATTN_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* pt = reinterpret_cast<uint8_t*>(prior) + prior_table_bytes(d);
  dim3 grid(d.np / 32, d.np / 32), block(32, 8);
  if (d.bf16) prior_dense_kernel<true><<<grid, block, 0, st>>>(dist, ld_dist, ang, ld_ang, d.N, d.np, prior, pt);
  else prior_dense_kernel<false><<<grid, block, 0, st>>>(dist, ld_dist, ang, ld_ang, d.N, d.np, prior, pt);
  return cudaGetLastError() == cudaSuccess ? GEOATTN_OK : GEOATTN_ERR_LAUNCH;
}

int geoattn_prior_from_coords(const GeoAttnShape* shape, const double* lat_deg, const double* lon_deg,
                              const double* elev_ft, void* prior, float* dist_out, float* ang_out, void* stream) {
  Dims d;
  if (int rc = check_shape(shape, d)) return rc;
  if (!dev_ptr(lat_deg) || !dev_ptr(lon_deg) || !dev_ptr(elev_ft) || (!prior && !dist_out && !ang_out))
    return GEOATTN_ERR_INVALID;
  if ((prior && !dev_ptr(prior)) || (dist_out && !dev_ptr(dist_out)) || (ang_out && !dev_ptr(ang_out)))
    return GEOATTN_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* pt = prior ? reinterpret_cast<uint8_t*>(prior) + prior_table_bytes(d) : nullptr;
  dim3 grid(d.np / 32, d.np / 32), block(32, 8);
  if (d.bf16)
    prior_coords_kernel<true><<<grid, block, 0, st>>>(lat_deg, lon_deg, elev_ft, d.N, d.np, prior, pt, dist_out, ang_out);
  else
    prior_coords_kernel<false><<<grid, block, 0, st>>>(lat_deg, lon_deg, elev_ft, d.N, d.np, prior, pt, dist_out, ang_out);
  return cudaGetLastError() == cudaSuccess ? GEOATTN_OK : GEOATTN_ERR_LAUNCH;
}

size_t geoattn_stats_bytes(const GeoAttnShape* shape) {
  Dims d;
  if (check_shape(shape, d)) return 0;
  return (size_t)3 * d.B * d.H * d.N * 4;
}

size_t geoattn_fwd_workspace_bytes(const GeoAttnShape* shape) {
  Dims d;
  if (check_shape(shape, d)) return 0;
  return fwd_ws(d, nullptr, nullptr);
}

size_t geoattn_bwd_workspace_bytes(const GeoAttnShape* shape) {
  Dims d;
  if (check_shape(shape, d)) return 0;
  return bwd_ws(d, nullptr, nullptr, true);
}

int geoattn_fwd(const GeoAttnFwdArgs* a, void* stream) {
  if (!a) return GEOATTN_ERR_INVALID;
  Dims d;
  if (int rc = check_shape(&a->shape, d)) return rc;
  if (!dev_ptr(a->abg) || !dev_ptr(a->prior) || !dev_ptr(a->o) || !dev_ptr(a->stats) || !dev_ptr(a->workspace) ||
      !dev_ptr(a->q.data) || !dev_ptr(a->k.data) || !dev_ptr(a->v.data))
    return GEOATTN_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & (kAlign - 1)) != 0) return GEOATTN_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  FwdWs ws;
  fwd_ws(d, reinterpret_cast<uint8_t*>(a->workspace), &ws);
  if (cudaMemsetAsync(ws.status, 0, sizeof(int), st) != cudaSuccess) return GEOATTN_ERR_LAUNCH;
  TileMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  int rc;
  if (d.bf16) {
    if ((rc = map_user_bf16(&maps.q, a->q, d, kBM)) || (rc = map_user_bf16(&maps.k, a->k, d, 64)) ||
        (rc = map_user_bf16(&maps.v, a->v, d, 64)))
      return rc;
  } else {
    if ((rc = split(a->q, d, ws.qn, nullptr, st)) || (rc = split(a->k, d, ws.kn, nullptr, st)) ||
        (rc = split(a->v, d, nullptr, ws.vt, st)))
      return rc;
    if ((rc = map_planes(&maps.q, ws.qn, d, kBM)) || (rc = map_planes(&maps.k, ws.kn, d, 32)) ||
        (rc = map_transposed(&maps.v, ws.vt, d)))
      return rc;
  }
  if ((rc = map_prior(&maps.prior, a->prior, d))) return rc;
  KParams p = base_params(d, a->abg, a->shape.per_head, a->prior);
  p.o = a->o;
  for (int i = 0; i < 4; ++i) p.o_str[i] = a->o_stride[i];
  p.stats = a->stats;
  p.status = ws.status;
  p.out_tma = map_output(&maps.out0, a->o, a->o_stride, d) ? 1 : 0;
  if (d.bf16) {
    // up to 512 keys the bf16 forward keeps each row's 2^(t - m) in tensor memory and runs one score pass
    const bool one = d.N <= FwdCfg<true, 128, true>::MAX_KEYS_ONE;
    if (d.DP == 64) return one ? run_fwd<true, 64, true>(maps, p, d, st, a->events)
                               : run_fwd<true, 64>(maps, p, d, st, a->events);
    if (d.DP == 128) return one ? run_fwd<true, 128, true>(maps, p, d, st, a->events)
                                : run_fwd<true, 128>(maps, p, d, st, a->events);
    return run_fwd<true, 192>(maps, p, d, st, a->events);
  }
  if (d.DP == 64)  // single score pass up to 512 keys, as above (Q stays pooled in tensor memory)
    return d.N <= FwdCfg<false, 64, true>::MAX_KEYS_ONE ? run_fwd<false, 64, true>(maps, p, d, st, a->events)
                                                         : run_fwd<false, 64>(maps, p, d, st, a->events);
  if (d.DP == 128) return run_fwd<false, 128>(maps, p, d, st, a->events);
  return run_fwd<false, 192>(maps, p, d, st, a->events);
}

}  // extern "C"

namespace geoattn {
namespace {
// `with_ds`: the workspace holds the dS scratch (geoattn_bwd); without it (geoattn_bwd_noalloc, whose scratch is
// small) the BF16 backward forms dQ in the row pass's second sweep, as the FP32 path always does.
int backward(const GeoAttnBwdArgs* a, void* stream, bool with_ds) {
  if (!a) return GEOATTN_ERR_INVALID;
  Dims d;
  if (int rc = check_shape(&a->shape, d)) return rc;
  if (!dev_ptr(a->abg) || !dev_ptr(a->prior) || !dev_ptr(a->stats) || !dev_ptr(a->dq) || !dev_ptr(a->dk) ||
      !dev_ptr(a->dv) || !dev_ptr(a->dabg) || !dev_ptr(a->workspace) || !dev_ptr(a->o.data) ||
      !dev_ptr(a->dout.data) || !dev_ptr(a->q.data) || !dev_ptr(a->k.data) || !dev_ptr(a->v.data))
    return GEOATTN_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & (kAlign - 1)) != 0) return GEOATTN_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  BwdWs ws;
  with_ds = with_ds && uses_ds(d);
  bwd_ws(d, reinterpret_cast<uint8_t*>(a->workspace), &ws, with_ds);
  if (cudaMemsetAsync(ws.status, 0, sizeof(int), st) != cudaSuccess) return GEOATTN_ERR_LAUNCH;
  TileMaps rm, cm;
  std::memset(&rm, 0, sizeof(rm));
  std::memset(&cm, 0, sizeof(cm));
  int rc;
  if (d.bf16) {
    if ((rc = map_user_bf16(&rm.q, a->q, d, kBM)) || (rc = map_user_bf16(&rm.dout, a->dout, d, kBM)) ||
        (rc = map_user_bf16(&rm.k, a->k, d, 64)) || (rc = map_user_bf16(&rm.v, a->v, d, 64)) ||
        (rc = map_user_bf16(&cm.k, a->k, d, kBM)) || (rc = map_user_bf16(&cm.v, a->v, d, kBM)) ||
        (rc = map_user_bf16(&cm.q, a->q, d, 64)) || (rc = map_user_bf16(&cm.dout, a->dout, d, 64)))
      return rc;
  } else {
    if ((rc = split(a->q, d, ws.qn, ws.qt, st)) || (rc = split(a->k, d, ws.kn, ws.kt, st)) ||
        (rc = split(a->v, d, ws.vn, nullptr, st)) || (rc = split(a->dout, d, ws.don, ws.dot, st)))
      return rc;
    if ((rc = map_planes(&rm.q, ws.qn, d, kBM)) || (rc = map_planes(&rm.dout, ws.don, d, kBM)) ||
        (rc = map_planes(&rm.k, ws.kn, d, 32)) || (rc = map_planes(&rm.v, ws.vn, d, 32)) ||
        (rc = map_transposed(&rm.kt, ws.kt, d)) || (rc = map_planes(&cm.k, ws.kn, d, kBM)) ||
        (rc = map_planes(&cm.v, ws.vn, d, kBM)) || (rc = map_planes(&cm.q, ws.qn, d, 32)) ||
        (rc = map_planes(&cm.dout, ws.don, d, 32)) || (rc = map_transposed(&cm.qt, ws.qt, d)) ||
        (rc = map_transposed(&cm.dot, ws.dot, d)))
      return rc;
  }
  if ((rc = map_prior(&rm.prior, a->prior, d)) ||
      (rc = map_prior(&cm.prior, reinterpret_cast<const uint8_t*>(a->prior) + prior_table_bytes(d), d)))
    return rc;
  KParams p = base_params(d, a->abg, a->shape.per_head, a->prior);
  p.dout = a->dout.data;
  for (int i = 0; i < 4; ++i) {
    p.do_str[i] = a->dout.stride[i];
    p.dq_str[i] = a->dq_stride[i];
    p.dk_str[i] = a->dk_stride[i];
    p.dv_str[i] = a->dv_stride[i];
  }
  p.dq = a->dq;
  p.dk = a->dk;
  p.dv = a->dv;
  p.stats = const_cast<float*>(a->stats);
  p.rowrec = ws.rowrec;
  p.part = ws.part;
  p.status = ws.status;
  KParams prow = p, pcol = p;
  prow.out_tma = map_output(&rm.out0, a->dq, a->dq_stride, d) ? 1 : 0;
  pcol.out_tma =
      (map_output(&cm.out0, a->dk, a->dk_stride, d) && map_output(&cm.out1, a->dv, a->dv_stride, d)) ? 1 : 0;
  if (with_ds && !d.bf16 && d.DP > 64) {
    TileMaps qm;
    std::memset(&qm, 0, sizeof(qm));
    if ((rc = map_ds_f32(&cm.dsT, ws.dsT, d, kBM)) || (rc = map_ds_f32(&qm.dsT, ws.dsT, d, 32)) ||
        (rc = map_transposed(&qm.kt, ws.kt, d)))
      return rc;
    rc = d.DP == 128 ? run_bwd_ds_wide<128>(rm, cm, qm, prow, pcol, prow, d, st, a->events)
                     : run_bwd_ds_wide<192>(rm, cm, qm, prow, pcol, prow, d, st, a->events);
  } else if (with_ds && !d.bf16) {
    TileMaps qm;
    std::memset(&qm, 0, sizeof(qm));
    if ((rc = map_ds_f32(&cm.dsT, ws.dsT, d, 32)) || (rc = map_ds_f32(&qm.dsT, ws.dsT, d, kBM)) ||
        (rc = map_transposed(&qm.kt, ws.kt, d)))
      return rc;
    rc = run_bwd_ds_f32(rm, cm, qm, prow, pcol, prow, d, st, a->events);
  } else if (with_ds) {
    TileMaps qm;
    std::memset(&qm, 0, sizeof(qm));
    if ((rc = map_dsT(&cm.dsT, ws.dsT, d, kBM)) || (rc = map_dsT(&qm.dsT, ws.dsT, d, 64)) ||
        (rc = map_user_bf16(&qm.k, a->k, d, 64)))
      return rc;
    KParams pdq = prow;  // dQ output map and strides
    qm.out0 = rm.out0;
    if (d.DP == 64) rc = run_bwd_ds<64>(rm, cm, qm, prow, pcol, pdq, d, st, a->events);
    else if (d.DP == 128) rc = run_bwd_ds<128>(rm, cm, qm, prow, pcol, pdq, d, st, a->events);
    else rc = run_bwd_ds<192>(rm, cm, qm, prow, pcol, pdq, d, st, a->events);
  } else if (d.bf16) {
    if (d.DP == 64) rc = run_bwd<true, 64>(rm, cm, prow, pcol, d, st, a->events);
    else if (d.DP == 128) rc = run_bwd<true, 128>(rm, cm, prow, pcol, d, st, a->events);
    else rc = run_bwd<true, 192>(rm, cm, prow, pcol, d, st, a->events);
  } else {
    // fp32 always keeps the dS scratch (geoattn_bwd); the allocation-free entry rejects fp32 before this point
    rc = GEOATTN_ERR_UNSUPPORTED;
  }
  if (rc) return rc;
  finalize_abg_kernel<<<dim3(3, d.nabg), 256, 0, st>>>(ws.part, d.B, d.H, d.nrb, a->shape.per_head, a->dabg);
  return cudaGetLastError() == cudaSuccess ? GEOATTN_OK : GEOATTN_ERR_LAUNCH;
}
}  // namespace
}  // namespace geoattn

namespace geoattn {
// Address of geoattn_bwd_noalloc's static scratch on the current device (defined with the array below).
int noalloc_scratch(void** out);
}  // namespace geoattn

extern "C" {

int geoattn_bwd(const GeoAttnBwdArgs* a, void* stream) { return backward(a, stream, true); }

int geoattn_wait_selftest(void* status_word, void* stream) {
  if (!dev_ptr(status_word) || (reinterpret_cast<uintptr_t>(status_word) & 3) != 0) return GEOATTN_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(status_word, 0, sizeof(int), st) != cudaSuccess) return GEOATTN_ERR_LAUNCH;
  wait_selftest_kernel<<<1, 1, 0, st>>>(reinterpret_cast<int*>(status_word));
  return cudaGetLastError() == cudaSuccess ? GEOATTN_OK : GEOATTN_ERR_LAUNCH;
}

int geoattn_read_status(const void* workspace, int* status, void* stream) {
  if (!status) return GEOATTN_ERR_INVALID;
  if (!workspace) {  // geoattn_bwd_noalloc's status word: the first word of the current device's static scratch
    void* scratch = nullptr;
    if (int rc = geoattn::noalloc_scratch(&scratch)) return rc;
    workspace = scratch;
  }
  if (!dev_ptr(workspace)) return GEOATTN_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return GEOATTN_ERR_LAUNCH;
  if (cudaStreamSynchronize(st) != cudaSuccess) return GEOATTN_ERR_LAUNCH;
  return GEOATTN_OK;
}

}  // extern "C"

// ===============================================================================================================
// Allocation-free backward.
//
// Some callers of this library cannot allocate device memory for the backward's workspace: plugin or custom-op
// hosts that own every device buffer and hand an operator only its inputs and outputs, and code whose memory
// plan is fixed up front (an allocation there would synchronise the device or break the plan). For them,
// geoattn_bwd_noalloc takes its scratch (row records, bias-gradient partials, status word) from the static device
// array below instead of args->workspace. The array is 16 MiB in every device that loads the library, for the
// life of the process. Every call shares it and it keeps the last call's contents, so calls that overlap on the
// GPU (other streams, other threads) race; the status word is cleared at the start of each call and every other
// byte a call reads is written earlier in the same call. The first call on a device looks the array's address up
// (cudaGetSymbolAddress, that device current) and caches it; make that first call outside any stream capture.
// ===============================================================================================================
namespace geoattn {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
}  // namespace

int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return GEOATTN_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return GEOATTN_ERR_INVALID;
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return GEOATTN_ERR_LAUNCH;
    addr[dev] = p;
  }
  *out = addr[dev];
  return GEOATTN_OK;
}
}  // namespace geoattn

extern "C" int geoattn_bwd_noalloc(const GeoAttnBwdArgs* a, void* stream) {
  using namespace geoattn;
  if (!a) return GEOATTN_ERR_INVALID;
  Dims d;
  if (int rc = check_shape(&a->shape, d)) return rc;
  if (!d.bf16) return GEOATTN_ERR_UNSUPPORTED;  // the FP32 path's operand planes do not fit a modest static buffer
  if (bwd_ws(d, nullptr, nullptr, false) > kNoAllocScratchBytes) return GEOATTN_ERR_SCRATCH;
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  GeoAttnBwdArgs b = *a;
  b.workspace = scratch;
  return backward(&b, stream, false);
}
