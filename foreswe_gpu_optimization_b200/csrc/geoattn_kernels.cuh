// Geo-biased station attention for sm_100a: forward, backward row pass, backward key pass.
//
// Operator (fore_swe/custom_encoder_model.py:25-39):
//   S = Q K^T / sqrt(d);  P1 = softmax(S);  Z = alpha*P1 + beta*Dp + gamma*Ap;  P2 = softmax(Z);  O = P2 V
// with the geo prior Dp = 1/(1+dist_km), Ap = 1/(1+angle_deg) read from a table built once per station geometry
// (prior_coords_kernel / prior_dense_kernel in geoattn.cu).
//
// All kernels share one CTA shape: EW element-wise warpgroups (EW = 2 for bf16, 1 for fp32; a thread of warp w owns
// TMEM lane 32*(w%4) + lane, i.e. one row of every 128-row accumulator, and warpgroup w/4 owns every EW-th 32-column
// piece of each chunk), then one warp that issues the operand TMA loads, one that issues tcgen05.mma and one that
// stages the geo-prior tile of each chunk into shared memory (so the prior ring and the operand rings refill
// independently). Every MMA is M = 128 with fp32 accumulators in tensor memory. Shared-memory operand tiles use the
// 128-byte swizzle; one "region" is rows x 128 bytes (64 bf16 or 32 fp32 along the contiguous dimension). Where
// shared memory is full the prior is read from L2 directly. bf16 outputs (O, dQ, dK, dV) leave through a swizzled
// shared-memory tile and a TMA store; the operands of the next tile are prefetched into L2 while this one runs.
//
// fp32 storage (TF32 MMAs): operands come as round-to-nearest hi/lo planes and the score-shaped products take three
// terms (hi.hi + hi.lo + lo.hi). At head dim 64 the kernels are "pooled": the 128-row A operand of the score MMAs is
// copied into tensor memory once per tile (tcgen05.cp) and its shared-memory landing zone then holds the chunk
// rings; the forward issues its score MMAs over pairs of 32-key chunks. Above 64 ("wide") the score operands stream
// through slots that each hold one 32-wide head-dim chunk.
//
// Softmax #1 runs in log2 units: t = acc * (log2(e)/sqrt(d)) with row max m. Once the row sum l1 is known, the
// normalised probability is one fused multiply-add and one exp2: P1 = 2^(fma(acc, log2(e)/sqrt(d), -m1)) with
// m1 = m + log2(l1). Softmax #2 needs no running max: Z <= c = |alpha|+|beta|+|gamma| whenever dist, ang >= 0, so
// e = 2^((Z - c) log2 e) lies in (0, 1]; with its row sum l2, P2 = 2^(Z log2 e - c2), c2 = c log2 e + log2(l2).
#pragma once
#include <cuda_fp16.h>

#include <type_traits>

#include "sm100.cuh"

namespace geoattn {

constexpr int kBM = 128;        // rows per tile (TMEM lanes)
constexpr int kSmemPerBlock = 227 * 1024;  // opt-in shared memory per block (static + dynamic)

// Dynamic shared memory of every attention kernel. The 1024-byte alignment (what the 128-byte-swizzled TMA and MMA
// tiles need) is part of the declaration: the compiler pads the static shared data in front of it to a multiple of
// 1024 bytes, so no slack is allocated for aligning by hand. A kernel that finds it misaligned anyway reports an
// error instead of running (smem_misaligned).
extern __shared__ __align__(1024) uint8_t smem_raw[];

__device__ __forceinline__ bool smem_misaligned(int* status) {
  if ((smem_u32(smem_raw) & 1023u) == 0) return false;
  if (threadIdx.x == 0 && status) atomicCAS(status, kDevOk, kDevSmemMisaligned);
  return true;
}
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ constexpr int pow2_cols(int n) { return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512; }

// ---------------------------------------------------------------------------------------------------------------
// Launch parameters shared by the kernels (element strides; pointers are device pointers).
// ---------------------------------------------------------------------------------------------------------------
struct KParams {
  int B, H, N, D;
  int nrb;              // ceil(N / 128)
  int np;               // prior table row stride (pairs) = nrb * 128
  float scale_log2;     // log2(e) / sqrt(D)
  float inv_sqrt_d;     // 1 / sqrt(D)
  const float* abg;     // alpha[nabg], beta[nabg], gamma[nabg]
  int per_head;         // nabg == H (else 1)
  const void* prior;    // [np][np] pairs (Dp, Ap): half2 (bf16 path) or float2 (fp32 path)
  const void* priorT;   // transposed table
  void* o;              // forward output, strides o_str
  long long o_str[4];
  const void* dout;     // backward: dO
  long long do_str[4];
  void* dq;
  long long dq_str[4];
  void* dk;
  long long dk_str[4];
  void* dv;
  long long dv_str[4];
  float* stats;         // forward -> backward: [3][B*H*N] = m (log2 units), l1, l2
  float* rowrec;        // backward row records [B*H][nchp][NREC][CH] = m1, c2, delta1, delta2[, b] (chunk-blocked)
  int nchp;             // record chunks per b*h = np / CH
  double* part;         // [B*H*nrb][3] partial d(alpha), d(beta), d(gamma)
  int* status;          // device status word (0 = ok)
  int out_tma;          // outputs leave through TMA stores (bf16, TMA-compatible output tensors)
};

struct Abg {
  float a, b, g, c;
};
__device__ __forceinline__ Abg load_abg(const KParams& p, int h) {
  const int n = p.per_head ? p.H : 1;
  const int i = p.per_head ? h : 0;
  Abg r;
  r.a = __ldg(p.abg + i);
  r.b = __ldg(p.abg + n + i);
  r.g = __ldg(p.abg + 2 * n + i);
  r.c = fabsf(r.a) + fabsf(r.b) + fabsf(r.g);
  return r;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Element-wise warps wait warp-uniformly, so the collective tcgen05.ld that follows is never divergent.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, ctx));
}

// Named barrier among the element-wise threads only (nthreads = 128 * EW).
__device__ __forceinline__ void ew_sync(int nthreads) { asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory"); }

// Byte offset of 16-byte chunk `q` (0..7) of row `r` inside a 128-byte-swizzled region.
__device__ __forceinline__ uint32_t sw128(int r, int q) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((q ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------------------------------------------
// Prior pieces: 32 consecutive (Dp, Ap) pairs of one row. The bf16 path keeps them packed as half2 (one register per
// pair) and widens each pair where it is used; the fp32 path holds float pairs.
// ---------------------------------------------------------------------------------------------------------------
template <bool F16>
struct Prior32 {
  float dp[32], ap[32];
  __device__ __forceinline__ void get(int j, float& d, float& a) const {
    d = dp[j];
    a = ap[j];
  }
};
template <>
struct Prior32<true> {
  uint32_t w[32];
  __device__ __forceinline__ void get(int j, float& d, float& a) const {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    d = f.x;
    a = f.y;
  }
};

template <bool F16>
__device__ __forceinline__ void load_prior32(const void* table, int np, int row, int col0, Prior32<F16>& pr) {
  if constexpr (F16) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __half2*>(table) + (size_t)row * np + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = __ldg(src + i);
      pr.w[4 * i] = u.x;
      pr.w[4 * i + 1] = u.y;
      pr.w[4 * i + 2] = u.z;
      pr.w[4 * i + 3] = u.w;
    }
  } else {
    const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float2*>(table) + (size_t)row * np + col0);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 f = __ldg(src + i);
      pr.dp[2 * i] = f.x;
      pr.ap[2 * i] = f.y;
      pr.dp[2 * i + 1] = f.z;
      pr.ap[2 * i + 1] = f.w;
    }
  }
}

// Prior tile staged by TMA: [128 rows][64 pair-columns as 32-bit words] as two 128-byte-swizzled regions of
// 128 x 128 B. bf16 path: half2 pairs, piece p (32 pairs) = region p. fp32 path: float2 pairs, the single piece
// (32 pairs) spans both regions (16 pairs each).
constexpr int kPriorTileBytes = 2 * kBM * 128;

template <bool F16>
__device__ __forceinline__ void prior32_smem(const uint8_t* tile, int r, int piece, Prior32<F16>& pr) {
  if constexpr (F16) {
    const uint8_t* reg = tile + piece * (kBM * 128);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(reg + sw128(r, q));
      pr.w[4 * q] = u.x;
      pr.w[4 * q + 1] = u.y;
      pr.w[4 * q + 2] = u.z;
      pr.w[4 * q + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int rg = 0; rg < 2; ++rg)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 f = *reinterpret_cast<const float4*>(tile + rg * (kBM * 128) + sw128(r, q));
        pr.dp[rg * 16 + q * 2] = f.x;
        pr.ap[rg * 16 + q * 2] = f.y;
        pr.dp[rg * 16 + q * 2 + 1] = f.z;
        pr.ap[rg * 16 + q * 2 + 1] = f.w;
      }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Operand staging of element-wise results into a K-major A tile (one 128-byte region, 128 rows).
// bf16: 32 values = 4 chunks of 8.  fp32 (TF32): 32 values = 8 chunks of 4, rounded to TF32 (nearest).
// `piece` selects which 32 columns of the 128-byte row (bf16: 0..1; fp32: 0 only).
// ---------------------------------------------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void stage_row32(uint8_t* region, int row, int piece, const float (&v)[32]) {
  if constexpr (BF16) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 b2 = __floats2bfloat162_rn(v[q * 8 + 2 * k], v[q * 8 + 2 * k + 1]);
        w[k] = *reinterpret_cast<uint32_t*>(&b2);
      }
      *reinterpret_cast<uint4*>(region + sw128(row, piece * 4 + q)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 f = make_float4(round_tf32(v[q * 4]), round_tf32(v[q * 4 + 1]), round_tf32(v[q * 4 + 2]),
                             round_tf32(v[q * 4 + 3]));
      *reinterpret_cast<float4*>(region + sw128(row, q)) = f;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Global stores of one accumulator row (32 values starting at column d0), masked to d < D.
// ---------------------------------------------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void store_row32(void* base, long long off, long long sd, int d0, int D, const float (&v)[32],
                                            float scale) {
  if constexpr (BF16) {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(base) + off;
    if (sd == 1 && d0 + 32 <= D && ((reinterpret_cast<uintptr_t>(p + d0) & 15) == 0)) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(v[q * 8 + 2 * k] * scale, v[q * 8 + 2 * k + 1] * scale);
          w[k] = *reinterpret_cast<uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(p + d0 + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (d0 + i < D) p[(d0 + i) * sd] = __float2bfloat16_rn(v[i] * scale);
    }
  } else {
    float* p = reinterpret_cast<float*>(base) + off;
    if (sd == 1 && d0 + 32 <= D && ((reinterpret_cast<uintptr_t>(p + d0) & 15) == 0)) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(p + d0 + q * 4) =
            make_float4(v[q * 4] * scale, v[q * 4 + 1] * scale, v[q * 4 + 2] * scale, v[q * 4 + 3] * scale);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (d0 + i < D) p[(d0 + i) * sd] = v[i] * scale;
    }
  }
}

template <bool BF16>
__device__ __forceinline__ float load_elem(const void* base, long long off) {
  if constexpr (BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[off]);
  else return reinterpret_cast<const float*>(base)[off];
}

// ---------------------------------------------------------------------------------------------------------------
// Tile configuration. KB = elements per 128-byte row; every key/query chunk is KB wide so that a chunk row of the
// element-wise outputs (P, dS, P2^T, dS^T) is exactly one swizzle row, and a chunk row of the prior (CH pairs) is
// 256 bytes = two swizzle regions.
// ---------------------------------------------------------------------------------------------------------------
template <bool BF16, int DP_>
struct Tile {
  static constexpr bool kBF16 = BF16;
  static constexpr int DP = DP_;
  static constexpr int EB = BF16 ? 2 : 4;
  static constexpr int KB = 128 / EB;       // 64 bf16 / 32 fp32
  static constexpr int KS = BF16 ? 16 : 8;  // MMA K per instruction
  static constexpr int NKB = DP / KB;       // 128-byte regions along D
  static constexpr int CH = KB;             // chunk width (keys or queries)
  static constexpr int PIECES = CH / 32;    // 32-column pieces per chunk
  static constexpr int PL = BF16 ? 1 : 2;   // planes of Q, K, V, dO: hi[, lo]
  static constexpr int NTERM = BF16 ? 1 : 3;
  static constexpr Kind KIND = BF16 ? Kind::kF16 : Kind::kTF32;
  static constexpr uint32_t FMT = BF16 ? 1 : 2;
  static constexpr int EW = BF16 ? 2 : 1;   // element-wise warpgroups
  static constexpr int EWT = 128 * EW;      // element-wise threads
  // row records per query row: m1, c2, delta1, delta2; fp32 above head dim 64 also b = sum P2 P1, for the key pass's
  // d(alpha) = sum dZ (P1 - b)
  static constexpr int NREC = (!BF16 && DP_ > 64) ? 5 : 4;
  static constexpr int NTHREADS = EWT + 96;
  static constexpr int TMA_WARP = 4 * EW;
  static constexpr int MMA_WARP = 4 * EW + 1;
  static constexpr int PR_WARP = 4 * EW + 2;  // geo-prior tiles
  static_assert(DP % KB == 0, "padded head dim must be a whole number of 128-byte regions");
  static_assert(PIECES == EW, "each warpgroup owns exactly one piece of every chunk");
};

// Element-wise thread identity.
struct Ew {
  int r;          // TMEM lane = row of the 128-row accumulator
  int wg;         // warpgroup
  uint32_t lane_base;
};
__device__ __forceinline__ Ew ew_id(uint32_t tmem) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  Ew e;
  e.r = (warp & 3) * 32 + lane;
  e.wg = warp >> 2;
  e.lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  return e;
}

// Issue acc[128 x NB] (+)= A[128 x KD] . B[NB x KD]^T, both K-major, regions of 128 x 128 B (A) and NB x 128 B (B);
// KD = DP (the whole head dimension) or KB (one 128-byte head-dim chunk, added to the accumulator when
// `accumulate`). With NTERM == 3 the product is hi*hi + hi*lo + lo*hi (planes 0/1 at a_plane/b_plane byte strides).
template <class T, int NB, int KD = T::DP>
__device__ __forceinline__ void mma_qk(uint32_t tmem_acc, uint32_t a_base, uint32_t a_plane, uint32_t b_base,
                                       uint32_t b_plane, bool accumulate = false) {
  constexpr uint32_t idesc = instr_desc(T::FMT, 0, 0, 128, NB);
  constexpr int STEPS = KD / T::KS;
  int first = accumulate ? 0 : 1;
#pragma unroll
  for (int term = 0; term < T::NTERM; ++term) {
    const uint32_t ap = (term == 2) ? a_plane : 0;  // (hi,hi), (hi,lo), (lo,hi)
    const uint32_t bp = (term == 1) ? b_plane : 0;
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      const int kb = (s * T::KS) / T::KB;
      const uint32_t w = (uint32_t)((s * T::KS) % T::KB) * T::EB;
      const uint64_t ad = smem_desc_sw128(a_base + ap + kb * (128 * 128) + w, 16, 1024);
      const uint64_t bd = smem_desc_sw128(b_base + bp + kb * (NB * 128) + w, 16, 1024);
      mma_ss<T::KIND>(tmem_acc, ad, bd, idesc, first ? 0u : 1u);
      first = 0;
    }
  }
}

// Tensor-memory columns of a 128-row operand held as an MMA A operand: DP elements per plane, 32 bits per column.
template <class T>
constexpr int kAColsPerPlane = T::DP * T::EB / 4;

// Copies a resident 128-row K-major operand (planes hi[, lo] at a_plane byte strides, NKB swizzled regions each)
// from shared memory into tensor memory as an A operand: plane pl, head-dim element d -> lane = row, column
// tmem_a + pl * kAColsPerPlane + d * EB / 4. One 128x256b copy per MMA K step. Every MMA that read the previous
// contents of these columns must have completed before this is issued (copies after MMAs are not ordered).
template <class T>
__device__ __forceinline__ void cp_operand_tmem(uint32_t tmem_a, uint32_t a_base, uint32_t a_plane) {
  constexpr int STEPS = T::DP / T::KS;
  static_assert(T::KS * T::EB == 32, "one MMA K step is 256 bits");
#pragma unroll
  for (int pl = 0; pl < T::PL; ++pl)
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      const int kb = (s * T::KS) / T::KB;
      const uint32_t w = (uint32_t)((s * T::KS) % T::KB) * T::EB;
      tmem_cp_128x256b(tmem_a + pl * kAColsPerPlane<T> + s * 8,
                       smem_desc_sw128(a_base + pl * a_plane + kb * (128 * 128) + w, 16, 1024));
    }
}

// The shared-memory source of tcgen05.cp copies may be rewritten only once the copies have read it. A commit issued
// right after the copies does not wait for them, and neither does an MMA that reads only the last copied columns
// (measured: repeated runs differed where the next chunk's TMA overwrote a copied plane). This issues one MMA per
// copied 8-column block of an operand (each ordered after the copy it reads) into 32 scratch accumulator columns
// `acc`, with B any 32 x 32-byte swizzled slice of shared memory that nothing writes meanwhile; a commit issued after
// them tracks every copy.
template <class T>
__device__ __forceinline__ void cp_drain_operand(uint32_t acc, uint32_t tmem_a, uint32_t smem_b) {
  constexpr uint32_t idesc = instr_desc(T::FMT, 0, 0, 128, 32);
  const uint64_t bd = smem_desc_sw128(smem_b, 16, 1024);
#pragma unroll
  for (int pl = 0; pl < T::PL; ++pl)
#pragma unroll
    for (int s = 0; s < T::DP / T::KS; ++s) mma_ts<T::KIND>(acc, tmem_a + pl * kAColsPerPlane<T> + s * 8, bd, idesc, 0u);
}

// mma_qk with A = the whole head dimension of a tensor-memory operand copied by cp_operand_tmem, B in shared memory.
template <class T, int NB>
__device__ __forceinline__ void mma_qk_ts(uint32_t tmem_acc, uint32_t tmem_a, uint32_t b_base, uint32_t b_plane) {
  constexpr uint32_t idesc = instr_desc(T::FMT, 0, 0, 128, NB);
  constexpr int STEPS = T::DP / T::KS;
  int first = 1;
#pragma unroll
  for (int term = 0; term < T::NTERM; ++term) {
    const uint32_t ap = (term == 2) ? kAColsPerPlane<T> : 0;  // (hi,hi), (hi,lo), (lo,hi)
    const uint32_t bp = (term == 1) ? b_plane : 0;
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      const int kb = (s * T::KS) / T::KB;
      const uint32_t w = (uint32_t)((s * T::KS) % T::KB) * T::EB;
      const uint64_t bd = smem_desc_sw128(b_base + bp + kb * (NB * 128) + w, 16, 1024);
      mma_ts<T::KIND>(tmem_acc, tmem_a + ap + s * 8, bd, idesc, first ? 0u : 1u);
      first = 0;
    }
  }
}

// Issue acc[128 x DP] (+)= P[128 x CH] . V where P is one K-major region (128 x 128 B) and V is either
//   bf16: the natural chunk [CH rows x DP] (MN-major B: regions per 64-wide D block of CH x 128 B), or
//   fp32: the transposed chunk [DP rows x CH] (K-major B: one region of DP x 128 B).
template <class T>
__device__ __forceinline__ void mma_pv(uint32_t tmem_acc, uint32_t p_base, uint32_t v_base, bool accumulate) {
  constexpr int STEPS = T::CH / T::KS;  // 4
  if constexpr (T::kBF16) {
    constexpr uint32_t idesc = instr_desc(T::FMT, 0, 1, 128, T::DP);
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      const uint64_t ad = smem_desc_sw128(p_base + s * 32, 16, 1024);
      const uint64_t bd = smem_desc_sw128(v_base + s * T::KS * 128, T::CH * 128, 1024);
      mma_ss<T::KIND>(tmem_acc, ad, bd, idesc, (accumulate || s > 0) ? 1u : 0u);
    }
  } else {
    constexpr uint32_t idesc = instr_desc(T::FMT, 0, 0, 128, T::DP);
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      const uint64_t ad = smem_desc_sw128(p_base + s * 32, 16, 1024);
      const uint64_t bd = smem_desc_sw128(v_base + s * 32, 16, 1024);
      mma_ss<T::KIND>(tmem_acc, ad, bd, idesc, (accumulate || s > 0) ? 1u : 0u);
    }
  }
}

// TMA of one operand tile: `nrows` rows starting at `row0`, all NKB regions, planes 0..npl-1.
// 4-D maps: (d, n, h, b[+plane*B]) for natural tensors.
template <class T>
__device__ __forceinline__ void tma_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int nrows, int row0,
                                         int h, int b, int B, int npl) {
  for (int pl = 0; pl < npl; ++pl)
    for (int kb = 0; kb < T::NKB; ++kb)
      tma_load_4d(dst + (size_t)(pl * T::NKB + kb) * nrows * 128, map, bar, kb * T::KB, row0, h, b + pl * B);
}
// fp32 head dims above 64 ("wide"): the score-shaped products stream their operands through a ring of slots, each
// holding one 32-wide head-dim chunk dc of a 128-row A tile and of a BROWS-row B part (BROWS / 32 consecutive 32-row
// chunks: the wide kernels issue their score MMAs over chunk pairs, BROWS = 64), hi and lo planes:
// [plane 0: A (128 x 128 B) | B (BROWS x 128 B)][plane 1: A | B]. The MMA accumulates the head-dim chunks' products.
template <int BROWS>
constexpr int kSlotPlaneBytesRows = (kBM + BROWS) * 128;
template <class T, int BROWS>
__device__ __forceinline__ void tma_slot_rows(uint8_t* slot, uint64_t* bar, const CUtensorMap* amap, int arow0,
                                              const CUtensorMap* bmap, int brow0, int dc, int h, int b, int B,
                                              bool a_hi = true) {
  constexpr int SPB = kSlotPlaneBytesRows<BROWS>;
  for (int pl = 0; pl < 2; ++pl) {
    if (pl > 0 || a_hi) tma_load_4d(slot + pl * SPB, amap, bar, dc * T::KB, arow0, h, b + pl * B);
    for (int r = 0; r < BROWS; r += 32)
      tma_load_4d(slot + pl * SPB + (kBM + r) * 128, bmap, bar, dc * T::KB, brow0 + r, h, b + pl * B);
  }
}
template <class T, int BROWS>
__device__ __forceinline__ void mma_slot_rows(uint32_t tmem_acc, uint32_t slot, bool accumulate) {
  static_assert(!T::kBF16 && T::CH == 32, "slots carry fp32 planes with 32-row B chunks");
  constexpr int SPB = kSlotPlaneBytesRows<BROWS>;
  mma_qk<T, BROWS, T::KB>(tmem_acc, slot, SPB, slot + kBM * 128, SPB, accumulate);
}
// The same product with the A operand's hi plane resident in tensor memory (columns tmem_ah: the 32 fp32 of this
// head-dim chunk, lane = row): (hi,hi) and (hi,lo) read A from tensor memory, (lo,hi) the lo plane from the slot, so
// the slot needs no hi plane of A.
template <class T, int BROWS>
__device__ __forceinline__ void mma_slot_rows_ah(uint32_t tmem_acc, uint32_t slot, uint32_t tmem_ah, bool accumulate) {
  static_assert(!T::kBF16 && T::CH == 32 && T::NTERM == 3, "slots carry fp32 planes with 32-row B chunks");
  constexpr int SPB = kSlotPlaneBytesRows<BROWS>;
  constexpr uint32_t idesc = instr_desc(T::FMT, 0, 0, 128, BROWS);
  const uint32_t b0 = slot + kBM * 128;
  int first = accumulate ? 0 : 1;
#pragma unroll
  for (int term = 0; term < 3; ++term) {
#pragma unroll
    for (int s = 0; s < T::KB / T::KS; ++s) {  // K = 8 elements (32 bytes, 8 columns) per MMA
      const uint64_t bd = smem_desc_sw128(b0 + (term == 1 ? SPB : 0) + s * 32, 16, 1024);
      if (term < 2)
        mma_ts<T::KIND>(tmem_acc, tmem_ah + s * 8, bd, idesc, first ? 0u : 1u);
      else
        mma_ss<T::KIND>(tmem_acc, smem_desc_sw128(slot + SPB + s * 32, 16, 1024), bd, idesc, 1u);
      first = 0;
    }
  }
}
// Copies the hi plane of a slot's 128-row A chunk (one head-dim chunk, 128 rows x 128 B) into tensor memory as an A
// operand (columns tmem_ah .. tmem_ah + 31). Every MMA that read those columns before must have completed.
template <class T>
__device__ __forceinline__ void cp_slot_a_hi(uint32_t tmem_ah, uint32_t slot) {
#pragma unroll
  for (int s = 0; s < T::KB / T::KS; ++s) tmem_cp_128x256b(tmem_ah + s * 8, smem_desc_sw128(slot + s * 32, 16, 1024));
}
// Two consecutive chunks (rows c*CH .. c*CH + 2*CH) of a natural operand, hi[/lo] planes, into one ring slot laid out
// [plane][region][2*CH rows x 128 B], so that the slot is a 2*CH-row K-major B operand.
template <class T>
__device__ __forceinline__ void tma_pair(uint8_t* slot, const CUtensorMap* map, uint64_t* bar, int c, int h, int b,
                                         int B) {
  for (int pl = 0; pl < T::PL; ++pl)
    for (int kb = 0; kb < T::NKB; ++kb)
      for (int half = 0; half < 2; ++half)
        tma_load_4d(slot + ((pl * T::NKB + kb) * 2 + half) * (T::CH * 128), map, bar, kb * T::KB,
                    (c + half) * T::CH, h, b + pl * B);
}
// Transposed fp32 plane chunk: DP rows (d) x 32 columns (n) starting at column n0 -> one region of DP x 128 B.
__device__ __forceinline__ void tma_tileT(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int n0, int h, int b) {
  tma_load_4d(dst, map, bar, n0, 0, h, b);
}
// Prior tile of chunk c: rows [row0, row0+128), pair columns [c*CH, c*CH+CH) = 64 32-bit words.
__device__ __forceinline__ void tma_prior(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0, int c) {
  tma_load_2d(dst, map, bar, c * 64, row0);
  tma_load_2d(dst + kBM * 128, map, bar, c * 64 + 32, row0);
}

struct TileMaps {
  CUtensorMap q, k, v, dout, kt, qt, dot, prior;  // unused entries are left zero
  CUtensorMap out0, out1;                         // bf16 output stores: fwd O; rows / dQ GEMM dQ; cols dK, dV
  CUtensorMap dsT;                                // dS^T scratch [b*h][key][query]: cols stores, dQ GEMM loads
};

// L2 prefetch of a row block of a natural operand (boxes of `rows` rows, all NKB regions and planes).
template <class T>
__device__ __forceinline__ void prefetch_tile(const CUtensorMap* map, int row0, int h, int b, int B, int npl) {
  for (int pl = 0; pl < npl; ++pl)
    for (int kb = 0; kb < T::NKB; ++kb) tma_prefetch_4d(map, kb * T::KB, row0, h, b + pl * B);
}
// L2 prefetch of all rows [0, N) of a natural operand in boxes of CH rows.
template <class T>
__device__ __forceinline__ void prefetch_rows(const CUtensorMap* map, int N, int h, int b, int B, int npl) {
  for (int r0 = 0; r0 < N; r0 += T::CH) prefetch_tile<T>(map, r0, h, b, B, npl);
}

// bf16 output epilogue: 32 accumulator columns [d0, d0+32) of row r, scaled and rounded, into a swizzled tile of
// 128-row x 64-column regions (the layout a TMA store of box (64, 128) reads).
__device__ __forceinline__ void stage_out32(uint8_t* tile, int r, int d0, float (&v)[32], float scale) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] *= scale;
  stage_row32<true>(tile + (d0 / 64) * (kBM * 128), r, (d0 % 64) / 32, v);
}
// Loads NP 32-column pieces of this thread's accumulator row (TMEM columns c0, c0 + step, ...; also the output
// columns) with a single wait, then stages them scaled and rounded into the swizzled output tile.
template <int NP>
__device__ __forceinline__ void stage_acc(uint32_t tbase, int c0, int step, uint8_t* tile, int r, float scale) {
  uint32_t v[NP][32];
#pragma unroll
  for (int i = 0; i < NP; ++i) tmem_ld32_issue(tbase + c0 + i * step, v[i]);
  tmem_wait32(v[0]);
#pragma unroll
  for (int i = 1; i < NP; ++i) tmem_pin32(v[i]);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[i][j]);
    stage_out32(tile, r, c0 + i * step, f, scale);
  }
}

// Stores the staged tile (row block row0 of (b, h)) once every element-wise thread has staged its row. Called by all
// element-wise threads; thread 0 issues the stores. The caller's next rewrite of `tile` must follow a
// bulk_wait_read0() by thread 0 and a barrier among the element-wise threads.
template <class T>
__device__ __forceinline__ void store_tile(const CUtensorMap* map, const uint8_t* tile, int D, int row0, int h, int b,
                                           bool issue) {
  fence_proxy_async_smem();
  ew_sync(T::EWT);
  if (threadIdx.x == 0 && issue) {
    for (int kb = 0; kb < T::NKB && kb * 64 < D; ++kb) tma_store_4d(map, tile + kb * (kBM * 128), kb * 64, row0, h, b);
    bulk_commit();
  }
}

// ===============================================================================================================
// Forward: one CTA per (128-query row block, b*h). Pass A: row max / sum of softmax #1 over all key chunks.
// Pass B: recompute S (or, with a single score pass, read back the values pass A kept), form P1, Z and
// e = 2^((Z-c) log2 e), accumulate O += e V and l2 = sum e.
// ===============================================================================================================
template <bool BF16, int DP, bool ONE = false>
struct FwdCfg : Tile<BF16, DP> {
  using T = Tile<BF16, DP>;
  // ONE (bf16 up to head dim 128, fp32 at head dim 64; up to 512 keys): a single score pass. Pass A keeps, per row,
  // each chunk pair's 2^(t - m_c) against the running max m_c as fp16 pairs in tensor memory (256 columns for 512
  // keys); pass B reads them back, P1 = 2^(t - m_c) 2^(m_c - m1), and issues no score MMAs. bf16: Q stays in shared
  // memory (its tensor-memory columns hold the stored values) and the score MMAs take single 64-key chunks into two
  // buffers; fp32: Q stays pooled in tensor memory and the score MMAs take one pair of 32-key chunks (both buffers),
  // issued as soon as the element-wise warps have loaded the previous pair.
  static_assert(!ONE || (BF16 && DP <= 128) || (!BF16 && DP == 64), "single score pass: bf16 <= 128 or fp32 64");
  // fp32 beyond 64: no resident Q; Q and K reach the score MMA in head-dim chunks through the K ring's slots
  static constexpr bool WIDE = !BF16 && DP > 64;
  static constexpr int NDC = WIDE ? DP / T::KB : 1;                    // head-dim chunks per score MMA
  // wide fp32: the prior is read from L2 (loads issued before each chunk's wait) instead of a single staged buffer,
  // and the shared memory goes to a third K ring slot at every head dim
  static constexpr int NPR = WIDE ? 0 : (BF16 && DP > 128) ? 1 : 2;  // staged prior buffers (0: L2)
  // fp32 at head dim 64 ("pooled"): Q (hi/lo planes) is the tensor-memory A operand of the score MMAs, each of which
  // covers a pair of 32-key chunks (N = 64: half the instructions). Q lands by TMA in a shared-memory pool that,
  // once copied into tensor memory, holds the ring of K chunk pairs; the landing takes the ring's next NK positions.
  // Wide fp32 issues its score MMAs over chunk pairs too: each slot carries a head-dim chunk of Q and of two K chunks.
  // bf16 up to head dim 128 pools too: Q takes 32 / 64 tensor-memory columns, and a score MMA over a pair of 64-key
  // chunks (N = 128) runs at the tensor pipe's full rate, where an N = 64 MMA with both operands in shared memory
  // takes 48 cycles for 32 cycles of work (measured back to back on the B200). Head dim 192 keeps Q in shared memory
  // (4 score buffers + O + Q would need 544 columns).
  static constexpr bool POOL = !(ONE && BF16) && !WIDE && (!BF16 || DP <= 128);
  static constexpr int PAIR = (POOL || WIDE) ? 2 : 1;                 // chunks per score MMA / K ring slot
  // pooled bf16 at head dim 128: two pair slots (64 KB; a third would take the shared memory past the limit)
  static constexpr int NK = POOL ? ((BF16 && DP > 64) ? 2 : 3) : (DP <= 128 ? 3 : 2);   // K ring slots
  static constexpr int LAND = POOL ? NK : 0;                          // ring positions the Q landing takes
  static constexpr int Q_BYTES = WIDE ? 0 : kBM * DP * T::EB;          // per plane
  static constexpr int K_BYTES = WIDE ? kSlotPlaneBytesRows<PAIR * T::CH> : PAIR * T::CH * DP * T::EB;  // per plane
  static constexpr int V_BYTES = T::CH * DP * T::EB;        // hi only (natural bf16 / transposed fp32)
  static constexpr int P_BYTES = kBM * 128;
  static constexpr int OFF_Q = 0;
  static constexpr int Q_END = OFF_Q + T::PL * Q_BYTES;
  static constexpr int OFF_K = POOL ? 0 : Q_END;
  static constexpr int K_END = OFF_K + NK * T::PL * K_BYTES;
  static constexpr int OFF_V = (POOL && Q_END > K_END) ? Q_END : K_END;  // pooled: past the larger use
  static constexpr int OFF_P = OFF_V + 2 * V_BYTES;
  static constexpr int OFF_PR = OFF_P + 2 * P_BYTES;
  static constexpr int SMEM = OFF_PR + NPR * kPriorTileBytes;
  static_assert(SMEM + 4096 <= kSmemPerBlock, "forward: dynamic + static shared memory above the per-block limit");
  // 4 score buffers in tensor memory: the MMA warp runs up to 3 chunks ahead of the element-wise warps, and the
  // last score MMA of a tile (which frees Q for the next tile) issues ~3 chunks before the tile ends
  static constexpr int NSB = ONE ? 2 : 4;
  static_assert(NSB % PAIR == 0, "chunk pairs take aligned score buffers");
  // Pass B loads V of chunk c after the K of chunk c + VLAG: before its P.V MMA needs V(c), the MMA warp has issued
  // the scores of every chunk below c + NSB - PAIR + 1, so the K loads ahead of V(c) never wait on MMAs behind it. A
  // wide pair takes NDC ring slots, more than the ring holds, so its K cannot run further ahead (lag NSB - PAIR); a
  // pooled pair takes one slot.
  static constexpr int VLAG = WIDE ? NSB - PAIR : NSB - 1;
  static constexpr int TM_S = 0;
  static constexpr int TM_O = NSB * T::CH;
  static constexpr int TM_QA = TM_O + DP;  // pooled: Q (hi, lo)
  static constexpr int TM_E = TM_QA + (POOL ? T::PL * kAColsPerPlane<T> : 0);  // ONE: stored 2^(t - m_c)
  static constexpr int MAX_KEYS_ONE = 512;
  // wide: Q's hi plane in tensor memory (DP columns), copied from the tile's first slots, so that later slots carry
  // only Q's lo plane (a third fewer streamed bytes)
  static constexpr int TM_QH = TM_E + (ONE ? MAX_KEYS_ONE / 2 : 0);
  static constexpr int TMEM_NEED = TM_QH + (WIDE ? DP : 0);
  static_assert(TMEM_NEED <= 512, "forward: tensor-memory columns above 512");
  static constexpr int TMEM_COLS = pow2_cols(TMEM_NEED);
  // O leaves through the two P buffers (free once the tile's last P.V has run) when they hold the whole row block
  static constexpr bool EPI_TMA = BF16 && T::NKB * kBM * 128 <= 2 * P_BYTES;
};

template <bool BF16, int DP, bool ONE = false>
__global__ void __launch_bounds__(Tile<BF16, DP>::NTHREADS, 1)
    geoattn_fwd_kernel(const __grid_constant__ TileMaps maps, const KParams p) {
  using C = FwdCfg<BF16, DP, ONE>;
  using T = typename C::T;
  constexpr int NPR = C::NPR, NK = C::NK, NSB = C::NSB;
  constexpr int PRB = NPR > 0 ? NPR : 1;  // prior-ring modulus (unused when the prior is read from L2)
  static_assert(!C::EPI_TMA || T::EW > 1, "the TMA epilogue relies on the warpgroup exchange barrier");
  if (smem_misaligned(p.status)) return;  // uniform over the CTA, before any barrier or allocation
  uint8_t* smem = smem_raw;
  __shared__ uint64_t bar_qfull, bar_qempty, bar_kfull[4], bar_kempty[4], bar_vfull[2], bar_vempty[2], bar_sfull[4],
      bar_sempty[4], bar_pfull[2], bar_pempty[2], bar_prfull[2], bar_prempty[2], bar_ofull;
  static_assert(NK <= 4 && NSB <= 4 && NPR <= 2, "ring deeper than its barrier array");
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ float xch[3][Tile<BF16, DP>::EW][kBM];  // cross-warpgroup row statistics: m, l1, l2
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // chunks every role iterates; pooled: whole pairs (an extra chunk past N is masked like a ragged one)
  const int nch = C::PAIR == 2 ? (((p.N + T::CH - 1) / T::CH + 1) & ~1) : (p.N + T::CH - 1) / T::CH;
  static_assert(C::LAND == 0 || C::LAND == NK, "a landing takes every slot of the K ring once");
  const int ntiles = p.nrb * p.B * p.H;  // tile = (128-query row block, b*h); persistent CTAs stride over tiles
  WaitCtx ctx{&abort_flag, p.status};
  const bool epi_tma = C::EPI_TMA && p.out_tma;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_qfull, 1);
    mbar_init(&bar_qempty, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar_kfull[i], 1);
      mbar_init(&bar_kempty[i], 1);
      mbar_init(&bar_sfull[i], 1);
      mbar_init(&bar_sempty[i], T::EWT);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_vfull[i], 1);
      mbar_init(&bar_vempty[i], 1);
      mbar_init(&bar_pfull[i], T::EWT);
      mbar_init(&bar_pempty[i], 1);
      mbar_init(&bar_prfull[i], 1);
      mbar_init(&bar_prempty[i], T::EWT);
    }
    mbar_init(&bar_ofull, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t sbase = smem_u32(smem);

  if (warp == T::TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&maps.q);
      prefetch_tmap(&maps.k);
      prefetch_tmap(&maps.v);
      int kc = 0, vc = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
        if constexpr (C::POOL) {  // Q into the pool once its K ring positions are free
          for (int s = 0; s < C::LAND && ok; ++s, ++kc) ok = mbar_wait(&bar_kempty[kc % NK], ((kc / NK) & 1) ^ 1, ctx);
          if (!ok) break;
          mbar_arrive_expect_tx(&bar_qfull, T::PL * C::Q_BYTES);
          tma_tile<T>(smem + C::OFF_Q, &maps.q, &bar_qfull, kBM, rb * kBM, h, b, p.B, T::PL);
        } else if constexpr (!C::WIDE) {  // Q once the previous tile's last score MMA has read the old one
          if (!(ok = mbar_wait(&bar_qempty, (it & 1) ^ 1, ctx))) break;
          mbar_arrive_expect_tx(&bar_qfull, T::PL * C::Q_BYTES);
          tma_tile<T>(smem + C::OFF_Q, &maps.q, &bar_qfull, kBM, rb * kBM, h, b, p.B, T::PL);
        }
        for (int pass = 0; pass < 2 && ok; ++pass) {
          if (pass == 1 && tile + (int)gridDim.x < ntiles) {  // next tile's operands into L2
            const int nt = tile + gridDim.x, nbh = nt / p.nrb, nb = nbh / p.H, nh = nbh % p.H;
            prefetch_tile<T>(&maps.q, (nt % p.nrb) * kBM, nh, nb, p.B, T::PL);
            prefetch_rows<T>(&maps.k, p.N, nh, nb, p.B, T::PL);
            if constexpr (BF16) prefetch_rows<T>(&maps.v, p.N, nh, nb, p.B, 1);
          }
          // pass B in the MMA warp's order: K of chunk c, then V of chunk c - (NSB - 1), whose P.V MMA follows
          // the score MMA of chunk c
          auto load_v = [&](int cv) -> bool {
            const int vs = vc & 1;
            if (!mbar_wait(&bar_vempty[vs], ((vc >> 1) & 1) ^ 1, ctx)) return false;
            mbar_arrive_expect_tx(&bar_vfull[vs], C::V_BYTES);
            if constexpr (BF16)
              tma_tile<T>(smem + C::OFF_V + vs * C::V_BYTES, &maps.v, &bar_vfull[vs], T::CH, cv * T::CH, h, b, p.B, 1);
            else
              tma_tileT(smem + C::OFF_V + vs * C::V_BYTES, &maps.v, &bar_vfull[vs], cv * T::CH, h, b);
            ++vc;
            return true;
          };
          if (ONE && pass == 1) {  // single score pass: pass B reads V only
            for (int cv = 0; cv < nch && ok; ++cv) ok = load_v(cv);
            continue;
          }
          for (int c = 0; c < nch && ok; c += C::PAIR) {
            // wide: Q's hi plane only in the tile's first slots (the MMA warp keeps it in tensor memory)
            [[maybe_unused]] const bool qh = pass == 0 && c == 0;
            for (int dc = 0; dc < C::NDC && ok; ++dc) {
              const int ks = kc % NK;
              if (!(ok = mbar_wait(&bar_kempty[ks], ((kc / NK) & 1) ^ 1, ctx))) break;
              mbar_arrive_expect_tx(&bar_kfull[ks], T::PL * C::K_BYTES - ((C::WIDE && !qh) ? kBM * 128 : 0));
              uint8_t* slot = smem + C::OFF_K + ks * T::PL * C::K_BYTES;
              if constexpr (C::WIDE)
                tma_slot_rows<T, C::PAIR * T::CH>(slot, &bar_kfull[ks], &maps.q, rb * kBM, &maps.k, c * T::CH, dc, h,
                                                  b, p.B, qh);
              else if constexpr (C::POOL)
                tma_pair<T>(slot, &maps.k, &bar_kfull[ks], c, h, b, p.B);
              else
                tma_tile<T>(slot, &maps.k, &bar_kfull[ks], T::CH, c * T::CH, h, b, p.B, T::PL);
              ++kc;
            }
            for (int cc = c; cc < c + C::PAIR && ok; ++cc)
              if (pass == 1 && cc >= C::VLAG) ok = load_v(cc - C::VLAG);
          }
          if (pass == 1)
            for (int cv = nch - C::VLAG; cv < nch && ok; ++cv)
              if (cv >= 0) ok = load_v(cv);
        }
      }
    }
  } else if (warp == T::PR_WARP) {
    if (NPR > 0 && lane == 0) {
      prefetch_tmap(&maps.prior);
      int prc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int rb = tile % p.nrb;
        for (int c = 0; c < nch && ok; ++c) {  // pass B only
          const int ps = prc % PRB;
          if (!(ok = mbar_wait(&bar_prempty[ps], ((prc / PRB) & 1) ^ 1, ctx))) break;
          mbar_arrive_expect_tx(&bar_prfull[ps], kPriorTileBytes);
          tma_prior(smem + C::OFF_PR + ps * kPriorTileBytes, &maps.prior, &bar_prfull[ps], rb * kBM, c);
          ++prc;
        }
      }
    }
  } else if (warp == T::MMA_WARP) {
    if (lane == 0) {
      int kc = 0, sc = 0, pc = 0, it = 0;
      bool ok = true;
      auto issue_s = [&](bool land = false) -> bool {
        const int ss = sc % NSB;
        if constexpr (C::WIDE) {  // a chunk pair into two adjacent score buffers, accumulated over head-dim chunks
          if (!mbar_wait(&bar_sempty[ss], ((sc / NSB) & 1) ^ 1, ctx)) return false;
          if (!mbar_wait(&bar_sempty[ss + 1], (((sc + 1) / NSB) & 1) ^ 1, ctx)) return false;
          for (int dc = 0; dc < C::NDC; ++dc) {
            const int ks = kc % NK;
            if (!mbar_wait(&bar_kfull[ks], (kc / NK) & 1, ctx)) return false;
            tc_fence_after();
            const uint32_t slot = sbase + C::OFF_K + ks * T::PL * C::K_BYTES, qh = tmem + C::TM_QH + dc * T::KB;
            // the tile's first pair: Q's hi chunk into tensor memory (the MMAs below read it, after the copy, and
            // the slot is released once they have completed)
            if (land) cp_slot_a_hi<T>(qh, slot);
            mma_slot_rows_ah<T, C::PAIR * T::CH>(tmem + C::TM_S + ss * T::CH, slot, qh, dc > 0);
            mma_commit(&bar_kempty[ks]);
            ++kc;
          }
          mma_commit(&bar_sfull[ss]);
          mma_commit(&bar_sfull[ss + 1]);
          sc += 2;
          return true;
        } else if constexpr (C::POOL) {  // one N = 64 MMA for a chunk pair into two adjacent score buffers
          const int ks = kc % NK;
          // phases of the full barriers count only K loads; the Q landings (one per slot per tile, this tile's
          // included) complete none
          if (!mbar_wait(&bar_kfull[ks], ((kc / NK) - (it + 1)) & 1, ctx)) return false;
          if (!mbar_wait(&bar_sempty[ss], ((sc / NSB) & 1) ^ 1, ctx)) return false;
          if (!mbar_wait(&bar_sempty[ss + 1], (((sc + 1) / NSB) & 1) ^ 1, ctx)) return false;
          tc_fence_after();
          mma_qk_ts<T, C::PAIR * T::CH>(tmem + C::TM_S + ss * T::CH, tmem + C::TM_QA,
                                        sbase + C::OFF_K + ks * T::PL * C::K_BYTES, C::K_BYTES);
          mma_commit(&bar_kempty[ks]);
          ++kc;
          mma_commit(&bar_sfull[ss]);
          mma_commit(&bar_sfull[ss + 1]);
          sc += 2;
          return true;
        } else {
          const int ks = kc % NK;
          if (!mbar_wait(&bar_kfull[ks], (kc / NK) & 1, ctx)) return false;
          if (!mbar_wait(&bar_sempty[ss], ((sc / NSB) & 1) ^ 1, ctx)) return false;
          tc_fence_after();
          mma_qk<T, T::CH>(tmem + C::TM_S + ss * T::CH, sbase + C::OFF_Q, C::Q_BYTES,
                           sbase + C::OFF_K + ks * T::PL * C::K_BYTES, C::K_BYTES);
          mma_commit(&bar_kempty[ks]);
          ++kc;
        }
        mma_commit(&bar_sfull[ss]);
        ++sc;
        return true;
      };
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        if constexpr (!C::WIDE)
          if (!(ok = mbar_wait(&bar_qfull, it & 1, ctx))) break;
        if constexpr (C::POOL) {
          // Q into tensor memory. The previous tile's score MMAs, the last readers of these columns, completed before
          // its last K ring positions were released, and the TMA warp loaded this Q only after that. The landing's
          // ring positions are released once the copies have read the pool.
          tc_fence_after();
          cp_operand_tmem<T>(tmem + C::TM_QA, sbase + C::OFF_Q, C::Q_BYTES);
          // the copies are drained through the next score buffer (free once its previous use was read; the real
          // score MMA overwrites it) before the pool is released
          if (!(ok = mbar_wait(&bar_sempty[sc % NSB], ((sc / NSB) & 1) ^ 1, ctx))) break;
          cp_drain_operand<T>(tmem + C::TM_S + (sc % NSB) * T::CH, tmem + C::TM_QA, sbase + C::OFF_Q);
          for (int s = 0; s < C::LAND; ++s, ++kc) mma_commit(&bar_kempty[kc % NK]);
        }
        // wide: Q's hi plane of this tile replaces the previous tile's in tensor memory once every MMA that read it
        // (the previous tile's score MMAs, before its last P.V) has completed
        if constexpr (C::WIDE)
          if (it > 0 && !(ok = mbar_wait(&bar_ofull, (it - 1) & 1, ctx))) break;
        for (int c = 0; c < nch && ok; c += C::PAIR) ok = issue_s(c == 0);  // pass A
        if (ONE && !C::POOL && ok) mma_commit(&bar_qempty);  // single score pass: Q is free after pass A's MMAs
        int nb = ONE ? nch : 0;  // pass-B chunks whose score MMAs are issued (none with a single score pass)
        // keeps the pass-B scores up to NSB - 1 chunks ahead; Q is released once the tile's last one is issued
        auto top_up = [&](int upto) -> bool {
          for (; nb < nch && nb + C::PAIR - 1 < upto; nb += C::PAIR) {
            if (!issue_s()) return false;
            if (!C::WIDE && !C::POOL && nb + 1 == nch) mma_commit(&bar_qempty);
          }
          return true;
        };
        for (int c = 0; c < nch && ok; ++c) {
          if (!(ok = top_up(c + NSB))) break;
          const int ps = pc & 1;
          if (!(ok = mbar_wait(&bar_pfull[ps], (pc >> 1) & 1, ctx))) break;
          if (!(ok = mbar_wait(&bar_vfull[ps], (pc >> 1) & 1, ctx))) break;
          tc_fence_after();
          mma_pv<T>(tmem + C::TM_O, sbase + C::OFF_P + ps * C::P_BYTES, sbase + C::OFF_V + ps * C::V_BYTES, c > 0);
          mma_commit(&bar_pempty[ps]);
          mma_commit(&bar_vempty[ps]);
          ++pc;
        }
        if (ok) mma_commit(&bar_ofull);
      }
    }
  } else if (warp < T::TMA_WARP) {
    // ---------------- element-wise warps ----------------
    const Ew e = ew_id(tmem);
    const float sc_l2 = p.scale_log2;
    int sc = 0, pc = 0, prc = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
      const int row = rb * kBM + e.r;
      const Abg ab = load_abg(p, h);
      float m = -INFINITY, l = 0.f;
      // Pass A: running max and sum over this warpgroup's pieces. The max is taken over the raw accumulators
      // (scaling by a positive constant and rounding are monotonic), the sum from fma(acc, scale, -m). The next
      // chunk's scores are loaded from tensor memory while this chunk's are reduced (two register sets).
      const int piece = e.wg;
      auto reduce_a = [&](uint32_t (&u)[32], int c) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(u[j]);
        const int nvalid = p.N - (c * T::CH + piece * 32);  // >= 32: no masked column in this piece
        if (nvalid < 32) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = (j < nvalid) ? v[j] : -INFINITY;
        }
        // four independent partial maxima / sums keep the dependency chains short
        float mx4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
        for (int j = 4; j < 32; ++j) mx4[j & 3] = fmaxf(mx4[j & 3], v[j]);
        const float mn = fmaxf(m, fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sc_l2);
        // a warpgroup whose columns so far are all masked keeps m = -inf, l = 0 (never 2^(-inf - -inf))
        const float mref = (mn == -INFINITY) ? 0.f : mn;
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 32; ++j) s4[j & 3] += ex2(fmaf(v[j], sc_l2, -mref));
        l = l * ex2(m - mref) + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
        m = mn;
      };
      // two chunks' scores (c, c + 1) reduced together: one max over 64 values, then 64 independent exp2
      auto reduce_pair = [&](uint32_t (&u0)[32], uint32_t (&u1)[32], int c) {
        float v[64];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(u0[j]);
          v[32 + j] = __uint_as_float(u1[j]);
        }
        const int nv0 = p.N - (c * T::CH + piece * 32), nv1 = nv0 - T::CH;
        if (nv1 < 32) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = (j < nv0) ? v[j] : -INFINITY;
            v[32 + j] = (j < nv1) ? v[32 + j] : -INFINITY;
          }
        }
        float mx8[8] = {v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]};
#pragma unroll
        for (int j = 8; j < 64; ++j) mx8[j & 7] = fmaxf(mx8[j & 7], v[j]);
        const float mxa = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float mn = fmaxf(m, mxa * sc_l2);
        const float mref = (mn == -INFINITY) ? 0.f : mn;
        float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 64; ++j) s8[j & 7] += ex2(fmaf(v[j], sc_l2, -mref));
        l = l * ex2(m - mref) + (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
        m = mn;
      };
      // waits for chunk c's scores (global count g) and issues their load into u
      auto load_s = [&](int g, uint32_t (&u)[32]) -> bool {
        if (!warp_wait(&bar_sfull[g % NSB], (g / NSB) & 1, ctx)) return false;
        tc_fence_after();
        tmem_ld32_issue(e.lane_base + C::TM_S + (g % NSB) * T::CH + piece * 32, u);
        return true;
      };
      // the loaded scores are in registers: the MMA may refill their buffer
      auto release_s = [&](int g, uint32_t (&u)[32]) {
        tmem_wait32(u);
        tc_fence_before();
        mbar_arrive(&bar_sempty[g % NSB]);
      };
      // single score pass: each pair's reference max (the values stored for it are 2^(t - mc_k)); -inf: all masked.
      // Up to eight scalars (4 pairs of 64-key chunks in bf16, 8 of 32-key chunks in fp32), set and read under
      // warp-uniform branches (an array indexed by the pair would live in local memory).
      constexpr int NPAIR = C::MAX_KEYS_ONE / (2 * T::CH);
      static_assert(!ONE || NPAIR == 4 || NPAIR == 8, "single score pass: four or eight chunk pairs");
      [[maybe_unused]] float mc0 = -INFINITY, mc1 = -INFINITY, mc2 = -INFINITY, mc3 = -INFINITY, mc4 = -INFINITY,
                             mc5 = -INFINITY, mc6 = -INFINITY, mc7 = -INFINITY;
      auto set_mc = [&](int k, float x) {
        switch (k) {
          case 0: mc0 = x; break;
          case 1: mc1 = x; break;
          case 2: mc2 = x; break;
          case 3: mc3 = x; break;
          case 4: mc4 = x; break;
          case 5: mc5 = x; break;
          case 6: mc6 = x; break;
          default: mc7 = x; break;
        }
      };
      auto get_mc = [&](int k) -> float {
        switch (k) {
          case 0: return mc0;
          case 1: return mc1;
          case 2: return mc2;
          case 3: return mc3;
          case 4: return mc4;
          case 5: return mc5;
          case 6: return mc6;
          default: return mc7;
        }
      };
      (void)set_mc;
      (void)get_mc;
      if constexpr (ONE) {
        // as reduce_pair, and the pair's 2^(t - mref) go to tensor memory as fp16 pairs: chunk c, piece p take the
        // 16 columns TM_E + c CH / 2 + 16 p of this thread's lane
        auto reduce_store = [&](uint32_t (&u0)[32], uint32_t (&u1)[32], int c, bool two) -> float {
          float v[64];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __uint_as_float(u0[j]);
            v[32 + j] = two ? __uint_as_float(u1[j]) : -INFINITY;
          }
          const int nv0 = p.N - (c * T::CH + piece * 32), nv1 = nv0 - T::CH;
          if (nv1 < 32) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = (j < nv0) ? v[j] : -INFINITY;
              v[32 + j] = (j < nv1) ? v[32 + j] : -INFINITY;
            }
          }
          float mx8[8] = {v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]};
#pragma unroll
          for (int j = 8; j < 64; ++j) mx8[j & 7] = fmaxf(mx8[j & 7], v[j]);
          const float mxa = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                  fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
          const float mn = fmaxf(m, mxa * sc_l2);
          const float mref = (mn == -INFINITY) ? 0.f : mn;
          float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          uint32_t h0[16], h1[16];
#pragma unroll
          for (int j = 0; j < 64; j += 2) {
            const float e0 = ex2(fmaf(v[j], sc_l2, -mref)), e1 = ex2(fmaf(v[j + 1], sc_l2, -mref));
            s8[j & 7] += e0;
            s8[(j + 1) & 7] += e1;
            const __half2 hh = __floats2half2_rn(e0, e1);
            if (j < 32) h0[j / 2] = *reinterpret_cast<const uint32_t*>(&hh);
            else h1[(j - 32) / 2] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          l = l * ex2(m - mref) + (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
          m = mn;
          tmem_st16(e.lane_base + C::TM_E + c * (T::CH / 2) + piece * 16, h0);
          if (two) tmem_st16(e.lane_base + C::TM_E + (c + 1) * (T::CH / 2) + piece * 16, h1);
          return mn;
        };
        uint32_t ua[32], ub[32];
        const int g0 = sc;
#pragma unroll 1
        for (int pi = 0; pi < NPAIR; ++pi) {
          const int c = 2 * pi;
          if (c < nch && ok) {
            const bool two = c + 1 < nch;
            ok = load_s(g0 + c, ua);
            if (ok && two) ok = load_s(g0 + c + 1, ub);
            if (ok) {
              release_s(g0 + c, ua);
              if (two) {
                tc_fence_before();
                mbar_arrive(&bar_sempty[(g0 + c + 1) % NSB]);
                tmem_pin32(ub);
              }
              set_mc(pi, reduce_store(ua, ub, c, two));
            }
          }
        }
        tmem_wait_all();  // no load stays in flight past the loop (aborted paths included)
        tmem_wait_st();   // the stored values are complete before pass B reads them back
        sc += nch;
      } else {
        // chunks in pairs: both chunks' scores are loaded, then reduced together (64 independent values per thread)
        uint32_t ua[32], ub[32];
        const int g0 = sc;
        for (int c = 0; c < nch && ok; c += 2) {
          const bool two = c + 1 < nch;
          if (!(ok = load_s(g0 + c, ua))) break;
          if (two && !(ok = load_s(g0 + c + 1, ub))) break;
          release_s(g0 + c, ua);
          if (two) {
            tc_fence_before();
            mbar_arrive(&bar_sempty[(g0 + c + 1) % NSB]);
            tmem_pin32(ub);
            reduce_pair(ua, ub, c);
          } else {
            reduce_a(ua, c);
          }
        }
        tmem_wait_all();  // no load stays in flight past the loop (aborted paths included)
        sc += nch;
      }
      if constexpr (T::EW > 1) {  // combine the warpgroups' statistics (same order in every warpgroup)
        xch[0][e.wg][e.r] = m;
        xch[1][e.wg][e.r] = l;
        // the previous tile's O store has finished reading the P buffers before pass B rewrites them
        if (epi_tma && threadIdx.x == 0) bulk_wait_read0();
        ew_sync(T::EWT);
        m = xch[0][0][e.r];
#pragma unroll
        for (int w = 1; w < T::EW; ++w) m = fmaxf(m, xch[0][w][e.r]);
        l = 0.f;
#pragma unroll
        for (int w = 0; w < T::EW; ++w) {
          const float mw = xch[0][w][e.r];
          l += (mw == -INFINITY) ? 0.f : xch[1][w][e.r] * ex2(mw - m);
        }
        ew_sync(T::EWT);
      }
      const float m1 = m + log2f(l);  // P1 = 2^(t - m1)
      const float aL = ab.a * kLog2e, bL = ab.b * kLog2e, gL = ab.g * kLog2e, cL = ab.c * kLog2e;
      float l2 = 0.f;
      // single score pass: P1 of a stored value of pair k = value * 2^(mc_k - m1) (0 for an all-masked pair)
      if constexpr (ONE) {
        mc0 = ex2(mc0 - m1);
        mc1 = ex2(mc1 - m1);
        mc2 = ex2(mc2 - m1);
        mc3 = ex2(mc3 - m1);
        if constexpr (NPAIR > 4) {
          mc4 = ex2(mc4 - m1);
          mc5 = ex2(mc5 - m1);
          mc6 = ex2(mc6 - m1);
          mc7 = ex2(mc7 - m1);
        }
      }
      // Pass B
      for (int c = 0; c < nch && ok; ++c) {
        const int ss = sc % NSB, ps = pc & 1, prs = prc % PRB;
        Prior32<BF16> pr;
        if constexpr (NPR == 0) {  // from L2, issued before the waits (one piece per chunk)
          static_assert(T::PIECES == 1 && T::EW == 1, "prior read from L2 in one piece per chunk");
          load_prior32<BF16>(p.prior, p.np, row, c * T::CH, pr);
        }
        if constexpr (!ONE)
          if (!(ok = warp_wait(&bar_sfull[ss], (sc / NSB) & 1, ctx))) break;
        if constexpr (NPR > 0)
          if (!(ok = warp_wait(&bar_prfull[prs], (prc / PRB) & 1, ctx))) break;
        tc_fence_after();
        uint8_t* preg = smem + C::OFF_P + ps * C::P_BYTES;
        const uint8_t* prt = smem + C::OFF_PR + prs * kPriorTileBytes;
        {
          [[maybe_unused]] uint32_t vs[32];
          float v[32];
          [[maybe_unused]] float fc = 0.f;
          [[maybe_unused]] uint32_t ve[16];
          if constexpr (ONE) {
            // this row's stored values of the chunk (its own tensor-memory writes, complete since pass A's
            // wait::st)
            fc = get_mc(c >> 1);  // c is warp-uniform
            tmem_ld16_issue(e.lane_base + C::TM_E + c * (T::CH / 2) + piece * 16, ve);
            if constexpr (NPR > 0 && !BF16) prior32_smem<BF16>(prt, e.r, piece, pr);  // overlaps the TMEM load
            tmem_wait16(ve);
          } else {
            tmem_ld32_issue(e.lane_base + C::TM_S + ss * T::CH + piece * 32, vs);
            if constexpr (NPR > 0 && !BF16) prior32_smem<BF16>(prt, e.r, piece, pr);  // overlaps the TMEM load
            tmem_wait32(vs);
            tc_fence_before();
            mbar_arrive(&bar_sempty[ss]);  // the scores are in registers: the MMA may refill the buffer
          }
          const int nvalid = p.N - (c * T::CH + piece * 32);
          float l24[4] = {0.f, 0.f, 0.f, 0.f};
          // phase-ordered: 32 independent exp2 for P1, then the biased exp2 (more independent work per warp)
          auto body = [&](auto masked) {
            float p1[32];
            if constexpr (ONE) {
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ve[j / 2]));
                p1[j] = f.x * fc;
                p1[j + 1] = f.y * fc;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) p1[j] = ex2(fmaf(__uint_as_float(vs[j]), sc_l2, -m1));
            }
            // bf16 staged prior: four pairs per 16-byte shared-memory load next to their use (no 32-register copy)
            [[maybe_unused]] uint32_t pw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float dpj, apj;
              if constexpr (BF16 && NPR > 0) {
                if ((j & 3) == 0) {
                  const uint4 u = *reinterpret_cast<const uint4*>(prt + piece * (kBM * 128) + sw128(e.r, j / 4));
                  pw[0] = u.x;
                  pw[1] = u.y;
                  pw[2] = u.z;
                  pw[3] = u.w;
                }
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pw[j & 3]));
                dpj = f.x;
                apj = f.y;
              } else {
                pr.get(j, dpj, apj);
              }
              float ev = ex2(fmaf(aL, p1[j], fmaf(bL, dpj, fmaf(gL, apj, -cL))));
              if constexpr (decltype(masked)::value) ev = (j < nvalid) ? ev : 0.f;
              l24[j & 3] += ev;
              v[j] = ev;
            }
          };
          if (nvalid >= 32) body(std::false_type{});
          else body(std::true_type{});
          l2 += (l24[0] + l24[1]) + (l24[2] + l24[3]);
          // the prior tile is released once every value read from it has been used (not when the loads are issued)
          if constexpr (NPR > 0) mbar_arrive(&bar_prempty[prs]);
          // the P buffer is free once the P.V two chunks back has run (waited here, after the math)
          if (!(ok = warp_wait(&bar_pempty[ps], ((pc >> 1) & 1) ^ 1, ctx))) break;
          stage_row32<BF16>(preg, e.r, piece, v);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bar_pfull[ps]);
        if constexpr (!ONE) ++sc;
        ++pc;
        ++prc;
      }
      if constexpr (T::EW > 1) {
        xch[2][e.wg][e.r] = l2;
        ew_sync(T::EWT);
        l2 = 0.f;
#pragma unroll
        for (int w = 0; w < T::EW; ++w) l2 += xch[2][w][e.r];
      }
      if (ok) ok = warp_wait(&bar_ofull, it & 1, ctx);
      tc_fence_after();
      const float inv_l2 = __frcp_rn(l2);
      if (epi_tma) {
        // every P.V of the tile has completed (ofull), so the P buffers hold the staged O tile
        if (ok) stage_acc<DP / (32 * T::EW)>(e.lane_base + C::TM_O, e.wg * 32, 32 * T::EW, smem + C::OFF_P, e.r, inv_l2);
        store_tile<T>(&maps.out0, smem + C::OFF_P, p.D, rb * kBM, h, b, ok);
      } else if (ok) {
        const long long ooff = (long long)b * p.o_str[0] + (long long)h * p.o_str[1] + (long long)row * p.o_str[2];
#pragma unroll
        for (int d0 = e.wg * 32; d0 < DP; d0 += 32 * T::EW) {
          float v[32];
          tmem_ld32(e.lane_base + C::TM_O + d0, v);
          if (row < p.N && d0 < p.D) store_row32<BF16>(p.o, ooff, p.o_str[3], d0, p.D, v, inv_l2);
        }
      }
      if (ok && row < p.N && e.wg == 0) {
        const size_t s = (size_t)bh * p.N + row, n = (size_t)p.B * p.H * p.N;
        p.stats[s] = m;
        p.stats[n + s] = l;
        p.stats[2 * n + s] = l2;
      }
      tc_fence_before();  // the O reads above precede this warp's next hand-offs to the MMA warp
    }
    if (epi_tma && threadIdx.x == 0) bulk_wait_read0();  // shared memory outlives the last store's reads
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ===============================================================================================================
// Backward row pass: one CTA per (128-query row block, b*h).
// Sweep 1 recomputes S, dP = dO V^T, P1, P2 and accumulates, per row,
//   delta2 = sum P2 dP,  a = sum P2 dP P1,  b = sum P2 P1,
//   so that with dZ = P2 (dP - delta2): sum dZ P1 = a - delta2 b = d(alpha) of the row, delta1 = alpha (a - delta2 b).
// With DQ, sweep 2 recomputes the tiles again, forms dZ, dS = P1 (alpha dZ - delta1), accumulates dQ += dS K and
// the row's d(beta) = sum dZ Dp, d(gamma) = sum dZ Ap. Without DQ (bf16 with a dS scratch), the kernel stops after
// sweep 1: the key pass stores dS and the bias gradients of beta and gamma, and a GEMM forms dQ.
// The row records (m1, c2, delta1, delta2) go to the key pass.
// ===============================================================================================================
template <bool BF16, int DP, bool DQ = true>
struct RowsCfg : Tile<BF16, DP> {
  using T = Tile<BF16, DP>;
  // fp32 beyond 64: no resident Q / dO; (Q, K) and (dO, V) reach the S and dP MMAs in head-dim chunks through the
  // K ring's slots (the V ring is unused)
  static constexpr bool WIDE = !BF16 && DP > 64;
  static constexpr int NDC = WIDE ? DP / T::KB : 1;
  // fp32: the prior is read from L2 (loads issued before each chunk's wait, as in the key pass); at head dim 64 the
  // shared memory a staged prior tile would take holds a second K/V buffer instead
  // fp32 at head dim 64 ("pooled"): Q and dO (hi/lo planes) are the tensor-memory A operands of the S and dP MMAs.
  // They land by TMA in a shared-memory pool that, once copied into tensor memory, holds the K and V rings for the
  // rest of the tile: the landing takes the rings' next NKV positions, so their order and phases carry the hand-over.
  static constexpr bool POOL = !BF16 && !WIDE;
  static constexpr int NKV = WIDE ? 3 : POOL ? 4 : (DP > 128) ? 1 : DQ ? 2 : 3;  // K/V chunk buffers / ring slots
  static constexpr int LAND = POOL ? NKV : 0;  // ring positions the Q/dO landing takes per tile
  static constexpr int NPR = (BF16 && DP <= 128) ? 2 : !BF16 ? 0 : 1;  // staged prior buffers (0: L2)
  static constexpr int Q_BYTES = WIDE ? 0 : kBM * DP * T::EB;                   // per plane (Q and dO)
  // wide: the S and dP MMAs cover pairs of 32-key chunks (slots carry a head-dim chunk of Q or dO and of two K or
  // V chunks); the K^T loads for dQ trail the slots by one pair, so the TMA never waits on a dQ MMA that needs the
  // next pair's scores first
  static constexpr int PAIR = WIDE ? 2 : 1;
  static constexpr int K_BYTES = WIDE ? kSlotPlaneBytesRows<PAIR * T::CH> : T::CH * DP * T::EB;  // per plane per slot
  static constexpr int KT_BYTES = BF16 ? 0 : DP * 128;  // fp32: transposed K chunk (hi) for dQ
  static constexpr int DS_BYTES = kBM * 128;
  static constexpr int NDS = (BF16 || POOL) ? 2 : 1;  // dS / K^T buffers (ring size)
  static constexpr int NDS_ALLOC = DQ ? NDS : 0;      // allocated only with DQ
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + T::PL * Q_BYTES;
  static constexpr int QD_END = OFF_DO + T::PL * Q_BYTES;
  static constexpr int OFF_K = POOL ? 0 : QD_END;
  static constexpr int OFF_V = OFF_K + NKV * T::PL * K_BYTES;
  static constexpr int KV_END = OFF_V + (WIDE ? 0 : NKV * T::PL * K_BYTES);
  static constexpr int OFF_KT = (POOL && QD_END > KV_END) ? QD_END : KV_END;  // pooled: past the larger use
  static constexpr int OFF_DS = OFF_KT + NDS_ALLOC * KT_BYTES;
  static constexpr int OFF_PR = OFF_DS + NDS_ALLOC * DS_BYTES;
  static constexpr int OFF_XS = OFF_PR + NPR * kPriorTileBytes;  // without DQ: warpgroup 1's row sums
  static constexpr int SMEM = OFF_XS + (DQ ? 0 : 3 * kBM * 4);
  static_assert(SMEM + 1024 <= kSmemPerBlock, "row pass: dynamic + static shared memory above the per-block limit");
  // S / dP accumulator buffers in tensor memory: 4 without the dQ accumulator, so the MMA warp runs ~3 chunks ahead
  // and frees Q / dO for the next tile early enough to hide its reload
  static constexpr int NSB = (DQ && !WIDE) ? 2 : 4;
  static_assert(NSB % PAIR == 0, "chunk pairs take aligned score buffers");
  static constexpr int TM_S = 0;
  static constexpr int TM_DP = NSB * T::CH;
  static constexpr int TM_DQ = 2 * NSB * T::CH;
  static constexpr int TM_QA = TM_DQ + (DQ ? DP : 0);                              // pooled: Q (hi, lo)
  static constexpr int TM_DOA = TM_QA + (POOL ? T::PL * kAColsPerPlane<T> : 0);    // pooled: dO (hi, lo)
  static constexpr int TMEM_NEED = TM_DOA + (POOL ? T::PL * kAColsPerPlane<T> : 0);
  static_assert(TMEM_NEED <= 512, "row pass: tensor-memory columns above 512");
  static constexpr int TMEM_COLS = pow2_cols(TMEM_NEED);
  // dQ leaves through the dS buffers (free once the tile's last dQ MMA has run) when they hold the whole row block
  static constexpr bool EPI_TMA = DQ && BF16 && T::NKB * kBM * 128 <= NDS * DS_BYTES;
};

// Row record of `row` (chunk-blocked so that the key pass can fetch one query chunk's records in one bulk copy).
template <class T>
__device__ __forceinline__ float* rec_ptr(const KParams& p, int bh, int row) {
  return p.rowrec + ((size_t)bh * p.nchp + row / T::CH) * T::NREC * T::CH + row % T::CH;
}

template <bool BF16, int DP, bool DQ>
__global__ void __launch_bounds__(Tile<BF16, DP>::NTHREADS, 1)
    geoattn_bwd_rows_kernel(const __grid_constant__ TileMaps maps, const KParams p) {
  // one sweep (dS from the key pass's scratch): bf16, and fp32 at head dim 64 (the pooled layout)
  // without DQ: the dS-scratch backward (bf16; fp32 at head dim 64; fp32 above 64 with the transposing dQ GEMM)
  using C = RowsCfg<BF16, DP, DQ>;
  using T = typename C::T;
  constexpr int NKV = C::NKV, NPR = C::NPR, NSB = C::NSB;
  constexpr int PRB = NPR > 0 ? NPR : 1;  // prior-ring modulus (unused when the prior is read from L2)
  if (smem_misaligned(p.status)) return;  // uniform over the CTA, before any barrier or allocation
  uint8_t* smem = smem_raw;
  __shared__ uint64_t bar_qfull, bar_qempty, bar_kfull[4], bar_kempty[4], bar_vfull[4], bar_vempty[4], bar_sfull[4],
      bar_sempty[4], bar_dsfull[2], bar_dsempty[2], bar_ktfull[2], bar_ktempty[2], bar_prfull[2], bar_prempty[2], bar_dqfull;
  static_assert(NKV <= 4 && NSB <= 4 && C::NDS <= 2 && NPR <= 2, "ring deeper than its barrier array");
  static_assert(C::LAND == 0 || C::LAND == NKV, "a landing takes every slot of the K/V rings once");
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ double red[8][3];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // chunks every role iterates; wide: whole pairs (an extra chunk past N is masked like a ragged one)
  const int nch = C::PAIR == 2 ? (((p.N + T::CH - 1) / T::CH + 1) & ~1) : (p.N + T::CH - 1) / T::CH;
  const int ntiles = p.nrb * p.B * p.H;  // tile = (128-query row block, b*h); persistent CTAs stride over tiles
  WaitCtx ctx{&abort_flag, p.status};
  const bool epi_tma = DQ && C::EPI_TMA && p.out_tma;
  constexpr int SWEEPS = DQ ? 2 : 1;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_qfull, 1);
    mbar_init(&bar_qempty, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar_kfull[i], 1);
      mbar_init(&bar_kempty[i], 1);
      mbar_init(&bar_vfull[i], 1);
      mbar_init(&bar_vempty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar_sfull[i], 1);
      mbar_init(&bar_sempty[i], T::EWT);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_dsfull[i], T::EWT);
      mbar_init(&bar_dsempty[i], 1);
      mbar_init(&bar_ktfull[i], 1);
      mbar_init(&bar_ktempty[i], 1);
      mbar_init(&bar_prfull[i], 1);
      mbar_init(&bar_prempty[i], T::EWT);
    }
    mbar_init(&bar_dqfull, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t sbase = smem_u32(smem);

  if (warp == T::TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&maps.q);
      prefetch_tmap(&maps.k);
      prefetch_tmap(&maps.v);
      prefetch_tmap(&maps.dout);
      int kc = 0, tc = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
      if constexpr (C::POOL) {  // Q and dO into the pool once its K/V ring positions are free
        for (int s = 0; s < C::LAND && ok; ++s, ++kc) {
          const int ks = kc % NKV, par = ((kc / NKV) & 1) ^ 1;
          ok = mbar_wait(&bar_kempty[ks], par, ctx) && mbar_wait(&bar_vempty[ks], par, ctx);
        }
        if (!ok) break;
        mbar_arrive_expect_tx(&bar_qfull, 2 * T::PL * C::Q_BYTES);
        tma_tile<T>(smem + C::OFF_Q, &maps.q, &bar_qfull, kBM, rb * kBM, h, b, p.B, T::PL);
        tma_tile<T>(smem + C::OFF_DO, &maps.dout, &bar_qfull, kBM, rb * kBM, h, b, p.B, T::PL);
      } else if constexpr (!C::WIDE) {  // Q and dO once the previous tile's last S/dP MMAs have read the old ones
        if (!(ok = mbar_wait(&bar_qempty, (it & 1) ^ 1, ctx))) break;
        mbar_arrive_expect_tx(&bar_qfull, 2 * T::PL * C::Q_BYTES);
        tma_tile<T>(smem + C::OFF_Q, &maps.q, &bar_qfull, kBM, rb * kBM, h, b, p.B, T::PL);
        tma_tile<T>(smem + C::OFF_DO, &maps.dout, &bar_qfull, kBM, rb * kBM, h, b, p.B, T::PL);
      }
      for (int sweep = 0; sweep < SWEEPS && ok; ++sweep) {
        if (sweep == SWEEPS - 1 && tile + (int)gridDim.x < ntiles) {  // next tile's operands into L2
          const int nt = tile + gridDim.x, nbh = nt / p.nrb, nb = nbh / p.H, nh = nbh % p.H, nrow = (nt % p.nrb) * kBM;
          prefetch_tile<T>(&maps.q, nrow, nh, nb, p.B, T::PL);
          prefetch_tile<T>(&maps.dout, nrow, nh, nb, p.B, T::PL);
          prefetch_rows<T>(&maps.k, p.N, nh, nb, p.B, T::PL);
          prefetch_rows<T>(&maps.v, p.N, nh, nb, p.B, T::PL);
        }
        auto load_kt = [&](int cc) -> bool {  // transposed K chunk (hi) for the dQ MMA of chunk cc
          const int ts = tc % C::NDS;
          if (!mbar_wait(&bar_ktempty[ts], ((tc / C::NDS) & 1) ^ 1, ctx)) return false;
          mbar_arrive_expect_tx(&bar_ktfull[ts], C::KT_BYTES);
          tma_tileT(smem + C::OFF_KT + ts * C::KT_BYTES, &maps.kt, &bar_ktfull[ts], cc * T::CH, h, b);
          ++tc;
          return true;
        };
        for (int c = 0; c < nch && ok; c += C::PAIR) {
          if constexpr (C::WIDE) {  // (Q, K) head-dim chunks for S, then (dO, V) chunks for dP, two K/V chunks each
            for (int j = 0; j < 2 * C::NDC && ok; ++j) {
              const int ks = kc % NKV, dc = j % C::NDC;
              if (!(ok = mbar_wait(&bar_kempty[ks], ((kc / NKV) & 1) ^ 1, ctx))) break;
              mbar_arrive_expect_tx(&bar_kfull[ks], T::PL * C::K_BYTES);
              uint8_t* slot = smem + C::OFF_K + ks * T::PL * C::K_BYTES;
              if (j < C::NDC)
                tma_slot_rows<T, C::PAIR * T::CH>(slot, &bar_kfull[ks], &maps.q, rb * kBM, &maps.k, c * T::CH, dc, h,
                                                  b, p.B);
              else
                tma_slot_rows<T, C::PAIR * T::CH>(slot, &bar_kfull[ks], &maps.dout, rb * kBM, &maps.v, c * T::CH, dc,
                                                  h, b, p.B);
              ++kc;
            }
            if (!ok) break;
            if (sweep == 1 && c >= C::PAIR)  // K^T of the previous pair (its dQ MMAs follow this pair's scores)
              for (int cc = c - C::PAIR; cc < c && ok; ++cc) ok = load_kt(cc);
            continue;
          } else {
            const int ks = kc % NKV;
            if (!(ok = mbar_wait(&bar_kempty[ks], ((kc / NKV) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&bar_kfull[ks], T::PL * C::K_BYTES);
            tma_tile<T>(smem + C::OFF_K + ks * T::PL * C::K_BYTES, &maps.k, &bar_kfull[ks], T::CH, c * T::CH, h, b,
                        p.B, T::PL);
            if (!(ok = mbar_wait(&bar_vempty[ks], ((kc / NKV) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&bar_vfull[ks], T::PL * C::K_BYTES);
            tma_tile<T>(smem + C::OFF_V + ks * T::PL * C::K_BYTES, &maps.v, &bar_vfull[ks], T::CH, c * T::CH, h, b,
                        p.B, T::PL);
            ++kc;
          }
          if constexpr (!BF16)
            if (sweep == 1 && !(ok = load_kt(c))) break;
        }
        if constexpr (C::WIDE)  // K^T of the last pair
          if (sweep == 1)
            for (int cc = nch - C::PAIR; cc < nch && ok; ++cc) ok = load_kt(cc);
      }
      }
    }
  } else if (warp == T::PR_WARP) {
    if constexpr (NPR > 0) {
    prefetch_tmap(&maps.prior);
    int pc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int rb = tile % p.nrb;
      if (lane == 0) {
        for (int sweep = 0; sweep < SWEEPS && ok; ++sweep) {
          for (int c = 0; c < nch && ok; ++c) {
            const int ps = pc % NPR;
            if (!(ok = mbar_wait(&bar_prempty[ps], ((pc / NPR) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&bar_prfull[ps], kPriorTileBytes);
            tma_prior(smem + C::OFF_PR + ps * kPriorTileBytes, &maps.prior, &bar_prfull[ps], rb * kBM, c);
            ++pc;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    }
  } else if (warp == T::MMA_WARP) {
    if (lane == 0) {
      int kc = 0, sc = 0, dc = 0, it = 0;
      bool ok = true;
      auto issue = [&](bool release_k) -> bool {
        if constexpr (C::WIDE) {  // S then dP of a chunk pair, each accumulated over the head-dim chunks of its slots
          const int ss = sc % NSB;
          if (!mbar_wait(&bar_sempty[ss], ((sc / NSB) & 1) ^ 1, ctx)) return false;
          if (!mbar_wait(&bar_sempty[ss + 1], (((sc + 1) / NSB) & 1) ^ 1, ctx)) return false;
          for (int j = 0; j < 2 * C::NDC; ++j) {
            const int ks = kc % NKV, dc = j % C::NDC;
            if (!mbar_wait(&bar_kfull[ks], (kc / NKV) & 1, ctx)) return false;
            tc_fence_after();
            mma_slot_rows<T, C::PAIR * T::CH>(tmem + (j < C::NDC ? C::TM_S : C::TM_DP) + ss * T::CH,
                                              sbase + C::OFF_K + ks * T::PL * C::K_BYTES, dc > 0);
            mma_commit(&bar_kempty[ks]);
            ++kc;
          }
          mma_commit(&bar_sfull[ss]);
          mma_commit(&bar_sfull[ss + 1]);
          sc += 2;
          return true;
        }
        const int ks = kc % NKV, ss = sc % NSB;
        // phases of the full barriers count only chunk loads; the pooled landings (one per slot per tile, this
        // tile's included) complete none
        const int kpar = ((kc / NKV) - (C::POOL ? it + 1 : 0)) & 1;
        if (!mbar_wait(&bar_kfull[ks], kpar, ctx)) return false;
        if (!mbar_wait(&bar_vfull[ks], kpar, ctx)) return false;
        if (!mbar_wait(&bar_sempty[ss], ((sc / NSB) & 1) ^ 1, ctx)) return false;
        tc_fence_after();
        const uint32_t kb = sbase + C::OFF_K + ks * T::PL * C::K_BYTES;
        const uint32_t vb = sbase + C::OFF_V + ks * T::PL * C::K_BYTES;
        if constexpr (C::POOL) {
          mma_qk_ts<T, T::CH>(tmem + C::TM_S + ss * T::CH, tmem + C::TM_QA, kb, C::K_BYTES);
          mma_qk_ts<T, T::CH>(tmem + C::TM_DP + ss * T::CH, tmem + C::TM_DOA, vb, C::K_BYTES);
        } else {
          mma_qk<T, T::CH>(tmem + C::TM_S + ss * T::CH, sbase + C::OFF_Q, C::Q_BYTES, kb, C::K_BYTES);
          mma_qk<T, T::CH>(tmem + C::TM_DP + ss * T::CH, sbase + C::OFF_DO, C::Q_BYTES, vb, C::K_BYTES);
        }
        mma_commit(&bar_sfull[ss]);
        mma_commit(&bar_vempty[ks]);
        if (release_k) mma_commit(&bar_kempty[ks]);
        ++kc;
        ++sc;
        return true;
      };
      auto issue_dq = [&](int c, int kc0) -> bool {
        const int ds = dc % C::NDS;
        if (!mbar_wait(&bar_dsfull[ds], (dc / C::NDS) & 1, ctx)) return false;
        const int ks = (kc0 + c) % NKV;
        uint32_t bsrc;
        if constexpr (BF16) {
          bsrc = sbase + C::OFF_K + ks * T::PL * C::K_BYTES;
        } else {
          if (!mbar_wait(&bar_ktfull[ds], (dc / C::NDS) & 1, ctx)) return false;
          bsrc = sbase + C::OFF_KT + ds * C::KT_BYTES;
        }
        tc_fence_after();
        mma_pv<T>(tmem + C::TM_DQ, sbase + C::OFF_DS + ds * C::DS_BYTES, bsrc, c > 0);
        mma_commit(&bar_dsempty[ds]);
        if constexpr (!BF16) mma_commit(&bar_ktempty[ds]);
        if constexpr (!C::WIDE) mma_commit(&bar_kempty[ks]);  // wide: the slots were released by their MMAs
        ++dc;
        return true;
      };
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        if constexpr (!C::WIDE)
          if (!(ok = mbar_wait(&bar_qfull, it & 1, ctx))) break;
        if constexpr (C::POOL) {
          // Q and dO into tensor memory. The previous tile's S/dP MMAs, the last readers of these columns, completed
          // before its last K/V ring positions were released, and the TMA warp loaded this Q/dO only after that.
          // The landing's ring positions are released once the copies have read the pool.
          tc_fence_after();
          cp_operand_tmem<T>(tmem + C::TM_QA, sbase + C::OFF_Q, C::Q_BYTES);
          cp_operand_tmem<T>(tmem + C::TM_DOA, sbase + C::OFF_DO, C::Q_BYTES);
          // the copies are drained through the next S buffer (free once its previous use was read; the real S MMA
          // overwrites it) before the pool is released
          if (!(ok = mbar_wait(&bar_sempty[sc % NSB], ((sc / NSB) & 1) ^ 1, ctx))) break;
          cp_drain_operand<T>(tmem + C::TM_S + (sc % NSB) * T::CH, tmem + C::TM_QA, sbase + C::OFF_Q);
          cp_drain_operand<T>(tmem + C::TM_S + (sc % NSB) * T::CH, tmem + C::TM_DOA, sbase + C::OFF_Q);
          for (int s = 0; s < C::LAND; ++s, ++kc) {
            mma_commit(&bar_kempty[kc % NKV]);
            mma_commit(&bar_vempty[kc % NKV]);
          }
        }
        if constexpr (C::WIDE) {  // pairs: sweep 1; sweep 2 issues the next pair's scores before this pair's dQ
          for (int c = 0; c < nch && ok; c += C::PAIR) ok = issue(true);
          if constexpr (!DQ) continue;  // no resident Q / dO to release
          const int kc0 = kc;
          if (ok) ok = issue(false);
          for (int c = 0; c < nch && ok; c += C::PAIR) {
            if (c + C::PAIR < nch && !(ok = issue(false))) break;
            for (int cc = c; cc < c + C::PAIR && ok; ++cc) ok = issue_dq(cc, kc0);
          }
          if (ok) mma_commit(&bar_dqfull);
        } else {
        for (int c = 0; c < nch && ok; ++c) ok = issue(true);
        if constexpr (!DQ) {
          if (ok) mma_commit(&bar_qempty);  // every S/dP MMA of this tile has been issued
          continue;
        }
        const int kc0 = kc;  // first K use of sweep 2
        if (ok) ok = issue(false);
        // every S/dP MMA of this tile has been issued: Q and dO may take the next tile's (pooled: no separate buffer)
        if (!C::POOL && ok && nch == 1) mma_commit(&bar_qempty);
        for (int c = 0; c < nch && ok; ++c) {
          if constexpr (NKV >= 2 || C::WIDE) {  // look ahead: S/dP of the next chunk overlap the element-wise work
            if (c + 1 < nch && !(ok = issue(false))) break;
            if (!C::POOL && c + 2 == nch) mma_commit(&bar_qempty);
            if (!(ok = issue_dq(c, kc0))) break;
          } else {                   // one K/V buffer: the next chunk's K can only arrive after this chunk's dQ
            if (!(ok = issue_dq(c, kc0))) break;
            if (c + 1 < nch && !(ok = issue(false))) break;
            if (c + 2 == nch) mma_commit(&bar_qempty);
          }
        }
        if (ok) mma_commit(&bar_dqfull);
        }
      }
    }
  } else if (warp < T::TMA_WARP) {
    // ---------------- element-wise warps ----------------
    const Ew e = ew_id(tmem);
    const float sc_l2 = p.scale_log2;
    const size_t nrows_all = (size_t)p.B * p.H * p.N;
    int sc = 0, pc = 0, dc = 0, it = 0;
    bool ok = true;
    // the forward's row statistics (m, l1, l2) of a tile are loaded one tile ahead, so their latency is hidden
    auto load_stats = [&](int t, float (&st3)[3]) {
      const int r_ = (t % p.nrb) * kBM + e.r;
      if (t < ntiles && r_ < p.N) {
        const size_t sr = (size_t)(t / p.nrb) * p.N + r_;
        st3[0] = p.stats[sr];
        st3[1] = p.stats[nrows_all + sr];
        st3[2] = p.stats[2 * nrows_all + sr];
      }
    };
    float nst[3] = {0.f, 1.f, 1.f};
    load_stats(blockIdx.x, nst);
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
    const int row = rb * kBM + e.r;
    const bool valid = row < p.N;
    const float cst[3] = {nst[0], nst[1], nst[2]};
    load_stats(tile + gridDim.x, nst);
    const Abg ab = load_abg(p, h);
    const float aL = ab.a * kLog2e, bL = ab.b * kLog2e, gL = ab.g * kLog2e, cL = ab.c * kLog2e;
    // P1 = 2^(t - m1), P2 = 2^(Z log2 e - c2); rows past N get m1 = c2 = +inf (P1 = P2 = 0)
    float m1 = INFINITY, c2 = INFINITY;
    if (valid) {
      m1 = cst[0] + log2f(cst[1]);
      c2 = cL + log2f(cst[2]);
    }
    float acc[3] = {0.f, 0.f, 0.f};  // delta2, a, b
    for (int c = 0; c < nch && ok; ++c) {
      const int ss = sc % NSB, prs = pc % PRB;
      Prior32<BF16> pr;
      if constexpr (NPR == 0) load_prior32<BF16>(p.prior, p.np, row, c * T::CH, pr);  // before the waits
      if (!(ok = warp_wait(&bar_sfull[ss], (sc / NSB) & 1, ctx))) break;
      if constexpr (NPR > 0)
        if (!(ok = warp_wait(&bar_prfull[prs], (pc / PRB) & 1, ctx))) break;
      tc_fence_after();
      const uint8_t* prt = smem + C::OFF_PR + prs * kPriorTileBytes;
#pragma unroll 1
      for (int piece = e.wg; piece < T::PIECES; piece += T::EW) {
        uint32_t vs[32], ws[32];
        tmem_ld32_issue(e.lane_base + C::TM_S + ss * T::CH + piece * 32, vs);
        tmem_ld32_issue(e.lane_base + C::TM_DP + ss * T::CH + piece * 32, ws);
        const int nvalid = p.N - (c * T::CH + piece * 32);
        if constexpr (NPR > 0 && !BF16) prior32_smem<BF16>(prt, e.r, piece, pr);
        tmem_wait32(vs);
        tmem_pin32(ws);
        tc_fence_before();
        mbar_arrive(&bar_sempty[ss]);  // the scores are in registers: the MMA may refill the buffer
        float pa[2][3] = {};  // two interleaved partial sums per quantity (shorter dependency chains)
        auto body = [&](auto masked) {
          float p1[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            p1[j] = ex2(fmaf(__uint_as_float(vs[j]), sc_l2, -m1));
            if constexpr (decltype(masked)::value) p1[j] = (j < nvalid) ? p1[j] : 0.f;
          }
          // bf16 staged prior: four pairs per 16-byte shared-memory load next to their use (no 32-register copy)
          [[maybe_unused]] uint32_t pw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float dpj, apj;
            if constexpr (BF16 && NPR > 0) {
              if ((j & 3) == 0) {
                const uint4 u = *reinterpret_cast<const uint4*>(prt + piece * (kBM * 128) + sw128(e.r, j / 4));
                pw[0] = u.x;
                pw[1] = u.y;
                pw[2] = u.z;
                pw[3] = u.w;
              }
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pw[j & 3]));
              dpj = f.x;
              apj = f.y;
            } else {
              pr.get(j, dpj, apj);
            }
            float p2 = ex2(fmaf(aL, p1[j], fmaf(bL, dpj, fmaf(gL, apj, -c2))));
            if constexpr (decltype(masked)::value) p2 = (j < nvalid) ? p2 : 0.f;
            const float wv = p2 * __uint_as_float(ws[j]);
            float* q = pa[j & 1];
            q[0] += wv;
            q[1] = fmaf(wv, p1[j], q[1]);
            q[2] = fmaf(p2, p1[j], q[2]);
          }
        };
        if (nvalid >= 32) body(std::false_type{});
        else body(std::true_type{});
#pragma unroll
        for (int k = 0; k < 3; ++k) acc[k] += pa[0][k] + pa[1][k];
        if constexpr (NPR > 0) mbar_arrive(&bar_prempty[prs]);  // every value read from the prior tile has been used
      }
      ++sc;
      ++pc;
    }
    if constexpr (T::EW == 2) {
      if constexpr (DQ) {
        // combine the two warpgroups' row sums (warpgroup 0's first) through the dS buffers, unused until sweep 2,
        // once the previous tile's dQ store has finished reading them; both warpgroups need them for sweep 2
        if (epi_tma && threadIdx.x == 0) bulk_wait_read0();
        ew_sync(T::EWT);
        float* xs = reinterpret_cast<float*>(smem + C::OFF_DS);
#pragma unroll
        for (int k = 0; k < 3; ++k) xs[(e.wg * 3 + k) * kBM + e.r] = acc[k];
        ew_sync(T::EWT);
#pragma unroll
        for (int k = 0; k < 3; ++k) acc[k] = xs[k * kBM + e.r] + xs[(3 + k) * kBM + e.r];
        ew_sync(T::EWT);
      } else {
        // only warpgroup 0 uses the combined sums (records, d(alpha)): warpgroup 1 hands its sums over. The region
        // is rewritten only after the next tile's sweep, past this tile's partials barrier.
        float* xs = reinterpret_cast<float*>(smem + C::OFF_XS);
        if (e.wg == 1) {
#pragma unroll
          for (int k = 0; k < 3; ++k) xs[k * kBM + e.r] = acc[k];
        }
        ew_sync(T::EWT);
        if (e.wg == 0) {
#pragma unroll
          for (int k = 0; k < 3; ++k) acc[k] += xs[k * kBM + e.r];
        }
      }
    }
    const float delta2 = acc[0];
    const float ta = fmaf(-delta2, acc[2], acc[1]);  // sum dZ P1 of the row
    const float delta1 = ab.a * ta;
    if (e.wg == 0 && ok) {
      float* rec = rec_ptr<T>(p, bh, row);
      rec[0] = m1;
      rec[T::CH] = c2;
      rec[2 * T::CH] = valid ? delta1 : 0.f;
      rec[3 * T::CH] = valid ? delta2 : 0.f;
      if constexpr (T::NREC > 4) rec[4 * T::CH] = valid ? acc[2] : 0.f;  // b
    }
    // Sweep 2. d(alpha) of the row is summed again here from the explicit dZ, as sum dZ (P1 - b) with b = sum P2 P1:
    // sum dZ is 0 in exact arithmetic, but the recomputed P2 sum to 1 + eps (fp32 rounding of c2, exp2), which
    // leaves sum dZ = -eps delta2; with P1 near uniform that bias dominates sum dZ P1 (and a - delta2 b cancels to
    // a few ulps of delta2). Subtracting b sum dZ removes it to O(eps^2) for any P1.
    const float pb = acc[2];
    float gap[2] = {0.f, 0.f}, gbp[2] = {0.f, 0.f}, ggp[2] = {0.f, 0.f};  // d(alpha), d(beta), d(gamma) of the row
    if constexpr (DQ) {
    for (int c = 0; c < nch && ok; ++c) {
      const int ss = sc % NSB, ds = dc % C::NDS, prs = pc % PRB;
      Prior32<BF16> pr;
      if constexpr (NPR == 0) load_prior32<BF16>(p.prior, p.np, row, c * T::CH, pr);  // before the waits
      if (!(ok = warp_wait(&bar_sfull[ss], (sc / NSB) & 1, ctx))) break;
      if constexpr (NPR > 0)
        if (!(ok = warp_wait(&bar_prfull[prs], (pc / PRB) & 1, ctx))) break;
      tc_fence_after();
      uint8_t* dreg = smem + C::OFF_DS + ds * C::DS_BYTES;
      const uint8_t* prt = smem + C::OFF_PR + prs * kPriorTileBytes;
#pragma unroll 1
      for (int piece = e.wg; piece < T::PIECES; piece += T::EW) {
        uint32_t vs[32], ws[32];
        tmem_ld32_issue(e.lane_base + C::TM_S + ss * T::CH + piece * 32, vs);
        tmem_ld32_issue(e.lane_base + C::TM_DP + ss * T::CH + piece * 32, ws);
        const int nvalid = p.N - (c * T::CH + piece * 32);
        float v[32];
        if constexpr (NPR > 0) prior32_smem<BF16>(prt, e.r, piece, pr);
        tmem_wait32(vs);
        tmem_pin32(ws);
        tc_fence_before();
        mbar_arrive(&bar_sempty[ss]);
        auto body = [&](auto masked) {
          float p1[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            p1[j] = ex2(fmaf(__uint_as_float(vs[j]), sc_l2, -m1));
            if constexpr (decltype(masked)::value) p1[j] = (j < nvalid) ? p1[j] : 0.f;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float dpj, apj;
            pr.get(j, dpj, apj);
            float p2 = ex2(fmaf(aL, p1[j], fmaf(bL, dpj, fmaf(gL, apj, -c2))));
            if constexpr (decltype(masked)::value) p2 = (j < nvalid) ? p2 : 0.f;
            const float dz = p2 * (__uint_as_float(ws[j]) - delta2);
            v[j] = p1[j] * fmaf(ab.a, dz, -delta1);  // masked columns: p1 = 0 -> dS = 0
            gap[j & 1] = fmaf(dz, p1[j] - pb, gap[j & 1]);
            gbp[j & 1] = fmaf(dz, dpj, gbp[j & 1]);
            ggp[j & 1] = fmaf(dz, apj, ggp[j & 1]);
          }
        };
        if (nvalid >= 32) body(std::false_type{});
        else body(std::true_type{});
        if constexpr (NPR > 0) mbar_arrive(&bar_prempty[prs]);  // every value read from the prior tile has been used
        // the dS buffer is free once the dQ MMA that read it has run (waited here, after the math)
        if (!(ok = warp_wait(&bar_dsempty[ds], ((dc / C::NDS) & 1) ^ 1, ctx))) break;
        stage_row32<BF16>(dreg, e.r, piece, v);
      }
      if (!ok) break;
      fence_proxy_async_smem();
      mbar_arrive(&bar_dsfull[ds]);
      ++sc;
      ++dc;
      ++pc;
    }
    }
    // block partials of d(alpha) (without DQ: one per row from sweep 1, warpgroup 0), d(beta), d(gamma) (every
    // warpgroup's columns; without DQ the key pass writes those two)
    {
      double ga = DQ ? (valid ? (double)(gap[0] + gap[1]) : 0.0) : ((valid && e.wg == 0) ? (double)ta : 0.0);
      double gb = valid ? (double)(gbp[0] + gbp[1]) : 0.0,
             gg = valid ? (double)(ggp[0] + ggp[1]) : 0.0;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        ga += __shfl_down_sync(0xffffffffu, ga, off);
        gb += __shfl_down_sync(0xffffffffu, gb, off);
        gg += __shfl_down_sync(0xffffffffu, gg, off);
      }
      if (lane == 0) {
        red[warp][0] = ga;
        red[warp][1] = gb;
        red[warp][2] = gg;
      }
      ew_sync(T::EWT);
      if (threadIdx.x == 0) {
        double s3[3] = {0.0, 0.0, 0.0};
        for (int w = 0; w < 4 * T::EW; ++w)
          for (int k = 0; k < 3; ++k) s3[k] += red[w][k];
        double* out = p.part + ((size_t)bh * p.nrb + rb) * 3;
        if constexpr (DQ || !C::WIDE) out[0] = s3[0];  // wide without dQ: the key pass sums d(alpha)
        if constexpr (DQ) {
          out[1] = s3[1];
          out[2] = s3[2];
        }
      }
    }
    if (DQ && ok) ok = warp_wait(&bar_dqfull, it & 1, ctx);
    tc_fence_after();
    if constexpr (!DQ) {
    } else if (epi_tma) {
      // every dQ MMA of the tile has completed (dqfull), so the dS buffers hold the staged dQ tile
      if (ok) stage_acc<DP / (32 * T::EW)>(e.lane_base + C::TM_DQ, e.wg * 32, 32 * T::EW, smem + C::OFF_DS, e.r, p.inv_sqrt_d);
      store_tile<T>(&maps.out0, smem + C::OFF_DS, p.D, rb * kBM, h, b, ok);
    } else if (ok) {
      const long long qoff = (long long)b * p.dq_str[0] + (long long)h * p.dq_str[1] + (long long)row * p.dq_str[2];
#pragma unroll 1
      for (int d0 = e.wg * 32; d0 < DP; d0 += 32 * T::EW) {
        float v[32];
        tmem_ld32(e.lane_base + C::TM_DQ + d0, v);  // collective: every lane loads, valid rows store
        if (valid && d0 < p.D) store_row32<BF16>(p.dq, qoff, p.dq_str[3], d0, p.D, v, p.inv_sqrt_d);
      }
    }
    tc_fence_before();  // the dQ reads above precede this warp's next hand-offs to the MMA warp
    }
    if (epi_tma && threadIdx.x == 0) bulk_wait_read0();  // shared memory outlives the last store's reads
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ===============================================================================================================
// Backward key pass: one CTA per (128-key block, b*h); keys on TMEM lanes. For each chunk of CH queries:
//   S^T = K Q^T, dP^T = V dO^T; P1, P2, dZ, dS from the row records; dV += P2^T dO, dK += dS^T Q.
// The chunk's row records arrive by bulk copy together with its Q / dO tiles. With SDS (the dS-scratch backward) the
// TMA warp also stores each staged dS^T tile to the scratch (for the dQ GEMM; fp32 at head dim 64 stores it
// transposed) and the element-wise warps accumulate the key block's d(beta) = sum dZ Dp and d(gamma) = sum dZ Ap
// (fp32 above head dim 64 also d(alpha) = sum dZ (P1 - b)).
// ===============================================================================================================
template <bool BF16, int DP, bool SDS = false>
struct ColsCfg : Tile<BF16, DP> {
  using T = Tile<BF16, DP>;
  // fp32 beyond 64: no resident K / V blocks; (K, Q) and (V, dO) reach the S^T and dP^T MMAs in head-dim chunks
  // through a ring of NRS slots (the transposed Q / dO chunks for dK, dV still arrive per query chunk)
  static constexpr bool WIDE = !BF16 && DP > 64;
  static constexpr int NDC = WIDE ? DP / T::KB : 1;
  static constexpr int NRS = WIDE ? 3 : 0;
  // fp32 at head dim 64 ("pooled"): the K and V blocks (hi/lo planes) are the tensor-memory A operands of the S^T and
  // dP^T MMAs. They land by TMA in a shared-memory pool that, once copied into tensor memory, holds the query-chunk
  // ring for the rest of the tile: the landing takes the ring's next NQ positions, so the ring's order and phases
  // carry the hand-over both ways.
  static constexpr bool POOL = !BF16 && !WIDE;
  // pooled: 2 (a 3-deep ring, 8 % faster at C2, gave dK rows of one tile that differed between runs in ~1 run of 4,
  // with the drain and the single staging buffer alike; 2 is bitwise stable)
  static constexpr int NQ = (BF16 && DP <= 128) ? 3 : POOL ? 2 : 1;   // query-chunk (Q, dO) buffers
  // wide: the two buffers hold one pair of query chunks (below)
  static constexpr int NSB = ((BF16 && DP <= 128) || POOL || WIDE) ? 2 : 1;  // S^T / dP^T buffers in TMEM
  // wide: the S^T/dP^T MMAs cover pairs of 32-query chunks (the slots carry a head-dim chunk of K or V and of two Q or
  // dO chunks) into both score buffers; the next pair issues after the first chunk's dV/dK, and each chunk's row
  // records load before the next pair's slots (the element-wise warps read a chunk's records before they free its
  // scores, so records queued behind slots that wait for those scores would stop the pipeline)
  static constexpr int PAIR = WIDE ? 2 : 1;
  static constexpr int SLOT_PLANE = kSlotPlaneBytesRows<PAIR * T::CH>;
  static constexpr int LAND = POOL ? NQ : 0;               // ring positions the K/V landing takes per tile
  static_assert(LAND == 0 || LAND == NQ, "a landing takes every slot of the ring once");
  static constexpr int NR = 2;                             // row-record buffers
  static constexpr int NST = ((BF16 && DP <= 64) || POOL) ? 2 : 1;  // buffers for the staged P2^T / dS^T tiles
  static constexpr int NPR = !BF16 ? 0 : (DP <= 64 ? 2 : 1);  // staged prior buffers (0: read from L2)
  static constexpr int K_BYTES = WIDE ? 0 : kBM * DP * T::EB;    // per plane (K and V blocks)
  static constexpr int Q_BYTES = WIDE ? 0 : T::CH * DP * T::EB;  // per plane per buffer (Q and dO chunks)
  static constexpr int QT_BYTES = BF16 ? 0 : DP * 128;      // fp32: transposed Q / dO chunk (hi)
  static constexpr int ST_BYTES = kBM * 128;                // P2^T or dS^T tile
  static constexpr int REC_BYTES = T::NREC * T::CH * 4;     // row records of one query chunk: m1, c2, delta1, delta2[, b]
  static constexpr int OFF_RS = 0;
  static constexpr int OFF_K = OFF_RS + NRS * 2 * SLOT_PLANE;
  static constexpr int OFF_V = OFF_K + T::PL * K_BYTES;
  static constexpr int KV_END = OFF_V + T::PL * K_BYTES;
  static constexpr int OFF_Q = POOL ? OFF_K : KV_END;
  static constexpr int OFF_DO = OFF_Q + NQ * T::PL * Q_BYTES;
  static constexpr int OFF_QT = OFF_DO + NQ * T::PL * Q_BYTES;
  static constexpr int OFF_DOT = OFF_QT + NQ * QT_BYTES;
  static constexpr int RING_END = OFF_DOT + NQ * QT_BYTES;
  static constexpr int OFF_P2 = (POOL && KV_END > RING_END) ? KV_END : RING_END;  // pooled: past the larger use
  static constexpr int OFF_DS = OFF_P2 + NST * ST_BYTES;
  static constexpr int OFF_PR = OFF_DS + NST * ST_BYTES;
  static constexpr int OFF_REC = OFF_PR + NPR * kPriorTileBytes;
  // fp32 at head dim 64 with a dS scratch: the TF32 dQ GEMM needs dS K-major along the keys, so each staged tile is
  // also written transposed, [32 queries][128 keys] as four 128-byte-swizzled regions of 32 keys, for its TMA store
  // (above 64 there is no shared memory for it: the tile is stored as staged and the dQ GEMM transposes it)
  static constexpr bool DST = SDS && !BF16 && !WIDE;
  static constexpr int DST_BYTES = 32 * kBM * 4;
  static constexpr int OFF_DST = (OFF_REC + NR * REC_BYTES + 1023) / 1024 * 1024;
  static constexpr int SMEM = DST ? OFF_DST + NST * DST_BYTES : OFF_REC + NR * REC_BYTES;
  static_assert(SMEM + 1024 <= kSmemPerBlock, "key pass: dynamic + static shared memory above the per-block limit");
  static_assert(!DST || (T::CH == 32 && T::PIECES == 1 && T::EW == 1), "transposed dS staging: one 32-query piece");
  static constexpr int TM_S = 0;
  static constexpr int TM_DP = NSB * T::CH;
  static constexpr int TM_DK = 2 * NSB * T::CH;
  static constexpr int TM_DV = TM_DK + DP;
  static constexpr int TM_KA = TM_DV + DP;                                      // pooled: K (hi, lo) as A operand
  static constexpr int TM_VA = TM_KA + (POOL ? T::PL * kAColsPerPlane<T> : 0);  // pooled: V (hi, lo)
  static constexpr int TMEM_NEED = TM_VA + (POOL ? T::PL * kAColsPerPlane<T> : 0);
  static_assert(TMEM_NEED <= 512, "key pass: tensor-memory columns above 512");
  static constexpr int TMEM_COLS = pow2_cols(TMEM_NEED);
  // dK and dV leave in turn through the P2^T / dS^T buffers (contiguous, free once the tile's last MMA has run)
  static constexpr bool EPI_TMA = BF16 && T::NKB * kBM * 128 <= 2 * NST * ST_BYTES;
};

template <bool BF16, int DP, bool SDS>
__global__ void __launch_bounds__(Tile<BF16, DP>::NTHREADS, 1)
    geoattn_bwd_cols_kernel(const __grid_constant__ TileMaps maps, const KParams p) {
  using C = ColsCfg<BF16, DP, SDS>;
  using T = typename C::T;
  constexpr int NQ = C::NQ, NSB = C::NSB, NR = C::NR, NST = C::NST, NPR = C::NPR;
  constexpr int SLAG = NQ > 1 ? NQ - 1 : 1;  // chunks by which the dS stores trail the query-chunk loads
  static_assert(!SDS || SLAG <= NQ + NST - 1, "dS stores lagging further would wait on loads that wait on them");
  if (smem_misaligned(p.status)) return;  // uniform over the CTA, before any barrier or allocation
  uint8_t* smem = smem_raw;
  __shared__ uint64_t bar_kvfull, bar_kvempty, bar_qfull[3], bar_qempty[3], bar_sfull[2], bar_sempty[2], bar_tfull[2],
      bar_tempty[2], bar_prfull[2], bar_prempty[2], bar_recfull[2], bar_recempty[2], bar_done, bar_rsfull[3],
      bar_rsempty[3];
  static_assert(NQ <= 3 && NSB <= 2 && NST <= 2 && NPR <= 2 && NR <= 2 && C::NRS <= 3,
                "ring deeper than its barrier array");
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  __shared__ double redc[8][3];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // chunks every role iterates; wide: whole pairs (an extra chunk past N has +inf row records: P1 = P2 = dS = 0)
  const int nch = C::PAIR == 2 ? (((p.N + T::CH - 1) / T::CH + 1) & ~1) : (p.N + T::CH - 1) / T::CH;
  const int ntiles = p.nrb * p.B * p.H;  // tile = (128-key block, b*h); persistent CTAs stride over tiles
  WaitCtx ctx{&abort_flag, p.status};
  const bool epi_tma = C::EPI_TMA && p.out_tma;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_kvfull, 1);
    mbar_init(&bar_kvempty, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bar_qfull[i], 1);
      mbar_init(&bar_qempty[i], 1);
      mbar_init(&bar_rsfull[i], 1);
      mbar_init(&bar_rsempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_recfull[i], 1);
      mbar_init(&bar_recempty[i], T::EWT);
      mbar_init(&bar_sfull[i], 1);
      mbar_init(&bar_sempty[i], T::EWT);
      mbar_init(&bar_tfull[i], T::EWT);
      mbar_init(&bar_tempty[i], SDS ? 2 : 1);  // the MMAs that read the tile (and, with SDS, its store)
      mbar_init(&bar_prfull[i], 1);
      mbar_init(&bar_prempty[i], T::EWT);
    }
    mbar_init(&bar_done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t sbase = smem_u32(smem);

  if (warp == T::TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&maps.q);
      prefetch_tmap(&maps.k);
      prefetch_tmap(&maps.v);
      prefetch_tmap(&maps.dout);
      bool ok = true;
      int it = 0, rc = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int kblk = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
      // dS^T tile of chunk c (use g of its staging slot) to the scratch once the element-wise warps staged it; the
      // slot is handed back (second arrival on its empty barrier) once the store has read it
      auto store_ds = [&](int g, int c) -> bool {
        const int ts = g % NST;
        if (!mbar_wait(&bar_tfull[ts], (g / NST) & 1, ctx)) return false;
        if constexpr (C::DST) {  // fp32: the transposed tile, [queries][keys], one store per 32-key region
          for (int rg = 0; rg < 4; ++rg)
            tma_store_3d(&maps.dsT, smem + C::OFF_DST + ts * C::DST_BYTES + rg * (32 * 128), kblk * kBM + rg * 32,
                         c * T::CH, bh);
        } else {  // the staged dS^T tile itself, [keys][queries] (bf16; wide fp32: 32 queries, TF32-rounded)
          tma_store_3d(&maps.dsT, smem + C::OFF_DS + ts * C::ST_BYTES, c * T::CH, kblk * kBM, bh);
        }
        bulk_commit();
        bulk_wait_read0();
        mbar_arrive(&bar_tempty[ts]);
        return true;
      };
      const int q0 = it * (nch + C::LAND) + C::LAND;  // query-chunk ring position of chunk 0
      if constexpr (C::POOL) {  // K and V into the pool once its ring positions are free (the previous tile's MMAs ran)
        for (int s = q0 - C::LAND; s < q0 && ok; ++s) ok = mbar_wait(&bar_qempty[s % NQ], ((s / NQ) & 1) ^ 1, ctx);
        if (!ok) break;
        mbar_arrive_expect_tx(&bar_kvfull, 2 * T::PL * C::K_BYTES);
        tma_tile<T>(smem + C::OFF_K, &maps.k, &bar_kvfull, kBM, kblk * kBM, h, b, p.B, T::PL);
        tma_tile<T>(smem + C::OFF_V, &maps.v, &bar_kvfull, kBM, kblk * kBM, h, b, p.B, T::PL);
      } else if constexpr (!C::WIDE) {  // K and V blocks once the previous tile's last S^T/dP^T MMAs read the old ones
        if (!(ok = mbar_wait(&bar_kvempty, (it & 1) ^ 1, ctx))) break;
        mbar_arrive_expect_tx(&bar_kvfull, 2 * T::PL * C::K_BYTES);
        tma_tile<T>(smem + C::OFF_K, &maps.k, &bar_kvfull, kBM, kblk * kBM, h, b, p.B, T::PL);
        tma_tile<T>(smem + C::OFF_V, &maps.v, &bar_kvfull, kBM, kblk * kBM, h, b, p.B, T::PL);
      }
      if (tile + (int)gridDim.x < ntiles) {  // next tile's key block into L2
        const int nt = tile + gridDim.x, nbh = nt / p.nrb, nb = nbh / p.H, nh = nbh % p.H, nrow = (nt % p.nrb) * kBM;
        prefetch_tile<T>(&maps.k, nrow, nh, nb, p.B, T::PL);
        prefetch_tile<T>(&maps.v, nrow, nh, nb, p.B, T::PL);
      }
      // wide: the slots of the pair starting at chunk c, (K, Q) head-dim chunks for S^T then (V, dO) for dP^T
      auto load_slots = [&](int c) -> bool {
        if constexpr (!C::WIDE) {
          (void)c;
          return true;
        } else {
        for (int j = 0; j < 2 * C::NDC; ++j) {
          const int ss = rc % C::NRS, dc = j % C::NDC;
          if (!mbar_wait(&bar_rsempty[ss], ((rc / C::NRS) & 1) ^ 1, ctx)) return false;
          mbar_arrive_expect_tx(&bar_rsfull[ss], 2 * C::SLOT_PLANE);
          uint8_t* slot = smem + C::OFF_RS + ss * 2 * C::SLOT_PLANE;
          if (j < C::NDC)
            tma_slot_rows<T, C::PAIR * T::CH>(slot, &bar_rsfull[ss], &maps.k, kblk * kBM, &maps.q, c * T::CH, dc, h,
                                              b, p.B);
          else
            tma_slot_rows<T, C::PAIR * T::CH>(slot, &bar_rsfull[ss], &maps.v, kblk * kBM, &maps.dout, c * T::CH, dc,
                                              h, b, p.B);
          ++rc;
        }
        return true;
        }
      };
      for (int c = 0; c < nch; ++c) {
        const int gc = it * nch + c;  // chunk count over all tiles (buffer slots and phases)
        const int gq = q0 + c;            // query-chunk ring position
        const int qs = gq % NQ;
        const int rs = gc % NR;  // the chunk's row records, on their own ring
        auto load_records = [&]() -> bool {
          if (!mbar_wait(&bar_recempty[rs], ((gc / NR) & 1) ^ 1, ctx)) return false;
          mbar_arrive_expect_tx(&bar_recfull[rs], C::REC_BYTES);
          bulk_load(smem + C::OFF_REC + rs * C::REC_BYTES, p.rowrec + ((size_t)bh * p.nchp + c) * T::NREC * T::CH,
                    C::REC_BYTES, &bar_recfull[rs]);
          return true;
        };
        // wide: the chunk's records first (the element-wise warps read them before they free the chunk's score
        // buffer, which the next pair's MMA waits for), then a pair's slots before the previous pair's odd chunk
        // (before chunk 0 for the first pair), so the transposed Q/dO of each chunk, which waits for the dV/dK before
        // it, never holds back scores the MMA warp issues before that dV/dK
        if constexpr (C::WIDE) {
          if (!(ok = load_records())) break;
          const int pc = (c == 0) ? 0 : ((c & 1) ? c + 1 : -1);  // first chunk of the pair whose slots load here
          if (pc >= 0 && pc < nch && !(ok = load_slots(pc))) break;
        }
        if (!(ok = mbar_wait(&bar_qempty[qs], ((gq / NQ) & 1) ^ 1, ctx))) break;
        mbar_arrive_expect_tx(&bar_qfull[qs], 2 * T::PL * C::Q_BYTES + 2 * C::QT_BYTES);
        if constexpr (!C::WIDE) {
          tma_tile<T>(smem + C::OFF_Q + qs * T::PL * C::Q_BYTES, &maps.q, &bar_qfull[qs], T::CH, c * T::CH, h, b,
                      p.B, T::PL);
          tma_tile<T>(smem + C::OFF_DO + qs * T::PL * C::Q_BYTES, &maps.dout, &bar_qfull[qs], T::CH, c * T::CH, h, b,
                      p.B, T::PL);
        }
        if constexpr (!BF16) {
          tma_tileT(smem + C::OFF_QT + qs * C::QT_BYTES, &maps.qt, &bar_qfull[qs], c * T::CH, h, b);
          tma_tileT(smem + C::OFF_DOT + qs * C::QT_BYTES, &maps.dot, &bar_qfull[qs], c * T::CH, h, b);
        }
        if constexpr (!C::WIDE)
          if (!(ok = load_records())) break;
        // the dS stores trail the loads by SLAG chunks, so a store's wait for its tile never holds back the loads
        // the MMAs need next. The load of chunk c waits for the dV/dK of chunk c - NQ, which waits for its staging,
        // which waits for the store of chunk c - NQ - NST; by chunk c this loop has stored chunk c - 1 - SLAG, so
        // SLAG <= NQ + NST - 1 keeps the chain acyclic
        if constexpr (SDS)
          if (c >= SLAG && !(ok = store_ds(gc - SLAG, c - SLAG))) break;
      }
      if constexpr (SDS)
        for (int c2 = nch - SLAG < 0 ? 0 : nch - SLAG; c2 < nch && ok; ++c2)
          ok = store_ds(it * nch + c2, c2);
      }
    }
  } else if (warp == T::PR_WARP) {
    if constexpr (NPR > 0) {
      if (lane == 0) {
        prefetch_tmap(&maps.prior);
        bool ok = true;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
          const int kblk = tile % p.nrb;
          for (int c = 0; c < nch && ok; ++c) {
            const int gc = it * nch + c, ps = gc % NPR;
            if (!(ok = mbar_wait(&bar_prempty[ps], ((gc / NPR) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&bar_prfull[ps], kPriorTileBytes);
            tma_prior(smem + C::OFF_PR + ps * kPriorTileBytes, &maps.prior, &bar_prfull[ps], kblk * kBM, c);
          }
        }
      }
    }
  } else if (warp == T::MMA_WARP) {
    if (lane == 0) {
      bool ok = true;
      int it = 0, rc = 0;
      int qoff = 0;  // query-chunk ring position minus chunk count (the pooled K/V landings take ring positions)
      auto issue_s = [&](int gc) -> bool {
        if constexpr (C::WIDE) {  // the pair (gc, gc + 1) into both score buffers
          static_assert(NSB == C::PAIR, "a pair takes every score buffer");
          if (!mbar_wait(&bar_sempty[0], ((gc / NSB) & 1) ^ 1, ctx)) return false;
          if (!mbar_wait(&bar_sempty[1], (((gc + 1) / NSB) & 1) ^ 1, ctx)) return false;
          for (int j = 0; j < 2 * C::NDC; ++j) {
            const int rs = rc % C::NRS, dc = j % C::NDC;
            if (!mbar_wait(&bar_rsfull[rs], (rc / C::NRS) & 1, ctx)) return false;
            tc_fence_after();
            mma_slot_rows<T, C::PAIR * T::CH>(tmem + (j < C::NDC ? C::TM_S : C::TM_DP),
                                              sbase + C::OFF_RS + rs * 2 * C::SLOT_PLANE, dc > 0);
            mma_commit(&bar_rsempty[rs]);
            ++rc;
          }
          mma_commit(&bar_sfull[0]);
          mma_commit(&bar_sfull[1]);
          return true;
        }
        const int gq = gc + qoff, qs = gq % NQ, ss = gc % NSB;
        // phases of bar_qfull[qs] count only query-chunk loads; the pooled landings (one per slot per tile, this
        // tile's included) complete no phase of it
        const int qpar = ((gq / NQ) - (C::POOL ? it + 1 : 0)) & 1;
        if (!mbar_wait(&bar_qfull[qs], qpar, ctx)) return false;
        if (!mbar_wait(&bar_sempty[ss], ((gc / NSB) & 1) ^ 1, ctx)) return false;
        tc_fence_after();
        if constexpr (C::POOL) {
          mma_qk_ts<T, T::CH>(tmem + C::TM_S + ss * T::CH, tmem + C::TM_KA,
                              sbase + C::OFF_Q + qs * T::PL * C::Q_BYTES, C::Q_BYTES);
          mma_qk_ts<T, T::CH>(tmem + C::TM_DP + ss * T::CH, tmem + C::TM_VA,
                              sbase + C::OFF_DO + qs * T::PL * C::Q_BYTES, C::Q_BYTES);
        } else {
          mma_qk<T, T::CH>(tmem + C::TM_S + ss * T::CH, sbase + C::OFF_K, C::K_BYTES,
                           sbase + C::OFF_Q + qs * T::PL * C::Q_BYTES, C::Q_BYTES);
          mma_qk<T, T::CH>(tmem + C::TM_DP + ss * T::CH, sbase + C::OFF_V, C::K_BYTES,
                           sbase + C::OFF_DO + qs * T::PL * C::Q_BYTES, C::Q_BYTES);
        }
        mma_commit(&bar_sfull[ss]);
        return true;
      };
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int g0 = it * nch, q0 = it * (nch + C::LAND) + C::LAND;
      qoff = q0 - g0;
      if constexpr (!C::WIDE)
        if (!(ok = mbar_wait(&bar_kvfull, it & 1, ctx))) break;
      if constexpr (C::POOL) {
        // K and V into tensor memory. The previous tile's S^T/dP^T MMAs, the last readers of these columns, completed
        // before its last query chunks' ring positions were released, and the TMA warp loaded this K/V only after
        // that. The landing's ring positions are released once the copies have read the pool.
        tc_fence_after();
        cp_operand_tmem<T>(tmem + C::TM_KA, sbase + C::OFF_K, C::K_BYTES);
        cp_operand_tmem<T>(tmem + C::TM_VA, sbase + C::OFF_V, C::K_BYTES);
        // the copies are drained through chunk 0's S^T buffer (free once its previous use was read; the real S^T
        // MMA overwrites it) before the pool is released
        if (!(ok = mbar_wait(&bar_sempty[g0 % NSB], ((g0 / NSB) & 1) ^ 1, ctx))) break;
        cp_drain_operand<T>(tmem + C::TM_S + (g0 % NSB) * T::CH, tmem + C::TM_KA, sbase + C::OFF_K);
        cp_drain_operand<T>(tmem + C::TM_S + (g0 % NSB) * T::CH, tmem + C::TM_VA, sbase + C::OFF_K);
        for (int s = q0 - C::LAND; s < q0; ++s) mma_commit(&bar_qempty[s % NQ]);
      }
      if (ok) ok = issue_s(g0);
      // every S^T/dP^T MMA of this tile has been issued: the K/V buffers may take the next tile's blocks
      if (!C::POOL && ok && nch == 1) mma_commit(&bar_kvempty);
      for (int c = 0; c < nch && ok; ++c) {
        const int gc = g0 + c;
        if (!C::WIDE && NSB == 2 && c + 1 < nch) {
          if (!(ok = issue_s(gc + 1))) break;
          if (!C::POOL && c + 2 == nch) mma_commit(&bar_kvempty);
        }
        const int gq = gc + qoff, qs = gq % NQ, ts = gc % NST;
        if (!(ok = mbar_wait(&bar_tfull[ts], (gc / NST) & 1, ctx))) break;
        if constexpr (C::WIDE)  // the transposed Q / dO chunks (the slots carried the score operands)
          if (!(ok = mbar_wait(&bar_qfull[qs], (gq / NQ) & 1, ctx))) break;
        tc_fence_after();
        uint32_t dob, qb;
        if constexpr (BF16) {
          dob = sbase + C::OFF_DO + qs * C::Q_BYTES;
          qb = sbase + C::OFF_Q + qs * C::Q_BYTES;
        } else {
          dob = sbase + C::OFF_DOT + qs * C::QT_BYTES;
          qb = sbase + C::OFF_QT + qs * C::QT_BYTES;
        }
        mma_pv<T>(tmem + C::TM_DV, sbase + C::OFF_P2 + ts * C::ST_BYTES, dob, c > 0);
        mma_pv<T>(tmem + C::TM_DK, sbase + C::OFF_DS + ts * C::ST_BYTES, qb, c > 0);
        mma_commit(&bar_tempty[ts]);
        mma_commit(&bar_qempty[qs]);
        if (C::WIDE && (c & 1) == 0 && c + 2 < nch && !(ok = issue_s(gc + 2))) break;  // the next pair
        if (NSB == 1 && c + 1 < nch) {
          if (!(ok = issue_s(gc + 1))) break;
          if (c + 2 == nch) mma_commit(&bar_kvempty);
        }
      }
      if (ok) mma_commit(&bar_done);
      }
    }
  } else if (warp < T::TMA_WARP) {
    // ---------------- element-wise warps: thread = key ----------------
    const Ew e = ew_id(tmem);
    const float sc_l2 = p.scale_log2;
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int kblk = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
    const int key = kblk * kBM + e.r;
    const Abg ab = load_abg(p, h);
    const float aL = ab.a * kLog2e, bL = ab.b * kLog2e, gL = ab.g * kLog2e;
    const int pkey = key < p.np ? key : 0;
    const bool kvalid = key < p.N;
    (void)pkey;
    if (epi_tma) {  // the previous tile's dV store has finished reading the P2^T / dS^T buffers
      if (threadIdx.x == 0) bulk_wait_read0();
      ew_sync(T::EWT);
    }
    float gbp[2] = {0.f, 0.f}, ggp[2] = {0.f, 0.f};  // with SDS: this key's d(beta), d(gamma) partials
    // wide fp32 with SDS: this key's d(alpha) partial, sum dZ (P1 - b) with the row's b = sum P2 P1 (the row pass has
    // no second sweep to sum it there; the - b term cancels the bias of sum dZ, which the recomputed P2 leave at
    // -eps delta2 instead of 0)
    float gap[2] = {0.f, 0.f};
    // P2 and dS of one 32-column piece from its scores S^T, dP^T, the chunk's row records and the prior; keys past N
    // (last block only) produce rows of P2^T / dS^T that only reach dK/dV rows that are never stored, so no per-key
    // mask is needed
    // (bf16, staged prior tile `prt`: each group of four pairs is read from shared memory next to its use, one
    // 16-byte load, instead of 32 registers of pairs held across the piece)
    auto piece_math = [&](const float* rec, int piece, const uint32_t (&vs)[32], const uint32_t (&ws)[32],
                          const Prior32<BF16>& pr, const uint8_t* prt, float (&v)[32], float (&w)[32]) {
#pragma unroll
      for (int j4 = 0; j4 < 32; j4 += 4) {
        const int q = piece * 32 + j4;
        const float4 m4 = *reinterpret_cast<const float4*>(rec + q);
        const float4 c4 = *reinterpret_cast<const float4*>(rec + T::CH + q);
        const float4 d1 = *reinterpret_cast<const float4*>(rec + 2 * T::CH + q);
        const float4 d2 = *reinterpret_cast<const float4*>(rec + 3 * T::CH + q);
        const float mm[4] = {m4.x, m4.y, m4.z, m4.w}, cc[4] = {c4.x, c4.y, c4.z, c4.w};
        const float e1[4] = {d1.x, d1.y, d1.z, d1.w}, e2[4] = {d2.x, d2.y, d2.z, d2.w};
        [[maybe_unused]] float bb[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (SDS && C::WIDE) {
          const float4 b4 = *reinterpret_cast<const float4*>(rec + 4 * T::CH + q);
          bb[0] = b4.x;
          bb[1] = b4.y;
          bb[2] = b4.z;
          bb[3] = b4.w;
        }
        [[maybe_unused]] uint32_t pw[4] = {0u, 0u, 0u, 0u};
        if constexpr (BF16 && NPR > 0) {
          const uint4 u = *reinterpret_cast<const uint4*>(prt + piece * (kBM * 128) + sw128(e.r, j4 / 4));
          pw[0] = u.x;
          pw[1] = u.y;
          pw[2] = u.z;
          pw[3] = u.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = j4 + k;
          float dpj, apj;
          if constexpr (BF16 && NPR > 0) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pw[k]));
            dpj = f.x;
            apj = f.y;
          } else {
            pr.get(j, dpj, apj);
          }
          const float p1 = ex2(fmaf(__uint_as_float(vs[j]), sc_l2, -mm[k]));
          const float p2 = ex2(fmaf(aL, p1, fmaf(bL, dpj, fmaf(gL, apj, -cc[k]))));
          const float dz = p2 * (__uint_as_float(ws[j]) - e2[k]);
          v[j] = p2;
          w[j] = p1 * fmaf(ab.a, dz, -e1[k]);
          if constexpr (SDS) {
            gbp[k & 1] = fmaf(dz, dpj, gbp[k & 1]);
            ggp[k & 1] = fmaf(dz, apj, ggp[k & 1]);
          }
          if constexpr (SDS && C::WIDE) gap[k & 1] = fmaf(dz, p1 - bb[k], gap[k & 1]);
        }
      }
    };
    for (int c = 0; c < nch; ++c) {
      const int gc = it * nch + c;
      const int ss = gc % NSB, rs = gc % NR, ts = gc % NST;
      if (!ok) continue;
      Prior32<BF16> pr;
      // prior from L2 (no staged tile, fp32 only: one piece per chunk): loads issued before the waits, so that their
      // latency overlaps the wait for the chunk's scores instead of following it
      if constexpr (NPR == 0) {
        static_assert(T::PIECES == 1 && T::EW == 1, "prior read from L2 in one piece per chunk");
        load_prior32<BF16>(p.priorT, p.np, pkey, c * T::CH, pr);
      }
      if (!(ok = warp_wait(&bar_sfull[ss], (gc / NSB) & 1, ctx))) continue;
      if constexpr (NPR > 0)
        if (!(ok = warp_wait(&bar_prfull[gc % NPR], (gc / NPR) & 1, ctx))) continue;
      // the chunk's row records (rows past N carry m1 = c2 = +inf: P1 = P2 = dS = 0 in their columns)
      if (!(ok = warp_wait(&bar_recfull[rs], (gc / NR) & 1, ctx))) continue;
      tc_fence_after();
      const float* rec = reinterpret_cast<const float*>(smem + C::OFF_REC + rs * C::REC_BYTES);
      uint8_t* p2reg = smem + C::OFF_P2 + ts * C::ST_BYTES;
      uint8_t* dsreg = smem + C::OFF_DS + ts * C::ST_BYTES;
      const uint8_t* prt = smem + C::OFF_PR + (NPR > 0 ? (gc % (NPR > 0 ? NPR : 1)) : 0) * kPriorTileBytes;
#pragma unroll 1
      for (int piece = e.wg; piece < T::PIECES; piece += T::EW) {
        uint32_t vs[32], ws[32];
        tmem_ld32_issue(e.lane_base + C::TM_S + ss * T::CH + piece * 32, vs);
        tmem_ld32_issue(e.lane_base + C::TM_DP + ss * T::CH + piece * 32, ws);
        tmem_wait32(vs);
        tmem_pin32(ws);
        tc_fence_before();
        mbar_arrive(&bar_sempty[ss]);  // the scores are in registers: the MMA may refill the buffer
        float v[32], w[32];
        piece_math(rec, piece, vs, ws, pr, prt, v, w);
        mbar_arrive(&bar_recempty[rs]);  // the records and the prior tile are read and used
        if constexpr (NPR > 0) mbar_arrive(&bar_prempty[gc % NPR]);
        // the staging tiles are free once the previous chunk's dV/dK MMAs have run (waited here, after the math)
        if (!(ok = warp_wait(&bar_tempty[ts], ((gc / NST) & 1) ^ 1, ctx))) break;
        stage_row32<BF16>(p2reg, e.r, piece, v);
        stage_row32<BF16>(dsreg, e.r, piece, w);
        if constexpr (C::DST) {  // dS[query][key], TF32-rounded as for the MMAs: key e.r is word e.r % 32 of region e.r / 32
          uint8_t* treg = smem + C::OFF_DST + ts * C::DST_BYTES + (e.r >> 5) * (32 * 128);
          const int kk = e.r & 31;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            *reinterpret_cast<float*>(treg + sw128(j, kk >> 2) + (kk & 3) * 4) = round_tf32(w[j]);
        }
      }
      if (!ok) continue;
      fence_proxy_async_smem();
      mbar_arrive(&bar_tfull[ts]);
    }
    if constexpr (SDS) {  // block partials of d(beta), d(gamma) (keys past N excluded); wide: d(alpha) too
      double gb = kvalid ? (double)(gbp[0] + gbp[1]) : 0.0, gg = kvalid ? (double)(ggp[0] + ggp[1]) : 0.0;
      double ga = (C::WIDE && kvalid) ? (double)(gap[0] + gap[1]) : 0.0;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        gb += __shfl_down_sync(0xffffffffu, gb, off);
        gg += __shfl_down_sync(0xffffffffu, gg, off);
        ga += __shfl_down_sync(0xffffffffu, ga, off);
      }
      if (lane == 0) {
        redc[warp][0] = gb;
        redc[warp][1] = gg;
        redc[warp][2] = ga;
      }
      ew_sync(T::EWT);
      if (threadIdx.x == 0) {
        double s3[3] = {0.0, 0.0, 0.0};
        for (int w = 0; w < 4 * T::EW; ++w)
          for (int k = 0; k < 3; ++k) s3[k] += redc[w][k];
        double* out = p.part + ((size_t)bh * p.nrb + kblk) * 3;
        if constexpr (C::WIDE) out[0] = s3[2];
        out[1] = s3[0];
        out[2] = s3[1];
      }
    }
    if (ok) ok = warp_wait(&bar_done, it & 1, ctx);
    // with SDS the staging tiles are also read by the dS stores: wait for the last ones before the epilogue
    if constexpr (SDS) {
      for (int k = 0; k < NST && k < nch && ok; ++k) {
        const int g = it * nch + nch - 1 - k;
        ok = warp_wait(&bar_tempty[g % NST], (g / NST) & 1, ctx);
      }
    }
    tc_fence_after();
    if (epi_tma) {
      // every MMA of the tile has completed (done): the P2^T / dS^T buffers take dK, then dV
      uint8_t* stg = smem + C::OFF_P2;
      if (ok) stage_acc<DP / (32 * T::EW)>(e.lane_base + C::TM_DK, e.wg * 32, 32 * T::EW, stg, e.r, p.inv_sqrt_d);
      store_tile<T>(&maps.out0, stg, p.D, kblk * kBM, h, b, ok);
      if (threadIdx.x == 0) bulk_wait_read0();
      ew_sync(T::EWT);
      if (ok) stage_acc<DP / (32 * T::EW)>(e.lane_base + C::TM_DV, e.wg * 32, 32 * T::EW, stg, e.r, 1.0f);
      store_tile<T>(&maps.out1, stg, p.D, kblk * kBM, h, b, ok);
    } else if (ok) {
      const long long koff = (long long)b * p.dk_str[0] + (long long)h * p.dk_str[1] + (long long)key * p.dk_str[2];
      const long long voff = (long long)b * p.dv_str[0] + (long long)h * p.dv_str[1] + (long long)key * p.dv_str[2];
#pragma unroll 1
      for (int d0 = e.wg * 32; d0 < DP; d0 += 32 * T::EW) {
        float v[32];
        tmem_ld32(e.lane_base + C::TM_DK + d0, v);
        if (kvalid && d0 < p.D) store_row32<BF16>(p.dk, koff, p.dk_str[3], d0, p.D, v, p.inv_sqrt_d);
        tmem_ld32(e.lane_base + C::TM_DV + d0, v);
        if (kvalid && d0 < p.D) store_row32<BF16>(p.dv, voff, p.dv_str[3], d0, p.D, v, 1.0f);
      }
    }
    tc_fence_before();  // the dK/dV reads above precede this warp's next hand-offs to the MMA warp
    }
    if (epi_tma && threadIdx.x == 0) bulk_wait_read0();  // shared memory outlives the last store's reads
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ===============================================================================================================
// dQ = dS K / sqrt(d) (bf16), from the dS^T tiles [b*h][key][query] the key pass stored. One CTA per (128-query
// block, b*h), persistent; it loops over 64-key chunks: acc[128 x DP] += dS[128 x 64] . K[64 x DP], dS read as an
// MN-major A operand (queries contiguous) and K as an MN-major B operand (head dim contiguous), the accumulator
// double-buffered in tensor memory so that one tile's epilogue overlaps the next tile's MMAs.
// Warps: 4 epilogue warps (thread = TMEM lane = query row), 1 TMA warp, 1 MMA warp.
// ===============================================================================================================
template <int DP>
struct DqCfg {
  using T = Tile<true, DP>;
  static constexpr int NSTAGE = 4;
  static constexpr int A_BYTES = 2 * 64 * 128;            // dS: two 64-query halves x 64 keys x 128 B
  static constexpr int B_BYTES = T::NKB * 64 * 128;       // K chunk: NKB regions of 64 keys x 128 B
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int OFF_OUT = NSTAGE * STAGE;          // epilogue staging: NKB regions of 128 rows x 128 B
  static constexpr int SMEM = OFF_OUT + T::NKB * kBM * 128;
  static constexpr int TMEM_COLS = pow2_cols(2 * DP);
  static constexpr int NTHREADS = 128 + 64;
  static constexpr int TMA_WARP = 4, MMA_WARP = 5;
};

template <int DP>
__device__ __forceinline__ void mma_dq(uint32_t tmem_acc, uint32_t a_base, uint32_t b_base, bool accumulate) {
  constexpr uint32_t idesc = instr_desc(1, 1, 1, 128, DP);  // bf16, A and B MN-major
#pragma unroll
  for (int s = 0; s < 4; ++s) {                            // K = 16 keys per MMA
    const uint64_t ad = smem_desc_sw128(a_base + s * 16 * 128, 64 * 128, 1024);
    const uint64_t bd = smem_desc_sw128(b_base + s * 16 * 128, 64 * 128, 1024);
    mma_ss<Kind::kF16>(tmem_acc, ad, bd, idesc, (accumulate || s > 0) ? 1u : 0u);
  }
}

template <int DP>
__global__ void __launch_bounds__(DqCfg<DP>::NTHREADS, 1)
    geoattn_bwd_dq_kernel(const __grid_constant__ TileMaps maps, const KParams p) {
  using C = DqCfg<DP>;
  using T = typename C::T;
  constexpr int NS = C::NSTAGE;
  if (smem_misaligned(p.status)) return;  // uniform over the CTA, before any barrier or allocation
  uint8_t* smem = smem_raw;
  __shared__ uint64_t bar_full[NS], bar_empty[NS], bar_accfull[2], bar_accempty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nchunks = (p.N + 63) / 64;  // key chunks (keys past N meet zero-filled K rows)
  const int ntiles = p.nrb * p.B * p.H;
  WaitCtx ctx{&abort_flag, p.status};
  const bool epi_tma = p.out_tma != 0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_accfull[i], 1);
      mbar_init(&bar_accempty[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t sbase = smem_u32(smem);

  if (warp == C::TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&maps.dsT);
      prefetch_tmap(&maps.k);
      int sc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
        for (int c = 0; c < nchunks && ok; ++c, ++sc) {
          const int st = sc % NS;
          if (!(ok = mbar_wait(&bar_empty[st], ((sc / NS) & 1) ^ 1, ctx))) break;
          uint8_t* dst = smem + st * C::STAGE;
          mbar_arrive_expect_tx(&bar_full[st], C::STAGE);
          tma_load_3d(dst, &maps.dsT, &bar_full[st], rb * kBM, c * 64, bh);
          tma_load_3d(dst + 64 * 128, &maps.dsT, &bar_full[st], rb * kBM + 64, c * 64, bh);
          tma_tile<T>(dst + C::A_BYTES, &maps.k, &bar_full[st], 64, c * 64, h, b, p.B, 1);
        }
      }
    }
  } else if (warp == C::MMA_WARP) {
    if (lane == 0) {
      int sc = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!(ok = mbar_wait(&bar_accempty[ab], ((it >> 1) & 1) ^ 1, ctx))) break;
        tc_fence_after();
        for (int c = 0; c < nchunks && ok; ++c, ++sc) {
          const int st = sc % NS;
          if (!(ok = mbar_wait(&bar_full[st], (sc / NS) & 1, ctx))) break;
          tc_fence_after();
          mma_dq<DP>(tmem + ab * DP, sbase + st * C::STAGE, sbase + st * C::STAGE + C::A_BYTES, c > 0);
          mma_commit(&bar_empty[st]);
        }
        if (ok) mma_commit(&bar_accfull[ab]);
      }
    }
  } else {
    // ---------------- epilogue warps ----------------
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
      const int row = rb * kBM + r, ab = it & 1;
      if (ok) ok = warp_wait(&bar_accfull[ab], (it >> 1) & 1, ctx);
      tc_fence_after();
      if (epi_tma) {
        if (threadIdx.x == 0) bulk_wait_read0();  // the previous tile's store has read the staging tile
        ew_sync(128);
        if (ok) {
#pragma unroll 1
          for (int d0 = 0; d0 < DP; d0 += 64)  // two 32-column pieces per TMEM wait
            stage_acc<2>(lane_base + ab * DP, d0, 32, smem + C::OFF_OUT, r, p.inv_sqrt_d);
        }
        tc_fence_before();
        mbar_arrive(&bar_accempty[ab]);
        fence_proxy_async_smem();
        ew_sync(128);
        if (threadIdx.x == 0 && ok) {
          for (int kb = 0; kb < T::NKB && kb * 64 < p.D; ++kb)
            tma_store_4d(&maps.out0, smem + C::OFF_OUT + kb * (kBM * 128), kb * 64, rb * kBM, h, b);
          bulk_commit();
        }
      } else {
        const long long qoff = (long long)b * p.dq_str[0] + (long long)h * p.dq_str[1] + (long long)row * p.dq_str[2];
        if (ok) {
#pragma unroll 1
          for (int d0 = 0; d0 < DP; d0 += 32) {
            float v[32];
            tmem_ld32(lane_base + ab * DP + d0, v);
            if (row < p.N && d0 < p.D) store_row32<true>(p.dq, qoff, p.dq_str[3], d0, p.D, v, p.inv_sqrt_d);
          }
        }
        tc_fence_before();
        mbar_arrive(&bar_accempty[ab]);
      }
    }
    if (epi_tma && threadIdx.x == 0) bulk_wait_read0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ===============================================================================================================
// dQ = dS K / sqrt(d) for fp32 storage (TF32, 1 term) at head dim 64, from the fp32 dS tiles [b*h][query][key] the key
// pass stored (K-major along the keys: TF32 MMAs take K-major operands only) and the transposed hi plane of K
// [b*h][d][key] (K-major along the keys). One CTA per (128-query block, b*h), persistent; per 32-key chunk four
// M = 128, N = DP, K = 8 MMAs; the accumulator double-buffered in tensor memory. Warps: 4 epilogue, 1 TMA, 1 MMA.
// ===============================================================================================================
template <int DP>
struct DqTf32Cfg {
  using T = Tile<false, DP>;
  static constexpr int NSTAGE = 4;
  static constexpr int A_BYTES = kBM * 128;  // dS: 128 queries x 32 keys (one 128-byte region per row)
  static constexpr int B_BYTES = DP * 128;   // K^T: DP rows x 32 keys
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = NSTAGE * STAGE;
  static constexpr int TMEM_COLS = pow2_cols(2 * DP);
  static constexpr int NTHREADS = 128 + 64;
  static constexpr int TMA_WARP = 4, MMA_WARP = 5;
  static_assert(SMEM + 1024 <= kSmemPerBlock, "TF32 dQ GEMM: shared memory above the per-block limit");
};

template <int DP>
__global__ void __launch_bounds__(DqTf32Cfg<DP>::NTHREADS, 1)
    geoattn_bwd_dq_tf32_kernel(const __grid_constant__ TileMaps maps, const KParams p) {
  using C = DqTf32Cfg<DP>;
  constexpr int NS = C::NSTAGE;
  if (smem_misaligned(p.status)) return;  // uniform over the CTA, before any barrier or allocation
  uint8_t* smem = smem_raw;
  __shared__ uint64_t bar_full[NS], bar_empty[NS], bar_accfull[2], bar_accempty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nchunks = (p.N + 31) / 32;  // key chunks (keys past N meet the zero-padded columns of K^T)
  const int ntiles = p.nrb * p.B * p.H;
  WaitCtx ctx{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_accfull[i], 1);
      mbar_init(&bar_accempty[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t sbase = smem_u32(smem);

  if (warp == C::TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&maps.dsT);
      prefetch_tmap(&maps.kt);
      int sc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
        for (int c = 0; c < nchunks && ok; ++c, ++sc) {
          const int st = sc % NS;
          if (!(ok = mbar_wait(&bar_empty[st], ((sc / NS) & 1) ^ 1, ctx))) break;
          uint8_t* dst = smem + st * C::STAGE;
          mbar_arrive_expect_tx(&bar_full[st], C::STAGE);
          tma_load_3d(dst, &maps.dsT, &bar_full[st], c * 32, rb * kBM, bh);
          tma_tileT(dst + C::A_BYTES, &maps.kt, &bar_full[st], c * 32, h, b);
        }
      }
    }
  } else if (warp == C::MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(2, 0, 0, 128, DP);  // tf32, A and B K-major
      int sc = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!(ok = mbar_wait(&bar_accempty[ab], ((it >> 1) & 1) ^ 1, ctx))) break;
        tc_fence_after();
        for (int c = 0; c < nchunks && ok; ++c, ++sc) {
          const int st = sc % NS;
          if (!(ok = mbar_wait(&bar_full[st], (sc / NS) & 1, ctx))) break;
          tc_fence_after();
          const uint32_t a = sbase + st * C::STAGE, bsrc = a + C::A_BYTES;
#pragma unroll
          for (int s = 0; s < 4; ++s)  // K = 8 keys (32 bytes) per MMA
            mma_ss<Kind::kTF32>(tmem + ab * DP, smem_desc_sw128(a + s * 32, 16, 1024),
                                smem_desc_sw128(bsrc + s * 32, 16, 1024), idesc, (c > 0 || s > 0) ? 1u : 0u);
          mma_commit(&bar_empty[st]);
        }
        if (ok) mma_commit(&bar_accfull[ab]);
      }
    }
  } else {
    // ---------------- epilogue warps: thread = query row ----------------
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
      const int row = rb * kBM + r, ab = it & 1;
      if (ok) ok = warp_wait(&bar_accfull[ab], (it >> 1) & 1, ctx);
      tc_fence_after();
      const long long qoff = (long long)b * p.dq_str[0] + (long long)h * p.dq_str[1] + (long long)row * p.dq_str[2];
      if (ok) {
#pragma unroll 1
        for (int d0 = 0; d0 < DP; d0 += 32) {
          float v[32];
          tmem_ld32(lane_base + ab * DP + d0, v);
          if (row < p.N && d0 < p.D) store_row32<false>(p.dq, qoff, p.dq_str[3], d0, p.D, v, p.inv_sqrt_d);
        }
      }
      tc_fence_before();
      mbar_arrive(&bar_accempty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ===============================================================================================================
// dQ = dS K / sqrt(d) for fp32 storage (TF32, 1 term) above head dim 64, from the fp32 dS^T tiles [b*h][key][query]
// the wide key pass stored (its staged A operand of dK, queries contiguous). TF32 MMAs take K-major operands only, so
// the four element-wise warps transpose each 32-key x 128-query tile in shared memory into the K-major A operand
// [query][key] (thread = query row: 32 reads down one column of the landed tile, 8 swizzled 16-byte writes) before the
// MMA reads it; B is the transposed hi plane of K [b*h][d][key]. One CTA per (128-query block, b*h), persistent; per
// 32-key chunk four M = 128, N = DP, K = 8 MMAs; the accumulator double-buffered in tensor memory; the same warps
// store dQ (row stores). Warps: 4 transposing / epilogue, 1 TMA, 1 MMA.
// ===============================================================================================================
template <int DP>
struct DqTf32tCfg {
  using T = Tile<false, DP>;
  static constexpr int NSTAGE = 4;
  static constexpr int RAW_BYTES = 4 * 32 * 128;  // the landed dS^T tile: four 32-query boxes of 32 keys x 128 B
  static constexpr int A_BYTES = kBM * 128;       // dS K-major: 128 queries x 32 keys
  static constexpr int B_BYTES = DP * 128;        // K^T: DP rows x 32 keys
  static constexpr int STAGE = RAW_BYTES + A_BYTES + B_BYTES;
  static constexpr int SMEM = NSTAGE * STAGE;
  static constexpr int TMEM_COLS = pow2_cols(2 * DP);
  static constexpr int NTHREADS = 128 + 64;
  static constexpr int TMA_WARP = 4, MMA_WARP = 5;
  static_assert(SMEM + 1024 <= kSmemPerBlock, "transposing TF32 dQ GEMM: shared memory above the per-block limit");
  static_assert(2 * DP <= 512, "transposing TF32 dQ GEMM: two accumulators in tensor memory");
};

template <int DP>
__global__ void __launch_bounds__(DqTf32tCfg<DP>::NTHREADS, 1)
    geoattn_bwd_dq_tf32t_kernel(const __grid_constant__ TileMaps maps, const KParams p) {
  using C = DqTf32tCfg<DP>;
  constexpr int NS = C::NSTAGE;
  if (smem_misaligned(p.status)) return;  // uniform over the CTA, before any barrier or allocation
  uint8_t* smem = smem_raw;
  __shared__ uint64_t bar_full[NS], bar_afull[NS], bar_empty[NS], bar_accfull[2], bar_accempty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nchunks = (p.N + 31) / 32;  // key chunks (keys past N meet zero dS rows and zero-padded K^T columns)
  const int ntiles = p.nrb * p.B * p.H;
  WaitCtx ctx{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_afull[i], 128);
      mbar_init(&bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_accfull[i], 1);
      mbar_init(&bar_accempty[i], 128);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t sbase = smem_u32(smem);

  if (warp == C::TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&maps.dsT);
      prefetch_tmap(&maps.kt);
      int sc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
        for (int c = 0; c < nchunks && ok; ++c, ++sc) {
          const int st = sc % NS;
          if (!(ok = mbar_wait(&bar_empty[st], ((sc / NS) & 1) ^ 1, ctx))) break;
          uint8_t* dst = smem + st * C::STAGE;
          mbar_arrive_expect_tx(&bar_full[st], C::RAW_BYTES + C::B_BYTES);
          for (int j = 0; j < 4; ++j)
            tma_load_3d(dst + j * (32 * 128), &maps.dsT, &bar_full[st], rb * kBM + j * 32, c * 32, bh);
          tma_tileT(dst + C::RAW_BYTES + C::A_BYTES, &maps.kt, &bar_full[st], c * 32, h, b);
        }
      }
    }
  } else if (warp == C::MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(2, 0, 0, 128, DP);  // tf32, A and B K-major
      int sc = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!(ok = mbar_wait(&bar_accempty[ab], ((it >> 1) & 1) ^ 1, ctx))) break;
        tc_fence_after();
        for (int c = 0; c < nchunks && ok; ++c, ++sc) {
          const int st = sc % NS;
          if (!(ok = mbar_wait(&bar_afull[st], (sc / NS) & 1, ctx))) break;
          tc_fence_after();
          const uint32_t a = sbase + st * C::STAGE + C::RAW_BYTES, bsrc = a + C::A_BYTES;
#pragma unroll
          for (int s = 0; s < 4; ++s)  // K = 8 keys (32 bytes) per MMA
            mma_ss<Kind::kTF32>(tmem + ab * DP, smem_desc_sw128(a + s * 32, 16, 1024),
                                smem_desc_sw128(bsrc + s * 32, 16, 1024), idesc, (c > 0 || s > 0) ? 1u : 0u);
          mma_commit(&bar_empty[st]);
        }
        if (ok) mma_commit(&bar_accfull[ab]);
      }
    }
  } else {
    // ---------------- transposing / epilogue warps: thread = query row ----------------
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    int sc = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int rb = tile % p.nrb, bh = tile / p.nrb, b = bh / p.H, h = bh % p.H;
      const int row = rb * kBM + r, ab = it & 1;
      for (int c = 0; c < nchunks; ++c, ++sc) {
        const int st = sc % NS;
        if (ok) ok = warp_wait(&bar_full[st], (sc / NS) & 1, ctx);
        // the landed tile (box j = queries 32 j .. 32 j + 31): key k of query r at row k of box r / 32, word r % 32
        const uint8_t* raw = smem + st * C::STAGE + (r >> 5) * (32 * 128);
        uint8_t* arow = smem + st * C::STAGE + C::RAW_BYTES;
        if (ok) {
#pragma unroll
          for (int k4 = 0; k4 < 8; ++k4) {
            float4 v;
            v.x = *reinterpret_cast<const float*>(raw + sw128(4 * k4, (r & 31) >> 2) + (r & 3) * 4);
            v.y = *reinterpret_cast<const float*>(raw + sw128(4 * k4 + 1, (r & 31) >> 2) + (r & 3) * 4);
            v.z = *reinterpret_cast<const float*>(raw + sw128(4 * k4 + 2, (r & 31) >> 2) + (r & 3) * 4);
            v.w = *reinterpret_cast<const float*>(raw + sw128(4 * k4 + 3, (r & 31) >> 2) + (r & 3) * 4);
            *reinterpret_cast<float4*>(arow + sw128(r, k4)) = v;
          }
        }
        fence_proxy_async_smem();  // the generic writes above become visible to the MMA's reads
        mbar_arrive(&bar_afull[st]);
      }
      if (ok) ok = warp_wait(&bar_accfull[ab], (it >> 1) & 1, ctx);
      tc_fence_after();
      const long long qoff = (long long)b * p.dq_str[0] + (long long)h * p.dq_str[1] + (long long)row * p.dq_str[2];
      if (ok) {
#pragma unroll 1
        for (int d0 = 0; d0 < DP; d0 += 32) {
          float v[32];
          tmem_ld32(lane_base + ab * DP + d0, v);
          if (row < p.N && d0 < p.D) store_row32<false>(p.dq, qoff, p.dq_str[3], d0, p.D, v, p.inv_sqrt_d);
        }
      }
      tc_fence_before();
      mbar_arrive(&bar_accempty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace geoattn
