// Segmented flash-attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// Gradient of the segmented non-causal attention of attention.cu (the reference calls
// FA3 / FA2 / SDPA backward through autograd: ospnext/modules/attention.py:460-517).
// Inputs q, k, v, o, dO and the forward's LSE; δ = rowsum(dO ∘ O) comes from a small
// pre-kernel.  P is recomputed from S and the LSE, never stored.
//
// Two kernels, no atomics:
//   dkdv: one CTA per 128-key tile.  It loops over the query tiles of its segment and
//         computes, with the keys on the TMEM lanes,
//           Sᵀ  = K·Qᵢᵀ,   Pᵀ = 2^(Sᵀ·scale·log2e − LSE·log2e)   (bf16 back over Sᵀ in TMEM)
//           dPᵀ = V·dOᵢᵀ,  dSᵀ = Pᵀ∘(dPᵀ − δ)                  (bf16 back over dPᵀ)
//           dV += Pᵀ·dOᵢ,  dK += dSᵀ·Qᵢ                         (A operand from TMEM)
//         TMEM: Sᵀ | dPᵀ | dV | dK (512 columns for D = 128).
//   dq:   one CTA per 128-query tile, looping over the key tiles of its segment:
//           S = Q·Kⱼᵀ, dP = dO·Vⱼᵀ, dS = P∘(dP − δ) (bf16 over dP), dQ += dS·Kⱼ.
// The MMA order lets the elementwise warps of one step overlap the tensor core:
//   dkdv: … dV(i) Sᵀ(i+1) | dK(i) dPᵀ(i+1) | dV(i+1) Sᵀ(i+2) …
//   dq:   … S(j+1) once S(j) is in registers, dQ(j) then dP(j+1) …
// Warps: 0 TMA producer, 1 MMA issuer (one elected thread), 4..11 elementwise (two warps
// per TMEM lane quarter, each owning half of the 128 columns).  Every wait is bounded.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"
#include "attn_common.cuh"

namespace osp {

namespace bwd {
constexpr int kT = 128;          // rows per tile (queries or keys)
constexpr int kThreads = 384;
constexpr float kLog2e = 1.4426950408889634f;
}  // namespace bwd

struct AttnBwdArgs {
  const int* seg_q;
  const int* seg_k;
  int Nq, Nk, H;
  const float* lse;        // [B, H, Nq] natural log
  const float* delta;      // [B, H, Nq]
  __nv_bfloat16* dq;       // [B, Nq, H, D]
  __nv_bfloat16* dk;       // [B, Nk, H, D]
  __nv_bfloat16* dv;       // [B, Nk, H, D]
  float scale;             // softmax scale
  int* err;
};

// ---------------------------------------------------------------------------- δ = rowsum(dO∘O)
// One warp per (token, head) row; D/32 elements per lane.
template <int D>
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                      float* __restrict__ delta, int B, int N, int H) {
  const long row = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;   // over B·N·H
  const int lane = threadIdx.x % 32;
  if (row >= (long)B * N * H) return;
  const long base = row * D;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    const int c = (i * 32 + lane) * 2;
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(o + base + c);
    const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(dout + base + c);
    acc = fmaf(__low2float(a), __low2float(g), acc);
    acc = fmaf(__high2float(a), __high2float(g), acc);
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) {
    const int h = (int)(row % H);
    const long bn = row / H;
    const int b = (int)(bn / N), n = (int)(bn % N);
    delta[((long)b * H + h) * N + n] = acc;
  }
}

// bf16 operands written back into TMEM: each of the two warps sharing a lane quarter owns
// 64 fp32 columns of a row and packs its 64 values as 32 bf16-pair columns at the start of
// its own range (half h → columns 64h … 64h+31), so neither overwrites columns the other
// has not read yet.  K-step k (16 rows of the MMA's K dimension = 8 pair columns) of the
// TS-form MMA therefore starts at column 8k, plus 32 for the second half.
__device__ __forceinline__ uint32_t tmem_pair_col(int k) { return 8u * k + (k >= 4 ? 32u : 0u); }

// Store 32 fp32 values (one TMEM row chunk) scaled, as bf16, to 64 contiguous bytes.
__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16* dst, const uint32_t* v, float mul) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w;
    w.x = pack_bf16x2(__uint_as_float(v[8 * i + 0]) * mul, __uint_as_float(v[8 * i + 1]) * mul);
    w.y = pack_bf16x2(__uint_as_float(v[8 * i + 2]) * mul, __uint_as_float(v[8 * i + 3]) * mul);
    w.z = pack_bf16x2(__uint_as_float(v[8 * i + 4]) * mul, __uint_as_float(v[8 * i + 5]) * mul);
    w.w = pack_bf16x2(__uint_as_float(v[8 * i + 6]) * mul, __uint_as_float(v[8 * i + 7]) * mul);
    d4[i] = w;
  }
}

// ---------------------------------------------------------------------------- dK, dV
template <int D>
struct DkdvSmem {
  static constexpr int BOX = bwd::kT * 128;          // 128 rows × 128 bytes
  static constexpr int DB = D / 64;
  static constexpr int TILE = DB * BOX;              // one 128 × D bf16 tile
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = TILE;
  static constexpr int OFF_STAGE = 2 * TILE;         // 2 stages of (Qᵢ, dOᵢ)
  static constexpr int STAGE = 2 * TILE;
  static constexpr int OFF_VEC = OFF_STAGE + 2 * STAGE;   // 2 stages × (lse2[128], δ[128]) fp32
  static constexpr int OFF_BAR = OFF_VEC + 2 * 2 * bwd::kT * 4;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
};

template <int D>
__global__ void __launch_bounds__(bwd::kThreads, 1)
attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                     AttnBwdArgs args) {
  using L = DkdvSmem<D>;
  using namespace bwd;
  const int kblk = blockIdx.x;
  const int s = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / args.H;
  const int h = bh % args.H;
  const int q_seg0 = args.seg_q[s], q_seg1 = args.seg_q[s + 1];
  const int k_seg0 = args.seg_k[s], k_seg1 = args.seg_k[s + 1];
  const int k_start = k_seg0 + kblk * kT;
  if (k_start >= k_seg1) return;                                   // CTA-uniform
  const int n_q = (q_seg1 - q_seg0 + kT - 1) / kT;
  const int krow0 = b * args.Nk + k_start;
  const int qrow0 = b * args.Nq + q_seg0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sStage = smem + L::OFF_STAGE;
  float* sVec = reinterpret_cast<float*>(smem + L::OFF_VEC);       // [stage][lse2 | δ][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;      // [2]  (TMA tx + 32 producer-lane arrivals)
  uint64_t* q_empty = bars + 3;     // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* dp_full = bars + 6;
  uint64_t* p_full = bars + 7;      // 8 warps
  uint64_t* ds_full = bars + 8;     // 8 warps
  uint64_t* done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 11);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&q_full[i], 1 + 32); mbar_init(&q_empty[i], 1); }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_full, 8);
    mbar_init(ds_full, 8);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128u, tDV = tmem + 256u, tDK = tmem + 256u + (uint32_t)D;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0 && n_q > 0) {          // (nothing is loaded for a segment without queries)
      mbar_expect_tx(kv_full, 2 * L::TILE);
      for (int db = 0; db < L::DB; ++db) {
        tma_load_3d(&tmK, kv_full, sK + db * L::BOX, db * 64, h, krow0);
        tma_load_3d(&tmV, kv_full, sV + db * L::BOX, db * 64, h, krow0);
      }
    }
    const float* lse_bh = args.lse + ((long)b * args.H + h) * args.Nq;
    const float* del_bh = args.delta + ((long)b * args.H + h) * args.Nq;
    for (int i = 0; i < n_q && !*abort_flag; ++i) {
      const int st = i & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&q_empty[st], ((i >> 1) & 1) ^ 1, args.err, kErrAttnProducer);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) { *abort_flag = 1; break; }
      if (lane == 0) {
        mbar_expect_tx(&q_full[st], L::STAGE);
        uint8_t* dst = sStage + st * L::STAGE;
        for (int db = 0; db < L::DB; ++db) {
          tma_load_3d(&tmQ, &q_full[st], dst + db * L::BOX, db * 64, h, qrow0 + i * kT);
          tma_load_3d(&tmDO, &q_full[st], dst + L::TILE + db * L::BOX, db * 64, h, qrow0 + i * kT);
        }
      }
      // LSE·log2e and δ of this query tile (0 past the segment end: those columns are masked)
      float* v = sVec + st * 2 * kT;
#pragma unroll
      for (int c = lane; c < kT; c += 32) {
        const int q = q_seg0 + i * kT + c;
        const bool in = q < q_seg1;
        v[c] = in ? lse_bh[q] * kLog2e : 0.f;
        v[kT + c] = in ? del_bh[q] : 0.f;
      }
      mbar_arrive(&q_full[st]);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_T = idesc_bf16(128, kT);                       // Sᵀ, dPᵀ: N = 128 queries
      constexpr uint32_t ID_G = idesc_bf16(128, D, /*b_mn_major=*/true);   // dV, dK: N = D
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
      // X·Yᵀ with X (keys) and Y (queries) both K-major tiles in smem
      auto mma_nt = [&](uint32_t d, uint32_t xa, uint32_t ya) {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k / 4) * L::BOX + (k % 4) * 32;
          umma_bf16(d, sdesc_sw128(xa + off, 16, 1024), sdesc_sw128(ya + off, 16, 1024), ID_T, k > 0 ? 1u : 0u);
        }
      };
      // acc += A·Y with A (bf16, keys × queries) in TMEM and Y (queries × D) MN-major in smem
      auto mma_ts = [&](uint32_t d, uint32_t a_tmem, uint32_t ya, bool acc) {
#pragma unroll
        for (int k = 0; k < kT / 16; ++k)
          umma_bf16_ts(d, a_tmem + tmem_pair_col(k), sdesc_sw128(ya + k * 2048, L::BOX, 1024), ID_G,
                       (acc || k > 0) ? 1u : 0u);
      };
      auto qa = [&](int i) { return smem_u32(sStage + (i & 1) * L::STAGE); };
      auto da = [&](int i) { return smem_u32(sStage + (i & 1) * L::STAGE + L::TILE); };
      bool ok = n_q > 0 && mbar_wait(kv_full, 0, args.err, kErrAttnMma);
      if (ok) ok = mbar_wait(&q_full[0], 0, args.err, kErrAttnMma);
      if (ok) {
        tc_fence_after();
        mma_nt(tS, ka, qa(0));
        umma_commit(s_full);
        mma_nt(tDP, va, da(0));
        umma_commit(dp_full);
      }
      for (int i = 0; i < n_q && ok; ++i) {
        if (!(ok = mbar_wait(p_full, i & 1, args.err, kErrAttnMma))) break;
        tc_fence_after();
        mma_ts(tDV, tS, da(i), i > 0);                      // dV += Pᵀ·dOᵢ
        const bool more = i + 1 < n_q;
        if (more) {
          if (!(ok = mbar_wait(&q_full[(i + 1) & 1], ((i + 1) >> 1) & 1, args.err, kErrAttnMma))) break;
          tc_fence_after();
          mma_nt(tS, ka, qa(i + 1));                         // Sᵀ(i+1) after dV(i) read Pᵀ(i)
          umma_commit(s_full);
        }
        if (!(ok = mbar_wait(ds_full, i & 1, args.err, kErrAttnMma))) break;
        tc_fence_after();
        mma_ts(tDK, tDP, qa(i), i > 0);                     // dK += dSᵀ·Qᵢ
        umma_commit(&q_empty[i & 1]);
        if (more) {
          mma_nt(tDP, va, da(i + 1));                        // dPᵀ(i+1) after dK(i) read dSᵀ(i)
          umma_commit(dp_full);
        }
      }
      if (!ok) *abort_flag = 1;
      if (n_q > 0) umma_commit(done);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ elementwise (warps 4..11)
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;                       // columns half·64 … +63
    const int r = quarter * 32 + lane;                      // key row inside the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float c2 = args.scale * kLog2e;
    bool ok = true;
    for (int i = 0; i < n_q; ++i) {
      const int st = i & 1;
      const float* v = sVec + st * 2 * kT + half * 64;
      const int nvq = min(kT, q_seg1 - q_seg0 - i * kT) - half * 64;   // valid columns in this half
      // ---- Pᵀ
      // the stage's LSE/δ (written by the producer lanes before their q_full arrival)
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[st], (i >> 1) & 1, args.err, kErrAttnSoftmax)))) break;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(s_full, i & 1, args.err, kErrAttnSoftmax)))) break;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(tS + lane_off + half * 64, sr);
      tmem_ld32(tS + lane_off + half * 64 + 32, sr + 32);
      tmem_ld_wait();
      float p[64];
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 l4 = *reinterpret_cast<const float4*>(v + 4 * c4);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 4 * c4 + e;
          const float x = fmaf(__uint_as_float(sr[c]), c2, -lv[e]);
          p[c] = c < nvq ? ex2(x) : 0.f;
        }
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        tmem_st4(tS + lane_off + half * 64 + c8 * 4, pack_bf16x2(p[8 * c8 + 0], p[8 * c8 + 1]),
                 pack_bf16x2(p[8 * c8 + 2], p[8 * c8 + 3]), pack_bf16x2(p[8 * c8 + 4], p[8 * c8 + 5]),
                 pack_bf16x2(p[8 * c8 + 6], p[8 * c8 + 7]));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // ---- dSᵀ = Pᵀ∘(dPᵀ − δ)
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(dp_full, i & 1, args.err, kErrAttnSoftmax)))) break;
      tc_fence_after();
      tmem_ld32(tDP + lane_off + half * 64, sr);
      tmem_ld32(tDP + lane_off + half * 64 + 32, sr + 32);
      tmem_ld_wait();
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const float4 d0 = *reinterpret_cast<const float4*>(v + kT + 8 * c8);
        const float4 d1 = *reinterpret_cast<const float4*>(v + kT + 8 * c8 + 4);
        const float dl[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
        float g[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = p[8 * c8 + e] * (__uint_as_float(sr[8 * c8 + e]) - dl[e]);
        tmem_st4(tDP + lane_off + half * 64 + c8 * 4, pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]),
                 pack_bf16x2(g[4], g[5]), pack_bf16x2(g[6], g[7]));
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (!ok) *abort_flag = 1;
    // ---- epilogue: dV, dK·scale → bf16 (zeros when the segment has no queries)
    if (n_q > 0) {
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(done, 0, args.err, kErrAttnTeardown)))) *abort_flag = 1;
      tc_fence_after();
    }
    const int key = k_start + r;
    const bool valid = ok && key < k_seg1;
    const long orow = (((long)b * args.Nk + key) * args.H + h) * D;
#pragma unroll 1
    for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
      uint32_t a[32], g[32];
      if (n_q > 0) {
        tmem_ld32(tDV + lane_off + c, a);
        tmem_ld32(tDK + lane_off + c, g);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) a[e] = g[e] = 0u;
      }
      if (valid) {
        store_row32_bf16(args.dv + orow + c, a, 1.0f);
        store_row32_bf16(args.dk + orow + c, g, args.scale);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------- dQ
template <int D>
struct DqSmem {
  static constexpr int BOX = bwd::kT * 128;
  static constexpr int DB = D / 64;
  static constexpr int TILE = DB * BOX;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = TILE;
  static constexpr int OFF_KV = 2 * TILE;            // 2 slots of (Kⱼ, Vⱼ)
  static constexpr int SLOT = 2 * TILE;
  static constexpr int OFF_BAR = OFF_KV + 2 * SLOT;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
};

template <int D>
__global__ void __launch_bounds__(bwd::kThreads, 1)
attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   AttnBwdArgs args) {
  using L = DqSmem<D>;
  using namespace bwd;
  const int qblk = blockIdx.x;
  const int s = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / args.H;
  const int h = bh % args.H;
  const int q_seg0 = args.seg_q[s], q_seg1 = args.seg_q[s + 1];
  const int k_seg0 = args.seg_k[s], k_seg1 = args.seg_k[s + 1];
  const int q_start = q_seg0 + qblk * kT;
  if (q_start >= q_seg1) return;
  const int n_kv = (k_seg1 - k_seg0 + kT - 1) / kT;
  const int qrow0 = b * args.Nq + q_start;
  const int krow0 = b * args.Nk + k_seg0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sDO = smem + L::OFF_DO;
  uint8_t* sKV = smem + L::OFF_KV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;     // [2]
  uint64_t* kv_empty = bars + 3;    // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_cons = bars + 6;      // 8 warps: S(j) is in registers
  uint64_t* dp_full = bars + 7;
  uint64_t* ds_full = bars + 8;     // 8 warps
  uint64_t* done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 11);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    mbar_init(s_full, 1);
    mbar_init(s_cons, 8);
    mbar_init(dp_full, 1);
    mbar_init(ds_full, 8);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128u, tDQ = tmem + 256u;

  if (warp == 0) {
    if (lane == 0 && n_kv > 0) {         // (nothing is loaded for a segment without keys)
      mbar_expect_tx(q_full, 2 * L::TILE);
      for (int db = 0; db < L::DB; ++db) {
        tma_load_3d(&tmQ, q_full, sQ + db * L::BOX, db * 64, h, qrow0);
        tma_load_3d(&tmDO, q_full, sDO + db * L::BOX, db * 64, h, qrow0);
      }
      for (int j = 0; j < n_kv && !*abort_flag; ++j) {
        const int sl = j & 1;
        if (!mbar_wait(&kv_empty[sl], ((j >> 1) & 1) ^ 1, args.err, kErrAttnProducer)) { *abort_flag = 1; break; }
        mbar_expect_tx(&kv_full[sl], L::SLOT);
        uint8_t* dst = sKV + sl * L::SLOT;
        for (int db = 0; db < L::DB; ++db) {
          tma_load_3d(&tmK, &kv_full[sl], dst + db * L::BOX, db * 64, h, krow0 + j * kT);
          tma_load_3d(&tmV, &kv_full[sl], dst + L::TILE + db * L::BOX, db * 64, h, krow0 + j * kT);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_T = idesc_bf16(128, kT);
      constexpr uint32_t ID_G = idesc_bf16(128, D, /*b_mn_major=*/true);
      const uint32_t qa = smem_u32(sQ), doa = smem_u32(sDO);
      auto mma_nt = [&](uint32_t d, uint32_t xa, uint32_t ya) {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k / 4) * L::BOX + (k % 4) * 32;
          umma_bf16(d, sdesc_sw128(xa + off, 16, 1024), sdesc_sw128(ya + off, 16, 1024), ID_T, k > 0 ? 1u : 0u);
        }
      };
      auto ka = [&](int j) { return smem_u32(sKV + (j & 1) * L::SLOT); };
      auto va = [&](int j) { return smem_u32(sKV + (j & 1) * L::SLOT + L::TILE); };
      bool ok = n_kv > 0 && mbar_wait(q_full, 0, args.err, kErrAttnMma);
      if (ok) ok = mbar_wait(&kv_full[0], 0, args.err, kErrAttnMma);
      if (ok) {
        tc_fence_after();
        mma_nt(tS, qa, ka(0));
        umma_commit(s_full);
        mma_nt(tDP, doa, va(0));
        umma_commit(dp_full);
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const bool more = j + 1 < n_kv;
        if (more) {
          if (!(ok = mbar_wait(s_cons, j & 1, args.err, kErrAttnMma))) break;
          if (!(ok = mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, args.err, kErrAttnMma))) break;
          tc_fence_after();
          mma_nt(tS, qa, ka(j + 1));                         // S(j+1): S(j) already in registers
          umma_commit(s_full);
        }
        if (!(ok = mbar_wait(ds_full, j & 1, args.err, kErrAttnMma))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kT / 16; ++k)                     // dQ += dS·Kⱼ
          umma_bf16_ts(tDQ, tDP + tmem_pair_col(k), sdesc_sw128(ka(j) + k * 2048, L::BOX, 1024), ID_G,
                       (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(&kv_empty[j & 1]);
        if (more) {
          mma_nt(tDP, doa, va(j + 1));                       // dP(j+1) after dQ(j) read dS(j)
          umma_commit(dp_full);
        }
      }
      if (!ok) *abort_flag = 1;
      if (n_kv > 0) umma_commit(done);
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;                      // query row inside the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float c2 = args.scale * kLog2e;
    const int qrow = q_start + r;
    const bool row_in = qrow < q_seg1;
    const long vi = ((long)b * args.H + h) * args.Nq + (row_in ? qrow : q_seg0);
    const float lse2 = row_in ? args.lse[vi] * kLog2e : 0.f;
    const float dlt = row_in ? args.delta[vi] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int nvk = min(kT, k_seg1 - k_seg0 - j * kT) - half * 64;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, args.err, kErrAttnSoftmax)))) break;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(tS + lane_off + half * 64, sr);
      tmem_ld32(tS + lane_off + half * 64 + 32, sr + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_cons);
      float p[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) p[c] = c < nvk ? ex2(fmaf(__uint_as_float(sr[c]), c2, -lse2)) : 0.f;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(dp_full, j & 1, args.err, kErrAttnSoftmax)))) break;
      tc_fence_after();
      tmem_ld32(tDP + lane_off + half * 64, sr);
      tmem_ld32(tDP + lane_off + half * 64 + 32, sr + 32);
      tmem_ld_wait();
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float g[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = p[8 * c8 + e] * (__uint_as_float(sr[8 * c8 + e]) - dlt);
        tmem_st4(tDP + lane_off + half * 64 + c8 * 4, pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]),
                 pack_bf16x2(g[4], g[5]), pack_bf16x2(g[6], g[7]));
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (!ok) *abort_flag = 1;
    if (n_kv > 0) {
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(done, 0, args.err, kErrAttnTeardown)))) *abort_flag = 1;
      tc_fence_after();
    }
    const bool valid = ok && row_in;
    const long orow = (((long)b * args.Nq + qrow) * args.H + h) * D;
#pragma unroll 1
    for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
      uint32_t a[32];
      if (n_kv > 0) {
        tmem_ld32(tDQ + lane_off + c, a);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) a[e] = 0u;
      }
      if (valid) store_row32_bf16(args.dq + orow + c, a, args.scale);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------- host
template <typename K>
static void set_smem(K kernel, int bytes) {
  smem_opt_in(reinterpret_cast<const void*>(kernel), bytes);
}

void attention_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                   const at::Tensor& dout, const at::Tensor& lse, const at::Tensor& seg_q, const at::Tensor& seg_k,
                   at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, at::Tensor& delta, double scale, int64_t max_q,
                   int64_t max_k) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && o.is_cuda() && dout.is_cuda(), "attention_bwd: CUDA");
  for (const at::Tensor* t : {&q, &k, &v, &o, &dout})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4, "attention_bwd: bf16 [B, N, H, D] inputs");
  const int D = (int)q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "attention_bwd: head_dim 64 or 128");
  const int B = (int)q.size(0), Nq = (int)q.size(1), H = (int)q.size(2), Nk = (int)k.size(1);
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == B && k.size(2) == H && k.size(3) == D, "attention_bwd: k/v");
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous() && o.sizes() == q.sizes() && dout.sizes() == q.sizes(),
              "attention_bwd: contiguous o / dO shaped like q");
  TORCH_CHECK(dq.is_contiguous() && dq.scalar_type() == at::kBFloat16 && dq.sizes() == q.sizes(), "attention_bwd: dq");
  TORCH_CHECK(dk.is_contiguous() && dk.scalar_type() == at::kBFloat16 && dk.sizes() == k.sizes(), "attention_bwd: dk");
  TORCH_CHECK(dv.is_contiguous() && dv.scalar_type() == at::kBFloat16 && dv.sizes() == k.sizes(), "attention_bwd: dv");
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat && lse.numel() == (int64_t)B * H * Nq,
              "attention_bwd: fp32 lse [B, H, Nq]");
  TORCH_CHECK(delta.is_contiguous() && delta.scalar_type() == at::kFloat && delta.numel() == (int64_t)B * H * Nq,
              "attention_bwd: fp32 delta scratch [B, H, Nq]");
  TORCH_CHECK(seg_q.is_cuda() && seg_k.is_cuda() && seg_q.scalar_type() == at::kInt &&
              seg_k.scalar_type() == at::kInt && seg_q.numel() == seg_k.numel(), "attention_bwd: int32 segments");
  c10::cuda::CUDAGuard guard(q.device());
  const int nseg = (int)seg_q.numel() - 1;
  if (nseg <= 0 || B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const long rows = (long)B * Nq * H;
  if (rows > 0) {
    const int wpb = 8;
    const unsigned blocks = (unsigned)((rows + wpb - 1) / wpb);
    const auto* op = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
    const auto* gp = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
    if (D == 128) attn_bwd_delta_kernel<128><<<blocks, wpb * 32, 0, stream>>>(op, gp, delta.data_ptr<float>(), B, Nq, H);
    else attn_bwd_delta_kernel<64><<<blocks, wpb * 32, 0, stream>>>(op, gp, delta.data_ptr<float>(), B, Nq, H);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  CUtensorMap tq = attn_tmap(q, D), tk = attn_tmap(k, D), tv = attn_tmap(v, D), tdo = attn_tmap(dout, D);
  AttnBwdArgs a;
  a.seg_q = seg_q.data_ptr<int>();
  a.seg_k = seg_k.data_ptr<int>();
  a.Nq = Nq;
  a.Nk = Nk;
  a.H = H;
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  a.scale = (float)scale;
  a.err = error_word(q.get_device());
  if (max_k > 0) {
    dim3 grid((unsigned)((max_k + bwd::kT - 1) / bwd::kT), (unsigned)nseg, (unsigned)(B * H));
    if (D == 128) {
      set_smem(attn_bwd_dkdv_kernel<128>, DkdvSmem<128>::BYTES);
      attn_bwd_dkdv_kernel<128><<<grid, bwd::kThreads, DkdvSmem<128>::BYTES, stream>>>(tq, tk, tv, tdo, a);
    } else {
      set_smem(attn_bwd_dkdv_kernel<64>, DkdvSmem<64>::BYTES);
      attn_bwd_dkdv_kernel<64><<<grid, bwd::kThreads, DkdvSmem<64>::BYTES, stream>>>(tq, tk, tv, tdo, a);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (max_q > 0) {
    dim3 grid((unsigned)((max_q + bwd::kT - 1) / bwd::kT), (unsigned)nseg, (unsigned)(B * H));
    if (D == 128) {
      set_smem(attn_bwd_dq_kernel<128>, DqSmem<128>::BYTES);
      attn_bwd_dq_kernel<128><<<grid, bwd::kThreads, DqSmem<128>::BYTES, stream>>>(tq, tk, tv, tdo, a);
    } else {
      set_smem(attn_bwd_dq_kernel<64>, DqSmem<64>::BYTES);
      attn_bwd_dq_kernel<64><<<grid, bwd::kThreads, DqSmem<64>::BYTES, stream>>>(tq, tk, tv, tdo, a);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace osp
