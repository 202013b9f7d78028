// Segmented flash-attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's FA3 → FA2 → SDPA dispatch for Skiparse self-attention,
// dense self-attention and cross-attention (ospnext/modules/attention.py:460-517,
// osp_next.py:765-771, 782-816).  A *segment* is one Skiparse group (or the whole
// sequence): queries of segment s attend to keys of segment s only, non-causal.
// Segments come from the token layout, so no permuted / padded copy of q, k, v is
// ever made and padded tokens never exist (they are not in any segment).
//
// CTA = 2 query tiles of 128 rows (one head, one segment, one batch entry).
//   warp 0       TMA producer: Q0,Q1 once; then K_j, V_j into a 5-slot ring
//   warp 1       MMA issuer:   S_t = Q_t·K_jᵀ (TMEM, fp32), O_t += P_t·V_j (TMEM, fp32)
//   warps 4..7   softmax group 0 (tile 0), warps 8..11 softmax group 1 (tile 1):
//                thread ↔ query row (warp w reads TMEM lanes 32·(w mod 4)…);
//                S row from TMEM, online softmax in the exp2 domain with lazy O
//                rescaling (only when the running max grows by more than 2^8),
//                P written bf16 back into TMEM over S (tcgen05.st); epilogue O/l → bf16, LSE.
// The PV MMA takes P from TMEM (A operand) and V from smem, so P never touches
// shared memory; the 64 KiB this frees deepens the K/V ring to five slots.
// The tensor core alternates tile 0 / tile 1 work so each softmax group overlaps
// the other tile's MMAs.  TMEM: S0 | S1 | O0 | O1 (512 columns for D = 128).
// Softmax: one S row (128 fp32) per thread from four TMEM loads and one wait;
// full KV tiles skip the per-column key mask; 3-input max, packed f32x2 FMA/ADD
// (sm_100a) for the scale/shift, the row sum and the FMA-pipe exponentials.
// A share of the exponentials (OSP_ATTN_POLY_MASK) runs on the FMA/ALU pipes (exp2_fma2).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"
#include "attn_common.cuh"

namespace osp {

constexpr int kQT = 128;      // rows per query tile
constexpr int kKT = 128;      // keys per KV tile
constexpr int kSlots = 5;     // K/V ring slots (the smem freed by keeping P in TMEM)
constexpr int kAttnThreads = 384;

struct AttnArgs {
  const int* seg_q;
  const int* seg_k;
  int Nq, Nk, H;
  __nv_bfloat16* out;       // [B, Nq, H, D]
  float* lse;               // [B, H, Nq] or null
  float scale_log2;         // softmax scale · log2(e)
  int* err;
};

// Which 8-column groups (bit c16 mod 8) take exp2_fma2 instead of MUFU ex2.  Measured at
// the 14B shapes (TFLOP/s, same box): 1 group in 8 → 1062, none → 1056, 2 → 1019,
// 3 → 998; 4 and 5 slower still.  The softmax is issue-bound, and a polynomial
// exponential costs ~5 issue slots where MUFU costs one.
#ifndef OSP_ATTN_POLY_MASK
#define OSP_ATTN_POLY_MASK 0x80
#endif

// Packed f32x2 (1) or scalar (0) scale/shift and row sum: equal speed when measured.
#ifndef OSP_ATTN_PACKED
#define OSP_ATTN_PACKED 1
#endif

// One S row (128 fp32 in registers) → P = 2^(s·scale·log2e − m) as bf16 pairs stored over
// the S columns in TMEM (taddr = this warp's lanes of S_t); returns the row sum of P.
// kFull: all 128 keys valid (no per-column mask in the hot path).
template <bool kFull>
__device__ __forceinline__ float softmax_p_to_tmem(const uint32_t* sr, float sl2, float m, int n_valid,
                                                   uint32_t taddr) {
#if OSP_ATTN_PACKED
  const uint64_t sl2x2 = pk2(sl2, sl2), negm2 = pk2(-m, -m);
  uint64_t ls2 = pk2(0.f, 0.f);
#pragma unroll
  for (int c16 = 0; c16 < kKT / 8; ++c16) {
    uint32_t pw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c16 * 8 + 2 * i;
      const uint64_t xe = ffma2(pk2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sl2x2, negm2);
      float x0, x1;
      upk2(xe, x0, x1);
      uint64_t e;
      if ((OSP_ATTN_POLY_MASK >> (c16 & 7)) & 1) e = exp2_fma2(x0, x1);
      else e = pk2(ex2(x0), ex2(x1));
      float e0, e1;
      upk2(e, e0, e1);
      if (!kFull) {
        e0 = c < n_valid ? e0 : 0.f;
        e1 = c + 1 < n_valid ? e1 : 0.f;
        e = pk2(e0, e1);
      }
      ls2 = fadd2(ls2, e);
      pw[i] = pack_bf16x2(e0, e1);
    }
    tmem_st4(taddr + c16 * 4, pw[0], pw[1], pw[2], pw[3]);   // 8 keys → 4 TMEM columns
  }
  float a, b;
  upk2(ls2, a, b);
  return a + b;
#else
  float ls[4] = {0.f, 0.f, 0.f, 0.f};
  const float negm = -m;
#pragma unroll
  for (int c16 = 0; c16 < kKT / 8; ++c16) {
    uint32_t pw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c16 * 8 + 2 * i;
      const float x0 = fmaf(__uint_as_float(sr[c]), sl2, negm);
      const float x1 = fmaf(__uint_as_float(sr[c + 1]), sl2, negm);
      const bool poly = (OSP_ATTN_POLY_MASK >> (c16 & 7)) & 1;
      float e0 = poly ? exp2_fma(x0) : ex2(x0);
      float e1 = poly ? exp2_fma(x1) : ex2(x1);
      if (!kFull) {
        e0 = c < n_valid ? e0 : 0.f;
        e1 = c + 1 < n_valid ? e1 : 0.f;
      }
      ls[i] += e0 + e1;
      pw[i] = pack_bf16x2(e0, e1);
    }
    tmem_st4(taddr + c16 * 4, pw[0], pw[1], pw[2], pw[3]);
  }
  return (ls[0] + ls[1]) + (ls[2] + ls[3]);
#endif
}

template <int D>
struct AttnSmem {
  static constexpr int BOX = kQT * 128;                 // one 128-row × 128-byte box (16 KiB)
  static constexpr int DB = D / 64;                     // boxes per row of D
  static constexpr int Q_TILE = DB * BOX;
  static constexpr int KV_SLOT = DB * BOX;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + 2 * Q_TILE;
  static constexpr int OFF_BAR = OFF_KV + kSlots * KV_SLOT;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;   // barriers + alignment slack
};

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, AttnArgs args) {
  using L = AttnSmem<D>;
  const int qblk = blockIdx.x;
  const int s = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / args.H;
  const int h = bh % args.H;
  const int q_seg0 = args.seg_q[s], q_seg1 = args.seg_q[s + 1];
  const int k_seg0 = args.seg_k[s], k_seg1 = args.seg_k[s + 1];
  const int q_start = q_seg0 + qblk * 2 * kQT;
  if (q_start >= q_seg1 || k_seg1 <= k_seg0) return;          // CTA-uniform early exit
  const int n_kv = (k_seg1 - k_seg0 + kKT - 1) / kKT;
  const int qrow0 = b * args.Nq + q_start;                     // row in the flattened [B·Nq] map
  const int krow0 = b * args.Nk + k_seg0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sKV = smem + L::OFF_KV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                    // [kSlots]
  uint64_t* kv_empty = kv_full + kSlots;           // [kSlots]
  uint64_t* s_full = kv_empty + kSlots;            // [2]
  uint64_t* p_full = s_full + 2;                   // [2]
  uint64_t* pv_done = p_full + 2;                  // [2]
  uint64_t* done = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlots; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int t = 0; t < 2; ++t) { mbar_init(&s_full[t], 1); mbar_init(&p_full[t], 4); mbar_init(&pv_done[t], 1); }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < 4) {
  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_expect_tx(q_full, 2 * L::Q_TILE);
      for (int t = 0; t < 2; ++t)
        for (int db = 0; db < L::DB; ++db)
          tma_load_3d(&tmQ, q_full, sQ + t * L::Q_TILE + db * L::BOX, db * 64, h, qrow0 + t * kQT);
      for (int u = 0; u < 2 * n_kv && !*abort_flag; ++u) {
        const int slot = u % kSlots;
        const uint32_t ph = (u / kSlots) & 1;
        if (!mbar_wait(&kv_empty[slot], ph ^ 1, args.err, kErrAttnProducer)) { *abort_flag = 1; break; }
        mbar_expect_tx(&kv_full[slot], L::KV_SLOT);
        const CUtensorMap* tm = (u & 1) ? &tmV : &tmK;
        const int j = u >> 1;
        for (int db = 0; db < L::DB; ++db)
          tma_load_3d(tm, &kv_full[slot], sKV + slot * L::KV_SLOT + db * L::BOX, db * 64, h, krow0 + j * kKT);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, kKT);
      constexpr uint32_t ID_PV = idesc_bf16(128, D, /*b_mn_major=*/true);
      auto issue_s = [&](int t, int slot) {
        const uint32_t qa = smem_u32(sQ + t * L::Q_TILE);
        const uint32_t ka = smem_u32(sKV + slot * L::KV_SLOT);
        const uint32_t d = tmem + 128u * t;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k / 4) * L::BOX + (k % 4) * 32;
          umma_bf16(d, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), ID_S, k > 0 ? 1u : 0u);
        }
      };
      // O_t += P_t·V: P_t (bf16, written by the softmax group over the first 64 columns of
      // S_t) is the A operand straight from TMEM, 8 columns = 16 keys per step
      auto issue_pv = [&](int t, int slot, bool acc) {
        const uint32_t va = smem_u32(sKV + slot * L::KV_SLOT);
        const uint32_t d = tmem + 256u + (uint32_t)D * t;
        const uint32_t pa = tmem + 128u * t;
#pragma unroll
        for (int k = 0; k < kKT / 16; ++k)
          umma_bf16_ts(d, pa + 8u * k, sdesc_sw128(va + k * 2048, L::BOX, 1024), ID_PV, (acc || k > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(q_full, 0, args.err, kErrAttnMma);
      // prologue: S0(0), S1(0)
      if (ok) ok = mbar_wait(&kv_full[0], 0, args.err, kErrAttnMma);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        umma_commit(&s_full[0]);
        issue_s(1, 0);
        umma_commit(&s_full[1]);
        umma_commit(&kv_empty[0]);
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int uV = 2 * j + 1, uK = 2 * j + 2;
        const int sV = uV % kSlots, sK = uK % kSlots;
        if (!(ok = mbar_wait(&kv_full[sV], (uV / kSlots) & 1, args.err, kErrAttnMma))) break;
        if (!(ok = mbar_wait(&p_full[0], j & 1, args.err, kErrAttnMma))) break;
        tc_fence_after();
        issue_pv(0, sV, j > 0);
        umma_commit(&pv_done[0]);
        const bool more = j + 1 < n_kv;
        if (more) {
          if (!(ok = mbar_wait(&kv_full[sK], (uK / kSlots) & 1, args.err, kErrAttnMma))) break;
          tc_fence_after();
          issue_s(0, sK);
          umma_commit(&s_full[0]);
        }
        if (!(ok = mbar_wait(&p_full[1], j & 1, args.err, kErrAttnMma))) break;
        tc_fence_after();
        issue_pv(1, sV, j > 0);
        umma_commit(&pv_done[1]);
        umma_commit(&kv_empty[sV]);
        if (more) {
          issue_s(1, sK);
          umma_commit(&s_full[1]);
          umma_commit(&kv_empty[sK]);
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(done);
      mbar_wait(done, 0, args.err, kErrAttnTeardown);
    }
  }
  } else {

    // ------------------------------------------------------------------ softmax groups (warps 4..11)
    const int t = (warp - 4) / 4;                  // query tile of this group
    const int quarter = warp & 3;                  // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;             // row inside the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tSt = tmem + 128u * t;
    const uint32_t tOt = tmem + 256u + (uint32_t)D * t;
    const float sl2 = args.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, args.err, kErrAttnSoftmax)))) break;
      tc_fence_after();
      // S row → registers (four 32-column TMEM loads, one wait)
      const int n_valid = min(kKT, k_seg1 - k_seg0 - j * kKT);
      const bool full_tile = n_valid == kKT;
      uint32_t sr[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c) tmem_ld32(tSt + lane_off + c * 32, sr + c * 32);
      tmem_ld_wait();
      float mx;
      if (full_tile) {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};   // 4 independent chains
#pragma unroll
        for (int c = 0; c < kKT; c += 8) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            m4[q] = max3(m4[q], __uint_as_float(sr[c + 2 * q]), __uint_as_float(sr[c + 2 * q + 1]));
        }
        mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
      } else {
        mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kKT; ++c)
          if (c < n_valid) mx = fmaxf(mx, __uint_as_float(sr[c]));
      }
      mx *= sl2;
      const bool need = mx > m_ref + 8.0f;
      const float m_new = need ? mx : m_ref;
      if (j > 0) {
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (j - 1) & 1, args.err, kErrAttnSoftmax)))) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2(m_ref - m_new) : 1.0f;
          l *= alpha;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tOt + lane_off + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tOt + lane_off + c * 32, o);
          }
          tmem_st_wait();
        }
      }
      m_ref = m_new;
      // P = exp2(s·scale·log2e − m_ref) → bf16 pairs stored into TMEM over S
      const float lsum = full_tile ? softmax_p_to_tmem<true>(sr, sl2, m_ref, n_valid, tSt + lane_off)
                                   : softmax_p_to_tmem<false>(sr, sl2, m_ref, n_valid, tSt + lane_off);
      l += lsum;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (n_kv - 1) & 1, args.err, kErrAttnSoftmax));
    if (!ok) *abort_flag = 1;
    tc_fence_after();
    // epilogue: O / l → bf16, LSE
    const int qrow = q_start + t * kQT + r;            // row inside the batch entry
    const bool valid = ok && qrow < q_seg1;
    const float inv_l = (l > 0.f) ? 1.0f / l : 0.f;
    __nv_bfloat16* orow = args.out + (((long)b * args.Nq + qrow) * args.H + h) * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tOt + lane_off + c * 32, o);
      tmem_ld_wait();
      if (valid) {
        uint4* o4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[8 * i + 0]) * inv_l, __uint_as_float(o[8 * i + 1]) * inv_l);
          w.y = pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv_l, __uint_as_float(o[8 * i + 3]) * inv_l);
          w.z = pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv_l, __uint_as_float(o[8 * i + 5]) * inv_l);
          w.w = pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv_l, __uint_as_float(o[8 * i + 7]) * inv_l);
          o4[i] = w;
        }
      }
    }
    if (valid && args.lse)
      args.lse[((long)b * args.H + h) * args.Nq + qrow] = (m_ref + __log2f(l)) * 0.69314718055994531f;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg_q,
                   const at::Tensor& seg_k, at::Tensor& out, at::Tensor& lse, double scale, int64_t max_q) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "attention: CUDA tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "attention: bf16 q/k/v");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention: [B, N, H, D]");
  const int D = (int)q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim 64 or 128");
  TORCH_CHECK(k.size(3) == D && v.size(3) == D && k.size(2) == q.size(2) && v.size(2) == q.size(2) &&
              k.size(0) == q.size(0) && v.size(0) == q.size(0) && v.size(1) == k.size(1), "attention: shapes");
  TORCH_CHECK(seg_q.scalar_type() == at::kInt && seg_k.scalar_type() == at::kInt && seg_q.numel() == seg_k.numel(),
              "attention: int32 segments of equal count");
  TORCH_CHECK(seg_q.is_cuda() && seg_k.is_cuda(), "attention: segments on the device");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.sizes() == q.sizes(),
              "attention: bf16 contiguous out [B, Nq, H, D]");
  c10::cuda::CUDAGuard guard(q.device());
  const int B = (int)q.size(0), H = (int)q.size(2);
  const int nseg = (int)seg_q.numel() - 1;
  if (nseg <= 0 || max_q <= 0 || B == 0) return;
  CUtensorMap tq = attn_tmap(q, D), tk = attn_tmap(k, D), tv = attn_tmap(v, D);
  AttnArgs a;
  a.seg_q = seg_q.data_ptr<int>();
  a.seg_k = seg_k.data_ptr<int>();
  a.Nq = (int)q.size(1);
  a.Nk = (int)k.size(1);
  a.H = H;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = (lse.defined() && lse.numel() > 0) ? lse.data_ptr<float>() : nullptr;
  if (a.lse) TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == (int64_t)B * H * a.Nq, "attention: lse");
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.err = error_word(q.get_device());
  dim3 grid((unsigned)((max_q + 2 * kQT - 1) / (2 * kQT)), (unsigned)nseg, (unsigned)(B * H));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (D == 128) {
    static bool cfg = false;
    if (!cfg) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          AttnSmem<128>::BYTES));
      cfg = true;
    }
    attn_fwd_kernel<128><<<grid, kAttnThreads, AttnSmem<128>::BYTES, stream>>>(tq, tk, tv, a);
  } else {
    static bool cfg = false;
    if (!cfg) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          AttnSmem<64>::BYTES));
      cfg = true;
    }
    attn_fwd_kernel<64><<<grid, kAttnThreads, AttnSmem<64>::BYTES, stream>>>(tq, tk, tv, a);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace osp
