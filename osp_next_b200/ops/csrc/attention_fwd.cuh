// Segmented flash-attention forward kernel for sm_100a (tcgen05 + TMEM + TMA), torch-free.
//
// Replaces the reference's FA3 → FA2 → SDPA dispatch for Skiparse self-attention,
// dense self-attention and cross-attention (ospnext/modules/attention.py:460-517,
// osp_next.py:765-771, 782-816).  A *segment* is one Skiparse group (or the whole
// sequence): queries of segment s attend to keys of segment s only, non-causal.
// Segments come from the token layout, so no permuted / padded copy of q, k, v is
// ever made and padded tokens never exist (they are not in any segment).
//
// CTA = 2 query tiles of 128 rows (one head, one segment, one batch entry).
//   warps 0..7    softmax: warps 0-3 tile 0, warps 4-7 tile 1 (thread ↔ query row; warp w
//                 reads TMEM lanes 32·(w mod 4)…): S row from TMEM, online softmax in the
//                 exp2 domain with lazy O rescaling (only when the running max grows by
//                 more than 2^8), P written bf16 back over S in TMEM (tcgen05.st);
//                 epilogue O/l → bf16, LSE
//   warp 8        TMA producer: Q0, Q1 once; then K_j, V_j into a 5-slot ring
//   warp 9        MMA issuer (one thread): S_t = Q_t·K_jᵀ (TMEM, fp32), O_t += P_t·V_j (TMEM, fp32)
// The PV MMA takes P from TMEM (A operand) and V from smem, so P never touches shared
// memory.  The tensor core alternates tile 0 / tile 1 work (PV0, S0', PV1, S1') so each
// softmax overlaps the other tile's MMAs.  TMEM: S0 | S1 | O0 | O1 (512 columns, D = 128).
// With kSplitP the softmax publishes P in two halves (keys 0..63, then 64..127) and the
// first half of the PV MMA starts while the second half is still being exponentiated.
// A share of the exponentials (kPoly mask over 16-key groups) runs on the FMA/ALU pipes
// (exp2_fma2) to offload the MUFU unit.
//
// Every wait is bounded (common.cuh); on timeout the kernel records an error code and
// winds down.  With OSP_ATTN_TRACE defined, a few CTAs record clock64() stamps of each
// pipeline event into g_attn_trace (profiling builds only).
#pragma once
#include "common.cuh"
#include "attn_math.cuh"

namespace osp {

constexpr int kQT = 128;      // rows per query tile
constexpr int kKT = 128;      // keys per KV tile
constexpr int kSlots = 5;     // K/V ring slots

struct AttnArgs {
  const int* seg_q;
  const int* seg_k;
  int Nq, Nk, H;
  __nv_bfloat16* out;       // [B, Nq, H, D]
  float* lse;               // [B, H, Nq] or null
  float scale_log2;         // softmax scale · log2(e)
  int* err;
};

#ifdef OSP_ATTN_TRACE
constexpr int kTrSteps = 48, kTrEv = 8, kTrRoles = 4, kTrCtas = 4;
__device__ unsigned long long* g_attn_trace = nullptr;   // [kTrCtas][kTrRoles][kTrSteps][kTrEv]
__device__ __forceinline__ int attn_trace_cta() {
  return (blockIdx.y == 0 && blockIdx.x < 2 && blockIdx.z < 2) ? (int)(blockIdx.x + 2 * blockIdx.z) : -1;
}
#define ATTN_TR(role, j, ev)                                                                        \
  do {                                                                                              \
    const int _c = attn_trace_cta();                                                                \
    if (_c >= 0 && (j) < kTrSteps && g_attn_trace)                                                  \
      g_attn_trace[((_c * kTrRoles + (role)) * kTrSteps + (j)) * kTrEv + (ev)] = (unsigned long long)clock64(); \
  } while (0)
#else
#define ATTN_TR(role, j, ev) ((void)0)
#endif

template <int D>
struct AttnFwdCfg {
  static_assert(D == 64 || D == 128, "head dim 64 or 128");
  static constexpr int kSoftWarps = 4;                        // per query tile
  static constexpr int kProdWarp = 8;
  static constexpr int kMmaWarp = 9;
  static constexpr int kThreads = 320;                        // 10 warps: 168 registers per thread
  static constexpr int BOX = kQT * 128;                        // one 128-row × 128-byte box (16 KiB)
  static constexpr int DB = D / 64;                            // boxes per row of D
  static constexpr int Q_TILE = DB * BOX;
  static constexpr int KV_SLOT = DB * BOX;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + 2 * Q_TILE;
  static constexpr int OFF_BAR = OFF_KV + kSlots * KV_SLOT;
  static constexpr int USED = OFF_BAR + 256;
  static constexpr int kMaxSmem = 232448;                      // 227 KiB opt-in per CTA
  // room left for aligning the dynamic smem base to 1024 B (SW128 tiles)
  static constexpr int SLACK = (kMaxSmem - USED) < 1008 ? (kMaxSmem - USED) : 1008;
  static constexpr int BYTES = USED + SLACK;
};

// Exponentials of N consecutive S values (fp32 bits in sr, keys k0.. of this half) into
// P = 2^(s·scale·log2e − m) as bf16 pairs stored at TMEM column taddr (2 keys per column).
// Returns the row sum of P.  kFull: all N keys valid; else keys ≥ n_valid give 0.
// kPoly bit (kG0 + g) selects the FMA-pipe exponential for 16-key group g.
template <int N, bool kFull, uint32_t kPoly, int kG0>
__device__ __forceinline__ float attn_exp_store(const uint32_t* sr, float sl2, float m, int n_valid,
                                                uint32_t taddr) {
  const uint64_t sl2x2 = pk2(sl2, sl2), negm2 = pk2(-m, -m);
  uint64_t lsa = pk2(0.f, 0.f), lsb = pk2(0.f, 0.f);
#pragma unroll
  for (int g = 0; g < N / 16; ++g) {
    uint32_t pw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = g * 16 + 2 * i;
      const uint64_t xe = ffma2(pk2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sl2x2, negm2);
      float x0, x1;
      upk2(xe, x0, x1);
      uint64_t e;
      if ((kPoly >> (kG0 + g)) & 1u) e = exp2_fma2(x0, x1);
      else e = pk2(ex2(x0), ex2(x1));
      float e0, e1;
      upk2(e, e0, e1);
      if (!kFull) {
        e0 = c < n_valid ? e0 : 0.f;
        e1 = c + 1 < n_valid ? e1 : 0.f;
        e = pk2(e0, e1);
      }
      if (i & 1) lsb = fadd2(lsb, e);
      else lsa = fadd2(lsa, e);
      pw[i] = pack_bf16x2(e0, e1);
    }
    tmem_st8(taddr + g * 8, pw);   // 16 keys → 8 TMEM columns
  }
  float a, b;
  upk2(fadd2(lsa, lsb), a, b);
  return a + b;
}

// Row max of N S values (raw, unscaled); keys ≥ n_valid ignored unless kFull.
template <int N, bool kFull>
__device__ __forceinline__ float attn_row_max(const uint32_t* sr, int n_valid) {
  if (kFull) {
    float m8[8];                                 // 8 independent chains of 3-input max
#pragma unroll
    for (int q = 0; q < 8; ++q) m8[q] = fmaxf(__uint_as_float(sr[2 * q]), __uint_as_float(sr[2 * q + 1]));
#pragma unroll
    for (int c = 16; c < N; c += 16) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        m8[q] = max3(m8[q], __uint_as_float(sr[c + 2 * q]), __uint_as_float(sr[c + 2 * q + 1]));
    }
    return fmaxf(max3(m8[0], m8[1], m8[2]), max3(max3(m8[3], m8[4], m8[5]), m8[6], m8[7]));
  }
  float mx = -INFINITY;
#pragma unroll
  for (int c = 0; c < N; ++c)
    if (c < n_valid) mx = fmaxf(mx, __uint_as_float(sr[c]));
  return mx;
}

// O_t (this thread's row, TMEM columns [c0, c0 + n)) *= alpha
__device__ __forceinline__ void attn_rescale_o(uint32_t tO, int n, float alpha) {
#pragma unroll 1
  for (int c = 0; c < n; c += 32) {
    uint32_t o[32];
    tmem_ld32(tO + c, o);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st32(tO + c, o);
  }
}

// O row (TMEM columns [0, n) at tO) / l → bf16 at orow.
__device__ __forceinline__ void attn_store_o(uint32_t tO, int n, float inv_l, __nv_bfloat16* orow, bool valid) {
#pragma unroll 1
  for (int c = 0; c < n; c += 32) {
    uint32_t o[32];
    tmem_ld32(tO + c, o);
    tmem_ld_wait();
    if (valid) {
      uint4* o4 = reinterpret_cast<uint4*>(orow + c);
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
}

template <int D, uint32_t kPoly, bool kSplitP>
__global__ void __launch_bounds__(AttnFwdCfg<D>::kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, AttnArgs args) {
  using L = AttnFwdCfg<D>;
  const int qblk = blockIdx.x;
  const int s = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / args.H;
  const int h = bh % args.H;
  const int q_seg0 = args.seg_q[s], q_seg1 = args.seg_q[s + 1];
  const int k_seg0 = args.seg_k[s], k_seg1 = args.seg_k[s + 1];
  const int q_start = q_seg0 + qblk * 2 * kQT;
  if (q_start >= q_seg1 || k_seg1 <= k_seg0) return;          // CTA-uniform early exit
  const int n_keys = k_seg1 - k_seg0;
  const int n_kv = (n_keys + kKT - 1) / kKT;
  const int qrow0 = b * args.Nq + q_start;                     // row in the flattened [B·Nq] map
  const int krow0 = b * args.Nk + k_seg0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad > (uint32_t)L::SLACK) {                              // CTA-uniform: report, do nothing
    if (threadIdx.x == 0) record_error(args.err, kErrAttnLayout);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sKV = smem + L::OFF_KV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                    // [kSlots]
  uint64_t* kv_empty = kv_full + kSlots;           // [kSlots]
  uint64_t* s_full = kv_empty + kSlots;            // [2] S_t(j) complete (and every earlier MMA)
  uint64_t* p_half = s_full + 2;                   // [2] P_t(j) keys 0..63 in TMEM (kSplitP)
  uint64_t* p_full = p_half + 2;                   // [2] P_t(j) complete in TMEM
  uint64_t* o_done = p_full + 2;                   // [2] last PV of tile t complete
  uint64_t* done = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlots; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_half[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == L::kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == L::kProdWarp) {
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
        ATTN_TR(3, j, u & 1);
      }
    }
  } else if (warp == L::kMmaWarp) {
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
      // O_t += P_t·V over keys [16·k0, 16·k1): P_t (bf16, written by the softmax over the
      // first 64 columns of S_t) is the A operand straight from TMEM, 8 columns = 16 keys
      auto issue_pv = [&](int t, int slot, int k0, int k1, bool acc) {
        const uint32_t va = smem_u32(sKV + slot * L::KV_SLOT);
        const uint32_t d = tmem + 256u + (uint32_t)D * t;
        const uint32_t pa = tmem + 128u * t;
#pragma unroll
        for (int k = k0; k < k1; ++k)
          umma_bf16_ts(d, pa + 8u * k, sdesc_sw128(va + k * 2048, L::BOX, 1024), ID_PV, (acc || k > 0) ? 1u : 0u);
      };
      // wait for P_t(j) (in halves with kSplitP) and issue the PV MMAs
      auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        return mbar_wait(bar, parity, args.err, kErrAttnMma);
      };
      auto pv = [&](int t, int j, int sV) -> bool {
        if (kSplitP) {
          if (!wait(&p_half[t], j & 1)) return false;
          tc_fence_after();
          issue_pv(t, sV, 0, kKT / 32, j > 0);
          ATTN_TR(0, j, 4 * t + 0);
        }
        if (!wait(&p_full[t], j & 1)) return false;
        tc_fence_after();
        issue_pv(t, sV, kSplitP ? kKT / 32 : 0, kKT / 16, j > 0);
        ATTN_TR(0, j, 4 * t + 1);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, args.err, kErrAttnMma) && mbar_wait(&kv_full[0], 0, args.err, kErrAttnMma);
      if (ok) {                                    // prologue: S0(0), S1(0)
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
        const bool more = j + 1 < n_kv;
        if (!(ok = wait(&kv_full[sV], (uV / kSlots) & 1))) break;
        if (!(ok = pv(0, j, sV))) break;
        if (!more) umma_commit(&o_done[0]);
        if (more) {
          if (!(ok = wait(&kv_full[sK], (uK / kSlots) & 1))) break;
          tc_fence_after();
          issue_s(0, sK);
          umma_commit(&s_full[0]);
          ATTN_TR(0, j, 2);
        }
        if (!(ok = pv(1, j, sV))) break;
        umma_commit(&kv_empty[sV]);
        if (!more) umma_commit(&o_done[1]);
        if (more) {
          issue_s(1, sK);
          umma_commit(&s_full[1]);
          umma_commit(&kv_empty[sK]);
          ATTN_TR(0, j, 6);
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(done);
      mbar_wait(done, 0, args.err, kErrAttnTeardown);
    }
  } else if (warp < L::kProdWarp) {
    // ------------------------------------------------------------------ softmax
    const int t = warp / 4;                           // query tile of this warp
    const int quarter = warp & 3;                     // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;                // row inside the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + 128u * t + lane_off;   // S_t; P_t over its first 64 columns
    const uint32_t tO = tmem + 256u + (uint32_t)D * t + lane_off;
    const float sl2 = args.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const bool got = mbar_wait(&s_full[t], j & 1, args.err, kErrAttnSoftmax);
      if (!(ok = __all_sync(0xffffffffu, got))) break;
      tc_fence_after();
      if (lane == 0 && quarter == 0) ATTN_TR(1 + t, j, 0);
      const int n_valid = min(kKT, n_keys - j * kKT);
      const bool full_tile = n_valid == kKT;
      uint32_t sr[kKT];
#pragma unroll
      for (int c = 0; c < kKT / 32; ++c) tmem_ld32(tS + c * 32, sr + c * 32);
      tmem_ld_wait();
      if (lane == 0 && quarter == 0) ATTN_TR(1 + t, j, 1);
      float mx = full_tile ? attn_row_max<kKT, true>(sr, n_valid) : attn_row_max<kKT, false>(sr, n_valid);
      if (lane == 0 && quarter == 0) ATTN_TR(1 + t, j, 5);
      mx *= sl2;
      const bool need = mx > m_ref + 8.0f;
      const float m_new = need ? mx : m_ref;
      // O_t is stable here: PV_t(j-1) was issued before S_t(j), whose completion we waited for
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const float alpha = need ? ex2(m_ref - m_new) : 1.0f;
        l *= alpha;
        attn_rescale_o(tO, D, alpha);
      }
      m_ref = m_new;
      if (lane == 0 && quarter == 0) ATTN_TR(1 + t, j, 2);
      if (full_tile) l += attn_exp_store<64, true, kPoly, 0>(sr, sl2, m_ref, 64, tS);
      else l += attn_exp_store<64, false, kPoly, 0>(sr, sl2, m_ref, n_valid, tS);
      if (kSplitP) {
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_half[t]);
      }
      if (lane == 0 && quarter == 0) ATTN_TR(1 + t, j, 3);
      if (full_tile) l += attn_exp_store<64, true, kPoly, 4>(sr + 64, sl2, m_ref, 64, tS + 32);
      else l += attn_exp_store<64, false, kPoly, 4>(sr + 64, sl2, m_ref, n_valid - 64, tS + 32);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      if (lane == 0 && quarter == 0) ATTN_TR(1 + t, j, 4);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], 0, args.err, kErrAttnSoftmax));
    if (!ok) *abort_flag = 1;
    tc_fence_after();
    // epilogue: O / l → bf16, LSE
    const int qrow = q_start + t * kQT + r;            // row inside the batch entry
    const bool valid = ok && qrow < q_seg1;
    const float inv_l = (l > 0.f) ? 1.0f / l : 0.f;
    __nv_bfloat16* orow = args.out + (((long)b * args.Nq + qrow) * args.H + h) * D;
    attn_store_o(tO, D, inv_l, orow, valid);
    if (valid && args.lse)
      args.lse[((long)b * args.H + h) * args.Nq + qrow] = (m_ref + __log2f(l)) * 0.69314718055994531f;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == L::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace osp
