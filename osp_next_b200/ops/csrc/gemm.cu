// Persistent warp-specialised tcgen05 GEMM for sm_100a:  D[M,N] = A[M,K] · B[N,K]ᵀ
// (nn.Linear layout: activations and weights both K-major, bf16), fp32 accumulation
// in TMEM, fused epilogues.
//
// Reference hot ops this replaces (all cuBLAS + eager elementwise there):
//   q/k/v/o, cross-attn, FFN linears of OSPNextAttentionBlock
//   (ospnext/modules/osp_next.py:742-777, 873-877, 926-957), text/patch
//   embeddings and the head (osp_next.py:1092-1104, 1249-1252, want2v.py:262-287).
//
// Structure (one CTA per SM, 320 threads):
//   warp 0      TMA producer: A/B k-blocks into a STAGES-deep smem ring (128B swizzle)
//   warp 1      MMA issuer:  tcgen05.mma 128×BN×16 per step into one of two TMEM
//               accumulators (so the epilogue of tile i overlaps the MMAs of tile i+1)
//   warps 2..9  epilogue:    two groups of four warps (one per TMEM lane quarter), each
//               taking half of the tile's columns: tcgen05.ld 32 columns at a time, bias /
//               GELU-tanh / gated fp32 residual (+ row remap = fused layout change), global
//               store.  Two groups double the global loads in flight, which the residual
//               epilogue (a streaming fp32 read-modify-write) needs to keep up with the MMAs.
// Tiles are visited in M-groups of 16 so the weight stays L2-resident across a group.
// Optionally a second operand pair (A2 [M,K2], B2 [N,K2]) is streamed after the first into
// the same accumulator: D = A·Bᵀ + A2·B2ᵀ.  With A2 = x·Loraᵀ_A and B2 = s·Lora_B this is a
// LoRA-adapted Linear in one GEMM, keeping every epilogue (bias, GELU, gated residual,
// fused layout store) of the plain Linear.
// Either operand may instead be MN-major (stored [K, M] / [K, N], MN contiguous): the
// backward GEMMs dX = dY·W and dW = dYᵀ·X read dY, W and X in place, with no transposed
// copies.  An MN-major tile is MN/64 TMA boxes of 64 K-rows × 64 elements (128B swizzle).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

namespace osp {

constexpr int kBM = 128;
constexpr int kBK = 64;              // 64 bf16 = 128 B rows (one swizzle span)
constexpr int kGroupM = 16;
constexpr int kSmemBudget = 196608;  // 192 KiB of operand ring
constexpr int kGemmThreads = 320;
constexpr int kStageRow = 80;                 // bytes per staged row (64 B of bf16 + 16 B pad)
constexpr int kStageBytes = 32 * kStageRow;   // one epilogue warp's 32 × 32 staging tile

enum EpiMode : int { kEpiStore = 0, kEpiResidual = 1 };

struct GemmArgs {
  int M, N, K;
  const float* bias;        // [N] or null
  int act;                  // 0 none, 1 gelu_tanh
  void* out;                // [M or B*n_out, N] (bf16 or f32)
  const float* resid;       // [M, N] f32 (residual mode)
  const float* gate;        // [B, N] f32 or null (residual mode)
  const int* dest_row;      // [rows_per_batch] or null
  int rows_per_batch;       // n (residual mode)
  int n_out;                // rows per batch of out (residual mode with dest_row)
  const int64_t* out_ptrs;  // [world] peer output buffers (fused SSP exchange) or null
  const int* dest_rank;     // [rows_per_batch] owner rank of each row in the next layout
  __nv_bfloat16* aux;       // [M, N] bf16 pre-activation (store mode with GELU, training) or null
  int K2;                   // K of the second operand pair (0: none)
  int* err;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f;   // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

template <int BN, int MODE, typename OutT, bool A_MN = false, bool B_MN = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, GemmArgs args) {
  constexpr int STAGES = kSmemBudget / (kBM * kBK * 2 + BN * kBK * 2);
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t B_BYTES = BN * kBK * 2;
  constexpr uint32_t MN_BOX = 64 * kBK * 2;        // one MN-major box: 64 K-rows × 128 B
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16(kBM, BN, B_MN, A_MN);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // residual epilogue: per-warp staging of 32 rows × 32 bf16 (row stride 80 B, conflict-free)
  uint8_t* epi_stage = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(abort_flag + 1) + 127) & ~uintptr_t(127));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (args.M + kBM - 1) / kBM;
  const int num_n = (args.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb1 = (args.K + kBK - 1) / kBK;                 // k-blocks of the first pair
  const int num_kb = num_kb1 + (args.K2 + kBK - 1) / kBK;       // ... and of both

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 8); }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (args.K2 > 0) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrGemmProducer)) { *abort_flag = 1; break; }
          mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          const bool second = kb >= num_kb1;
          const CUtensorMap* ta = second ? &tmA2 : &tmA;
          const CUtensorMap* tb = second ? &tmB2 : &tmB;
          const int kc = (second ? kb - num_kb1 : kb) * kBK;   // K coordinate within the pair
          if constexpr (A_MN) {
#pragma unroll
            for (int c = 0; c < kBM / 64; ++c)
              tma_load_2d(ta, &full[stage], sA + stage * A_BYTES + c * MN_BOX, mb * kBM + 64 * c, kc);
          } else {
            tma_load_2d(ta, &full[stage], sA + stage * A_BYTES, kc, mb * kBM);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(tb, &full[stage], sB + stage * B_BYTES + c * MN_BOX, nb * BN + 64 * c, kc);
          } else {
            tma_load_2d(tb, &full[stage], sB + stage * B_BYTES, kc, nb * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.err, kErrGemmMma)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrGemmMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // K-major: +32 B per 16-wide K step; MN-major: +16 rows × 128 B, boxes MN_BOX apart
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + k * 2048, MN_BOX, 1024)
                                     : sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + k * 2048, MN_BOX, 1024)
                                     : sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&tfull[acc]);
        if (!ok) { *abort_flag = 1; break; }
      }
      // all MMAs issued by this thread done before teardown
      umma_commit(done);
      mbar_wait(done, 0, args.err, kErrGemmTeardown);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    const int quarter = warp & 3;               // TMEM lanes 32·quarter .. +31
    const int eg = (warp - 2) >> 2;             // column half of the tile
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      if (*abort_flag) break;
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, args.err, kErrGemmEpilogue))) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mb * kBM + quarter * 32 + lane;
      const bool row_ok = row < args.M;
      long out_row = row;
      int bidx = 0;
      float* out_base = reinterpret_cast<float*>(args.out);
      if (MODE == kEpiResidual && row_ok) {
        bidx = row / args.rows_per_batch;
        if (args.dest_row) {
          const int m = row - bidx * args.rows_per_batch;
          out_row = (long)bidx * args.n_out + args.dest_row[m];
          // fused SSP exchange: the row is stored into the owner's buffer over NVLink
          if (args.out_ptrs) out_base = reinterpret_cast<float*>(args.out_ptrs[args.dest_rank[m]]);
        }
      }
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      // residual mode writes rows cooperatively (8 lanes × 16 B = one 128-B row segment):
      // lane group `sub` handles rows sub, sub+4, …, so gather those rows' destinations once
      const int sub = lane >> 3, c4 = lane & 7;
      long t_orow[8];
      float* t_obase[8];
      int t_bidx[8];
      bool t_ok[8];
      if (MODE == kEpiResidual) {
        const unsigned long long ob = reinterpret_cast<unsigned long long>(out_base);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int src = i * 4 + sub;
          t_orow[i] = __shfl_sync(0xffffffffu, out_row, src);
          t_obase[i] = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, ob, src));
          t_bidx[i] = __shfl_sync(0xffffffffu, bidx, src);
          t_ok[i] = __shfl_sync(0xffffffffu, row_ok, src);
        }
      }
      uint8_t* stg = epi_stage + (warp - 2) * kStageBytes;
#pragma unroll 1
      for (int c = eg * (BN / 64); c < (eg + 1) * (BN / 64); ++c) {
        const int col0 = nb * BN + c * 32;
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait();
        if (col0 >= args.N) continue;                       // uniform across the warp
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (args.bias) {
          const float4* b4 = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 b = __ldg(b4 + j);
            v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
          }
        }
        if (MODE == kEpiStore) {
          if (args.aux && row_ok) {    // pre-activation kept for the GELU backward
            uint4* a4 = reinterpret_cast<uint4*>(args.aux + out_row * args.N + col0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 w;
              w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
              w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
              w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
              w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
              a4[j] = w;
            }
          }
          if (args.act == 1) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_tanh_f(v[j]);
          }
          // bf16: stage the warp's 32 rows × 32 outputs in smem, then write each row's 64 B
          // as one contiguous segment (4 lanes × 16 B) instead of 32 scattered 16-B stores
          if constexpr (sizeof(OutT) == 2) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 w;
              w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
              w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
              w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
              w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
              *reinterpret_cast<uint4*>(stg + lane * kStageRow + j * 16) = w;
            }
            __syncwarp();
            const int q = lane >> 2, cc = lane & 3;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rr = i * 8 + q;
              const long grow = (long)mb * kBM + quarter * 32 + rr;
              if (grow < args.M)
                *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(args.out) + grow * args.N + col0 + cc * 8) =
                    *reinterpret_cast<const uint4*>(stg + rr * kStageRow + cc * 16);
            }
            __syncwarp();
          } else if (row_ok) {
            // fp32 (weight gradients): each thread's 128-B row chunk is already a full line
            float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + out_row * args.N + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
        } else {
          // resid + bf16(y)·gate (the Linear output is bf16 under autocast in the reference).
          // bf16(y) goes through smem so that each row is then read, combined and written by
          // 8 lanes as one contiguous 128-B segment: full-line residual reads and, for the
          // fused SSP exchange, 128-B writes over NVLink instead of 32 scattered 16-B ones.
          // The residual stream is touched once: streaming (evict-first) accesses.
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 w;
            w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(stg + lane * kStageRow + j * 16) = w;
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (!t_ok[i]) continue;
            const int rr = i * 4 + sub;
            const long grow = (long)mb * kBM + quarter * 32 + rr;
            const uint2 yy = *reinterpret_cast<const uint2*>(stg + rr * kStageRow + c4 * 8);
            const float2 y01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yy.x));
            const float2 y23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&yy.y));
            float4 x = __ldcs(reinterpret_cast<const float4*>(args.resid + grow * args.N + col0) + c4);
            const float4 g = args.gate ? __ldg(reinterpret_cast<const float4*>(args.gate + (long)t_bidx[i] * args.N +
                                                                               col0) + c4)
                                       : make_float4(1.f, 1.f, 1.f, 1.f);
            x.x += y01.x * g.x;
            x.y += y01.y * g.y;
            x.z += y23.x * g.z;
            x.w += y23.y * g.w;
            __stcs(reinterpret_cast<float4*>(t_obase[i] + t_orow[i] * args.N + col0) + c4, x);
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int BN>
constexpr int gemm_smem_bytes() {
  constexpr int STAGES = kSmemBudget / (kBM * kBK * 2 + BN * kBK * 2);
  return 1024 + STAGES * (kBM * kBK * 2 + BN * kBK * 2) + (2 * STAGES + 5) * 8 + 16 + 128 + 8 * kStageBytes;
}

template <int BN, int MODE, typename OutT, bool A_MN = false, bool B_MN = false>
static void launch_gemm(const at::Tensor& a, const at::Tensor& b, GemmArgs& args, cudaStream_t stream,
                        const at::Tensor* a2 = nullptr, const at::Tensor* b2 = nullptr) {
  // K-major operand: rows of K elements (box 64 K × tile rows); MN-major: rows of M/N
  // elements, one row per K index (box 64 MN × 64 K)
  auto map_a = [&](const at::Tensor& t, int K) {
    return A_MN ? make_tmap_2d_bf16(t.data_ptr(), args.M, K, t.stride(0), 64, kBK)
                : make_tmap_2d_bf16(t.data_ptr(), K, args.M, t.stride(0), kBK, kBM);
  };
  auto map_b = [&](const at::Tensor& t, int K) {
    return B_MN ? make_tmap_2d_bf16(t.data_ptr(), args.N, K, t.stride(0), 64, kBK)
                : make_tmap_2d_bf16(t.data_ptr(), K, args.N, t.stride(0), kBK, BN);
  };
  CUtensorMap tmA = map_a(a, args.K), tmB = map_b(b, args.K);
  const bool dual = a2 != nullptr && args.K2 > 0;
  CUtensorMap tmA2 = dual ? map_a(*a2, args.K2) : tmA;
  CUtensorMap tmB2 = dual ? map_b(*b2, args.K2) : tmB;
  if (!dual) args.K2 = 0;
  auto kern = gemm_kernel<BN, MODE, OutT, A_MN, B_MN>;
  constexpr int smem = gemm_smem_bytes<BN>();
  smem_opt_in(reinterpret_cast<const void*>(kern), smem);
  const int tiles = ((args.M + kBM - 1) / kBM) * ((args.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, num_sms(a.get_device())));
  kern<<<grid, kGemmThreads, smem, stream>>>(tmA, tmB, tmA2, tmB2, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out = act(a·bᵀ [+ a2·b2ᵀ] + bias)  or  out[remap] = resid + (a·bᵀ [+ a2·b2ᵀ] + bias)·gate
static void gemm_impl(const at::Tensor& a, const at::Tensor& b, const at::Tensor* a2, const at::Tensor* b2,
                      const c10::optional<at::Tensor>& bias, at::Tensor& out, int64_t act,
                      const c10::optional<at::Tensor>& resid, const c10::optional<at::Tensor>& gate,
                      const c10::optional<at::Tensor>& dest_row, int64_t rows_per_batch, int64_t n_out) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm: a [M,K], b [N,K]");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm: operands must be K-contiguous");
  TORCH_CHECK(a.size(1) % 8 == 0, "gemm: K must be a multiple of 8 (16-byte TMA rows)");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm: row strides 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0, "gemm: 16-byte aligned operands");
  TORCH_CHECK(b.size(0) % 32 == 0, "gemm: N must be a multiple of 32");
  TORCH_CHECK(out.is_contiguous(), "gemm: contiguous output");
  if (a2 != nullptr) {
    TORCH_CHECK(b2 != nullptr && a2->is_cuda() && b2->is_cuda() && a2->scalar_type() == at::kBFloat16 &&
                b2->scalar_type() == at::kBFloat16 && a2->dim() == 2 && b2->dim() == 2 &&
                a2->size(0) == a.size(0) && b2->size(0) == b.size(0) && a2->size(1) == b2->size(1),
                "gemm_dual: a2 [M,K2], b2 [N,K2] bf16");
    TORCH_CHECK(a2->stride(1) == 1 && b2->stride(1) == 1 && a2->size(1) % 8 == 0 &&
                (a2->stride(0) * 2) % 16 == 0 && (b2->stride(0) * 2) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(a2->data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(b2->data_ptr()) % 16 == 0,
                "gemm_dual: K2-contiguous, K2 % 8 == 0, 16-byte aligned rows");
  }
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.M = (int)a.size(0);
  args.N = (int)b.size(0);
  args.K = (int)a.size(1);
  args.K2 = a2 != nullptr ? (int)a2->size(1) : 0;
  args.bias = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->is_contiguous() && bias->numel() == args.N,
                "gemm: bias f32 [N]");
    args.bias = bias->data_ptr<float>();
  }
  args.act = (int)act;
  args.out = out.data_ptr();
  args.err = error_word(a.get_device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (args.M == 0) return;
  if (resid.has_value()) {
    TORCH_CHECK(out.scalar_type() == at::kFloat && resid->scalar_type() == at::kFloat && resid->is_contiguous(),
                "gemm: residual mode is fp32");
    TORCH_CHECK(resid->numel() == (int64_t)args.M * args.N, "gemm: resid [M,N]");
    args.resid = resid->data_ptr<float>();
    args.gate = nullptr;
    args.rows_per_batch = (int)rows_per_batch;
    TORCH_CHECK(rows_per_batch > 0 && args.M % rows_per_batch == 0, "gemm: M = B·rows_per_batch");
    if (gate.has_value()) {
      TORCH_CHECK(gate->scalar_type() == at::kFloat && gate->is_contiguous() &&
                  gate->numel() == (int64_t)(args.M / rows_per_batch) * args.N, "gemm: gate f32 [B,N]");
      args.gate = gate->data_ptr<float>();
    }
    args.dest_row = nullptr;
    args.n_out = (int)n_out;
    if (dest_row.has_value()) {
      TORCH_CHECK(dest_row->scalar_type() == at::kInt && dest_row->numel() == rows_per_batch,
                  "gemm: dest_row int32 [n]");
      TORCH_CHECK(out.numel() == (int64_t)(args.M / rows_per_batch) * n_out * args.N, "gemm: out [B,n_out,N]");
      args.dest_row = dest_row->data_ptr<int>();
    } else {
      TORCH_CHECK(out.numel() == (int64_t)args.M * args.N, "gemm: out [M,N]");
    }
    if (args.N % 256 == 0) launch_gemm<256, kEpiResidual, float>(a, b, args, stream, a2, b2);
    else if (args.N % 128 == 0) launch_gemm<128, kEpiResidual, float>(a, b, args, stream, a2, b2);
    else launch_gemm<64, kEpiResidual, float>(a, b, args, stream, a2, b2);
    return;
  }
  TORCH_CHECK(out.numel() == (int64_t)args.M * args.N, "gemm: out [M,N]");
  if (out.scalar_type() == at::kBFloat16) {
    if (args.N % 256 == 0) launch_gemm<256, kEpiStore, __nv_bfloat16>(a, b, args, stream, a2, b2);
    else if (args.N % 128 == 0) launch_gemm<128, kEpiStore, __nv_bfloat16>(a, b, args, stream, a2, b2);
    else launch_gemm<64, kEpiStore, __nv_bfloat16>(a, b, args, stream, a2, b2);
  } else {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "gemm: out bf16 or f32");
    if (args.N % 256 == 0) launch_gemm<256, kEpiStore, float>(a, b, args, stream, a2, b2);
    else if (args.N % 128 == 0) launch_gemm<128, kEpiStore, float>(a, b, args, stream, a2, b2);
    else launch_gemm<64, kEpiStore, float>(a, b, args, stream, a2, b2);
  }
}

void gemm(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias, at::Tensor& out,
          int64_t act, const c10::optional<at::Tensor>& resid, const c10::optional<at::Tensor>& gate,
          const c10::optional<at::Tensor>& dest_row, int64_t rows_per_batch, int64_t n_out) {
  gemm_impl(a, b, nullptr, nullptr, bias, out, act, resid, gate, dest_row, rows_per_batch, n_out);
}

// D = a·bᵀ + a2·b2ᵀ with the epilogues of gemm() (LoRA folded into the base GEMM).
void gemm_dual(const at::Tensor& a, const at::Tensor& b, const at::Tensor& a2, const at::Tensor& b2,
               const c10::optional<at::Tensor>& bias, at::Tensor& out, int64_t act,
               const c10::optional<at::Tensor>& resid, const c10::optional<at::Tensor>& gate,
               const c10::optional<at::Tensor>& dest_row, int64_t rows_per_batch, int64_t n_out) {
  gemm_impl(a, b, &a2, &b2, bias, out, act, resid, gate, dest_row, rows_per_batch, n_out);
}

// Training forward of FFN-up: out = gelu_tanh(a·bᵀ + bias) and aux = a·bᵀ + bias (both bf16).
// Optional second operand pair (a2, b2) accumulated into the same GEMM (LoRA FFN-up).
void gemm_gelu_aux(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                   at::Tensor& aux, const c10::optional<at::Tensor>& a2, const c10::optional<at::Tensor>& b2) {
  TORCH_CHECK(aux.is_cuda() && aux.scalar_type() == at::kBFloat16 && aux.is_contiguous() &&
              out.scalar_type() == at::kBFloat16 && aux.sizes() == out.sizes(), "gemm_gelu_aux: bf16 out/aux");
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.dim() == 2 &&
              b.dim() == 2 && a.size(1) == b.size(1) && a.stride(1) == 1 && b.stride(1) == 1 &&
              a.size(1) % 8 == 0 && b.size(0) % 32 == 0 && out.is_contiguous() &&
              out.numel() == a.size(0) * b.size(0), "gemm_gelu_aux: bf16 K-contiguous operands, N % 32, K % 8");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_gelu_aux: row strides 16-byte aligned");
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.M = (int)a.size(0);
  args.N = (int)b.size(0);
  args.K = (int)a.size(1);
  args.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  if (bias.has_value()) TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == args.N, "gemm_gelu_aux: bias");
  args.act = 1;
  args.out = out.data_ptr();
  args.aux = reinterpret_cast<__nv_bfloat16*>(aux.data_ptr());
  args.err = error_word(a.get_device());
  const at::Tensor* pa2 = nullptr;
  const at::Tensor* pb2 = nullptr;
  if (a2.has_value()) {
    TORCH_CHECK(b2.has_value() && a2->scalar_type() == at::kBFloat16 && b2->scalar_type() == at::kBFloat16 &&
                a2->dim() == 2 && b2->dim() == 2 && a2->size(0) == a.size(0) && b2->size(0) == b.size(0) &&
                a2->size(1) == b2->size(1) && a2->stride(1) == 1 && b2->stride(1) == 1 && a2->size(1) % 8 == 0 &&
                (a2->stride(0) * 2) % 16 == 0 && (b2->stride(0) * 2) % 16 == 0,
                "gemm_gelu_aux: second pair a2 [M,K2], b2 [N,K2] bf16, K2 % 8 == 0");
    pa2 = &*a2;
    pb2 = &*b2;
    args.K2 = (int)a2->size(1);
  }
  if (args.M == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (args.N % 256 == 0) launch_gemm<256, kEpiStore, __nv_bfloat16>(a, b, args, stream, pa2, pb2);
  else if (args.N % 128 == 0) launch_gemm<128, kEpiStore, __nv_bfloat16>(a, b, args, stream, pa2, pb2);
  else launch_gemm<64, kEpiStore, __nv_bfloat16>(a, b, args, stream, pa2, pb2);
}

template <bool A_MN, bool B_MN, typename OutT>
static void launch_gemm_t(const at::Tensor& a, const at::Tensor& b, GemmArgs& args, cudaStream_t stream) {
  if (args.N % 256 == 0) launch_gemm<256, kEpiStore, OutT, A_MN, B_MN>(a, b, args, stream);
  else if (args.N % 128 == 0) launch_gemm<128, kEpiStore, OutT, A_MN, B_MN>(a, b, args, stream);
  else launch_gemm<64, kEpiStore, OutT, A_MN, B_MN>(a, b, args, stream);
}

// out[M,N] = A·Bᵀ with A given as a [M,K] (a_mn: stored [K,M]) and B as b [N,K]
// (b_mn: stored [K,N]); the backward-pass GEMMs.  No bias / epilogue op.
void gemm_t(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm_t: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_t: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm_t: 2-D row-major operands");
  const int64_t M = a_mn ? a.size(1) : a.size(0), K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0), Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_t: contraction sizes differ");
  TORCH_CHECK(a.size(1) % 8 == 0 && b.size(1) % 8 == 0, "gemm_t: rows must be a multiple of 8 elements (16 B)");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_t: row strides 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0, "gemm_t: 16-byte aligned operands");
  TORCH_CHECK(N % 32 == 0, "gemm_t: N must be a multiple of 32");
  TORCH_CHECK(out.is_contiguous() && out.numel() == M * N, "gemm_t: contiguous out [M,N]");
  TORCH_CHECK(a_mn || b_mn, "gemm_t: use gemm for two K-major operands");
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.out = out.data_ptr();
  args.err = error_word(a.get_device());
  if (M == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || out.scalar_type() == at::kBFloat16, "gemm_t: out bf16 or f32");
  if (a_mn && b_mn) {
    if (f32) launch_gemm_t<true, true, float>(a, b, args, stream);
    else launch_gemm_t<true, true, __nv_bfloat16>(a, b, args, stream);
  } else if (b_mn) {
    if (f32) launch_gemm_t<false, true, float>(a, b, args, stream);
    else launch_gemm_t<false, true, __nv_bfloat16>(a, b, args, stream);
  } else {
    if (f32) launch_gemm_t<true, false, float>(a, b, args, stream);
    else launch_gemm_t<true, false, __nv_bfloat16>(a, b, args, stream);
  }
}

// Fused SSP exchange: out_ptrs[dest_rank[m]][b·n_stride + dest_row[m]] = resid[b,m] + (a·bᵀ + bias)·gate[b]
void gemm_p2p(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& bias,
              const at::Tensor& resid, const c10::optional<at::Tensor>& gate, const at::Tensor& dest_rank,
              const at::Tensor& dest_row, const at::Tensor& out_ptrs, int64_t rows_per_batch, int64_t n_stride) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 &&
              a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.stride(1) == 1 && b.stride(1) == 1,
              "gemm_p2p: bf16 K-contiguous operands");
  TORCH_CHECK(a.size(1) % 8 == 0 && b.size(0) % 32 == 0, "gemm_p2p: K % 8 == 0, N % 32 == 0");
  TORCH_CHECK(resid.scalar_type() == at::kFloat && resid.is_contiguous(), "gemm_p2p: fp32 residual");
  TORCH_CHECK(dest_rank.scalar_type() == at::kInt && dest_row.scalar_type() == at::kInt &&
              dest_rank.numel() == rows_per_batch && dest_row.numel() == rows_per_batch, "gemm_p2p: int32 maps [n]");
  TORCH_CHECK(out_ptrs.scalar_type() == at::kLong && out_ptrs.is_cuda(), "gemm_p2p: int64 device pointer table");
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.M = (int)a.size(0);
  args.N = (int)b.size(0);
  args.K = (int)a.size(1);
  TORCH_CHECK(resid.numel() == (int64_t)args.M * args.N && args.M % rows_per_batch == 0, "gemm_p2p: shapes");
  args.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  args.act = 0;
  args.out = nullptr;
  args.resid = resid.data_ptr<float>();
  args.gate = gate.has_value() ? gate->data_ptr<float>() : nullptr;
  args.dest_row = dest_row.data_ptr<int>();
  args.dest_rank = dest_rank.data_ptr<int>();
  args.out_ptrs = out_ptrs.data_ptr<int64_t>();
  args.rows_per_batch = (int)rows_per_batch;
  args.n_out = (int)n_stride;
  args.err = error_word(a.get_device());
  if (args.M == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (args.N % 256 == 0) launch_gemm<256, kEpiResidual, float>(a, b, args, stream);
  else if (args.N % 128 == 0) launch_gemm<128, kEpiResidual, float>(a, b, args, stream);
  else launch_gemm<64, kEpiResidual, float>(a, b, args, stream);
}

}  // namespace osp
