// Tensor-core scaled GEMMs for sm_100a (tcgen05 + TMA + TMEM).
//
//   D[M, N] = A[M, K] * B[N, K]^T, both operands K-major ("NT"), FP32
//   accumulation in TMEM, output float32 / bfloat16 / float16.
//
// Kinds:
//   kPerTensor : kind::f8f6f4, E4M3/E5M2 codes, epilogue multiplies by the
//                two per-tensor scales (DelayedScaling / Float8CurrentScaling).
//   kMxfp8     : kind::mxf8f6f4.block_scale, UE8M0 scale per 32 K-elements.
//   kNvfp4     : kind::mxf4nvf4.block_scale.scale_vec::4X, packed E2M1 codes,
//                UE4M3 scale per 16 K-elements.
//   kBf16      : kind::f16 with bf16 operands (64 K-elements per stage), no
//                scales: the GEMM of dequantized operands for recipe pairs and
//                orientations without a block-scaled kind.
// Block scales are consumed in the 512-byte "atom" layout the casts write
// (128 rows x 4 scale columns per atom).
//
// One persistent CTA per SM, 10 warps (11 with the scale-factor copier; the
// block-FP8 kernel has its own 12-warp layout, described there):
//   warp 0    TMA producer (operand tiles + scale atoms) into a 4-stage ring
//   warp 1    TMEM owner and MMA warp (the whole warp runs the loop, lane 0 issues)
//   warps 2-9 epilogue: each pulls 128 accumulator columns of 32 rows from
//             TMEM into registers, releases the accumulator, then scales,
//             converts and stores while the next tile's MMAs run.
// Tile 128 x 256 x (128 bytes of K per stage). Tiles are visited in groups of
// 16 M-blocks so the A rows of a group stay in L2 while B streams.
//
// Every wait is bounded (sm100::mbar_wait); on a timeout the kernel records
// BRC_GEMM_STATUS_TIMEOUT, drains its own copies and MMAs, frees TMEM and
// returns.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "breccia_b200.h"
#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace brc {

__device__ uint32_t g_gemm_status = 0;  // sticky: bit 0 = a bounded wait timed out

namespace gemm {

using namespace sm100;

enum Kind { kPerTensor = 0, kMxfp8 = 1, kNvfp4 = 2, kBf16 = 3 };
// Kinds whose scale factors ride in the MMA (atoms staged and copied to TMEM).
template <int KIND>
constexpr bool kScaled = KIND == kMxfp8 || KIND == kNvfp4;



constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BKB = 128;  // K bytes per stage (one 128-byte swizzle row)
constexpr int STAGES = 4;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
// Single-CTA block-scaled GEMMs add one warp that copies the scale atoms
// into TMEM (tcgen05.cp), so the copies are issued beside the MMA warp
// rather than between its MMAs.
constexpr bool kSfCopier = true;
// Only block-scaled kinds have the copier warp: the role dispatch gives every
// warp past the epilogue warps to the copier, so a kind without scale factors
// must not launch one.
template <int KIND>
constexpr int kThreadsG = kThreads + ((kSfCopier && kScaled<KIND>) ? 32 : 0);
constexpr uint32_t A_BYTES = BM * BKB;  // 16 KB
constexpr uint32_t B_BYTES = BN * BKB;  // 32 KB
// Tiles are visited in groups of kGroupM row blocks, row block fastest: the
// CTAs in flight share kGroupM A panels (BM x K) and about 148 / kGroupM B
// panels (BN x K); A is read from DRAM about once and B about num_m / kGroupM
// times (C2, 16384 x 8192 x 8192: 664 MB read per launch). Measured on B200:
// 32 raised the reads to 1.5 GB and slowed the MXFP8 GEMM of 8192 x 28672 x
// 8192 from 1.63 to 2.18 ms; 4 and 8 were 3-15% slower than 16.
constexpr int kGroupM = 16;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_COL = 0;
constexpr uint32_t SF_COL = 256;

template <int KIND>
struct SfCfg {
  // scale atoms per stage: A (128 rows) and B per 128-row half
  static constexpr uint32_t kAtomsK = KIND == kNvfp4 ? 4 : (KIND == kMxfp8 ? 1 : 0);
  static constexpr uint32_t A_SF = 512 * kAtomsK;
  static constexpr uint32_t B_SF = 2 * 512 * kAtomsK;
  static constexpr uint32_t SFA_COLS = 4 * kAtomsK;  // TMEM columns per stage
  static constexpr uint32_t SFB_COLS = 8 * kAtomsK;
};

template <int KIND>
struct Smem {
  static constexpr uint32_t kA = 0;
  static constexpr uint32_t kB = kA + STAGES * A_BYTES;
  static constexpr uint32_t kSfA = kB + STAGES * B_BYTES;
  static constexpr uint32_t kSfB = kSfA + STAGES * SfCfg<KIND>::A_SF;
  static constexpr uint32_t kBar = kSfB + STAGES * SfCfg<KIND>::B_SF;
  // operand ring (full, empty), scale-factor rings (loaded, in TMEM, slot free),
  // accumulator / partial / drain barriers
  static constexpr uint32_t kNumBars = 5 * STAGES + 8;
  static constexpr uint32_t kMisc = kBar + 8 * kNumBars;
  static constexpr uint32_t kTotal = kMisc + 16;
  static constexpr uint32_t kAlloc = kTotal + 1024;  // manual 1024-byte alignment
  static_assert(kAlloc <= 227 * 1024, "stage ring exceeds shared memory");
};

struct Params {
  int M, N, K;           // K in elements
  int num_m, num_n, num_kb;
  const float* a_scale;  // per-tensor scales (kPerTensor)
  const float* b_scale;
  const uint8_t* sfa;    // scale atoms (block-scaled kinds)
  const uint8_t* sfb;
  uint32_t sf_col_tiles;  // atoms per 128-row group along K
  int sfb_row_atoms;      // ceil(N / 128)
  void* d;
  int64_t ldd;
  uint32_t* status;
  // block FP8 (per-K-block promotion): float32 scales
  const float* bsa;       // (M, K/128): one scale per row per 128-K block
  const float* bsb;       // (ceil(N/128), K/128): one scale per 128x128 tile of B
  int bs_ld;              // K / 128
  int group_m;            // row blocks per tile group (tile order)
  // fused activation cast (k_gemm_pair with CAST != 0): A's source tensor,
  // the codes the casters write (tmap_a reads them), the amax they reduce,
  // the cast-unit queue and the per-(256-row block, K chunk) ready counters
  const void* x;
  uint8_t* a_codes;
  uint32_t* amax_bits;
  uint32_t* cast_next;
  uint32_t* cast_ready;
  uint32_t* gemm_group;   // the highest tile group any producer has reached
  int first_rows;         // rows [0, first_rows) were encoded before the launch
  int kchunks;            // ceil(K / kCastChunk)
};

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& mb, int& nb) {
  const int per_group = p.group_m * p.num_n;
  const int g = tile / per_group;
  const int first = g * p.group_m;
  const int gsize = min(p.num_m - first, p.group_m);
  const int r = tile - g * per_group;
  mb = first + r % gsize;
  nb = r / gsize;
}

template <int OUT>
__device__ __forceinline__ void store_row_chunk(void* d, int64_t ldd, int row, int col0,
                                                int N, const float* v, int count) {
  // `count` consecutive columns starting at col0 (count % 8 == 0), clipped at N.
  if constexpr (OUT == BRC_DTYPE_F32) {
    float* out = static_cast<float*>(d) + (int64_t)row * ldd + col0;
#pragma unroll
    for (int c = 0; c < count; c += 4)
      if (col0 + c < N)
        *reinterpret_cast<float4*>(out + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
  } else {
    __half* out = static_cast<__half*>(d) + (int64_t)row * ldd + col0;
#pragma unroll
    for (int c = 0; c < count; c += 8) {
      if (col0 + c < N) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if constexpr (OUT == BRC_DTYPE_BF16) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[c + 2 * i], v[c + 2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
          } else {
            const __half2 h = __floats2half2_rn(v[c + 2 * i], v[c + 2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        *reinterpret_cast<uint4*>(out + c) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

template <int KIND, int AFMT, int BFMT, int OUT>
__global__ void __launch_bounds__(kThreadsG<KIND>, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
           const Params p) {
  using SF = SfCfg<KIND>;
  using L = Smem<KIND>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* drain = tmem_empty + 1;
  uint64_t* sf_full = drain + 1;        // scale factors of a stage are in TMEM
  uint64_t* sf_free = sf_full + STAGES;  // the MMAs reading a stage's TMEM slot are done
  uint64_t* cdrain = sf_free + STAGES;
  uint64_t* sf_loaded = cdrain + 1;     // a stage's scale atoms are in shared memory
  constexpr bool kCopier = kSfCopier && kScaled<KIND>;
  static_assert(5 * STAGES + 4 <= L::kNumBars, "barrier area too small");
  uint32_t* tmem_base_sh = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.num_m * p.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, kEpiWarps);
    mbar_init(drain, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sf_full[s], 1);
      mbar_init(&sf_free[s], 1);
      mbar_init(&sf_loaded[s], 1);
    }
    mbar_init(cdrain, 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_sh;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;  // per-stage bits for the drain
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, 1u)) {
            ok = false;
            break;
          }
          // The scale atoms go first and complete on their own barrier, so
          // their copies into TMEM can run while the operand tiles are
          // still in flight instead of after them.
          if constexpr (kScaled<KIND>) {
            const bool b_hi = (2 * nb + 1) < p.sfb_row_atoms;
            const uint32_t kcol = (uint32_t)kb * SF::kAtomsK;
            mbar_arrive_expect_tx(&sf_loaded[stage], SF::A_SF + (b_hi ? SF::B_SF : SF::B_SF / 2));
            bulk_load(smem + L::kSfA + stage * SF::A_SF,
                      p.sfa + ((size_t)mb * p.sf_col_tiles + kcol) * 512, SF::A_SF,
                      &sf_loaded[stage]);
            bulk_load(smem + L::kSfB + stage * SF::B_SF,
                      p.sfb + ((size_t)(2 * nb) * p.sf_col_tiles + kcol) * 512, SF::B_SF / 2,
                      &sf_loaded[stage]);
            if (b_hi)
              bulk_load(smem + L::kSfB + stage * SF::B_SF + SF::B_SF / 2,
                        p.sfb + ((size_t)(2 * nb + 1) * p.sf_col_tiles + kcol) * 512,
                        SF::B_SF / 2, &sf_loaded[stage]);
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(smem + L::kA + stage * A_BYTES, &tmap_a, kb * BKB, mb * BM, &full[stage]);
          tma_load_2d(smem + L::kB + stage * B_BYTES, &tmap_b, kb * BKB, nb * BN, &full[stage]);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // wait for this thread's copies in flight before the CTA exits
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(&full[s], (issued_parity >> s) & 1u) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
            while (kScaled<KIND> &&
                   !mbar_try_wait(&sf_loaded[s], (issued_parity >> s) & 1u) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA warp
    // The whole warp runs the loop, so addresses and descriptors stay
    // warp-uniform; lane 0 issues the copies, MMAs and every commit (a commit
    // tracks the tcgen05 operations of the thread that issues it). Run by one
    // lane inside a divergent branch, the loop's per-stage cost made the MMA
    // thread the bound of the block-FP8 GEMM.
    {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem + L::kA), b_base = smem_u32(smem + L::kB);
      const uint64_t dhi = desc_sw128_hi();
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!__all_sync(0xffffffffu, mbar_wait(tmem_empty, acc_phase ^ 1u, abort_flag, p.status, 1u))) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag, p.status, 1u))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t alo = desc_sw128_lo(a_base + stage * A_BYTES);
          const uint32_t blo = desc_sw128_lo(b_base + stage * B_BYTES);
          uint32_t sfa_col = 0, sfb_col = 0;
          if constexpr (kCopier) {
            sfa_col = tmem + SF_COL + stage * SF::SFA_COLS;
            sfb_col = tmem + SF_COL + STAGES * SF::SFA_COLS + stage * SF::SFB_COLS;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&sf_full[stage], phase, abort_flag, p.status, 1u))) {
              ok = false;
              break;
            }
            tc_fence_after();
          } else if constexpr (kScaled<KIND>) {
            sfa_col = tmem + SF_COL + stage * SF::SFA_COLS;
            sfb_col = tmem + SF_COL + STAGES * SF::SFA_COLS + stage * SF::SFB_COLS;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&sf_loaded[stage], phase, abort_flag, p.status, 1u))) {
              ok = false;
              break;
            }
          }
          if (elect_lane()) {
            if constexpr (!kCopier && kScaled<KIND>) {
              const uint32_t sa = smem_u32(smem + L::kSfA + stage * SF::A_SF);
              const uint32_t sb = smem_u32(smem + L::kSfB + stage * SF::B_SF);
#pragma unroll
              for (uint32_t j = 0; j < SF::kAtomsK; ++j) {
                tc_cp_sf(sfa_col + 4 * j, desc_sf_atom(sa + 512 * j));
                tc_cp_sf(sfb_col + 8 * j, desc_sf_atom(sb + 512 * j));
                tc_cp_sf(sfb_col + 8 * j + 4, desc_sf_atom(sb + SF::B_SF / 2 + 512 * j));
              }
            }
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) {
              const uint64_t ad = dhi | (uint64_t)(alo + 2 * k);
              const uint64_t bd = dhi | (uint64_t)(blo + 2 * k);
              const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
              if constexpr (KIND == kPerTensor) {
                mma_f8f6f4(tmem + ACC_COL, ad, bd, idesc_f8f6f4(AFMT, BFMT, BM, BN), acc);
              } else if constexpr (KIND == kBf16) {
                mma_bf16(tmem + ACC_COL, ad, bd, idesc_bf16(BM, BN), acc);
              } else if constexpr (KIND == kMxfp8) {
                mma_mxf8f6f4(tmem + ACC_COL, ad, bd,
                             idesc_block_scaled(AFMT, BFMT, BM, BN, 1u, k, k),
                             sfa_col | (k << 30), sfb_col | (k << 30), acc);
              } else {
                mma_mxf4nvf4_4x(tmem + ACC_COL, ad, bd,
                                idesc_block_scaled(1u, 1u, BM, BN, 0u, 0u, 0u), sfa_col + 4 * k,
                                sfb_col + 8 * k, acc);
              }
            }
            tc_commit(&empty[stage]);
            if constexpr (kCopier) tc_commit(&sf_free[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_lane()) tc_commit(tmem_full);
        __syncwarp();
        acc_phase ^= 1u;
      }
      // every MMA lane 0 issued has completed before TMEM is freed
      if (elect_lane()) {
        tc_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0u) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      __syncwarp();
    }
  } else if (kCopier && warp == 2 + kEpiWarps) {
    // ------------------------------------------------------------ scale-factor copier
    // Copies each stage's scale atoms from shared memory into that stage's
    // TMEM slot once the stage has landed and the MMAs that read the slot
    // last have completed; its commit tells the MMA warp the slot is ready.
    // The whole warp runs the loop; lane 0 issues the copies and commits.
    {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        for (int kb = 0; kb < p.num_kb; ++kb) {
          const bool w = mbar_wait(&sf_loaded[stage], phase, abort_flag, p.status, 1u) &&
                         mbar_wait(&sf_free[stage], phase ^ 1u, abort_flag, p.status, 1u);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_col = tmem + SF_COL + stage * SF::SFA_COLS;
          const uint32_t sfb_col = tmem + SF_COL + STAGES * SF::SFA_COLS + stage * SF::SFB_COLS;
          // atom j of a stage is 512 bytes (32 descriptor address units) after atom 0
          const uint64_t dsa = desc_sf_atom(smem_u32(smem + L::kSfA + stage * SF::A_SF));
          const uint64_t dsb = desc_sf_atom(smem_u32(smem + L::kSfB + stage * SF::B_SF));
          const uint64_t dsb2 = dsb + (SF::B_SF / 2) / 16;
          if (elect_lane()) {
#pragma unroll
            for (uint32_t j = 0; j < SF::kAtomsK; ++j) {
              tc_cp_sf(sfa_col + 4 * j, dsa + 32 * j);
              tc_cp_sf(sfb_col + 8 * j, dsb + 32 * j);
              tc_cp_sf(sfb_col + 8 * j + 4, dsb2 + 32 * j);
            }
            tc_commit(&sf_full[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every copy lane 0 issued has completed before TMEM is freed
      if (elect_lane()) {
        tc_commit(cdrain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(cdrain, 0u) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int half = ew / 4;          // which 128 accumulator columns
    float scale = 1.f;
    if constexpr (KIND == kPerTensor) scale = __fmul_rn(*p.a_scale, *p.b_scale);
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      if (!mbar_wait(tmem_full, acc_phase, abort_flag, p.status, 1u)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      uint32_t r[4][32];
      const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + ACC_COL + 128 * half;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + 32 * c, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_empty);
      const int row = mb * BM + 32 * quad + lane;
      const int col0 = nb * BN + 128 * half;
      if (row < p.M) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = __uint_as_float(r[c][i]);
            if constexpr (KIND == kPerTensor) v[i] = __fmul_rn(v[i], scale);
          }
          store_row_chunk<OUT>(p.d, p.ldd, row, col0 + 32 * c, p.N, v, 32);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ CTA pairs
// GEMMs on CTA pairs (tcgen05 cta_group::2). A cluster of two CTAs on a pair
// of SMs computes a 256 x 256 tile: each CTA loads its 128 rows of A and 128
// rows of B^T (its half of the tile's N) into its own shared memory, so a
// stage is ~32 KB per CTA and the ring is 5-7 deep (the single-CTA kernel
// moves 48 KB per stage through a 4-deep ring). Both CTAs' copies complete
// on the leader's (rank 0's) "full" barrier, lane 0 of the leader's MMA warp
// issues M = 256 MMAs, and their commits reach both CTAs' "empty" and
// accumulator barriers; both CTAs' epilogue warps release the accumulator on
// the leader's barrier. Block-scaled kinds: each CTA also stages the scale
// atoms of its 128 A rows and of all 256 B^T rows; the leader copies them
// into the same TMEM columns of both CTAs (tcgen05.cp cta_group::2), and the
// accumulator is single-buffered so the scale factors fit beside it. A
// cluster barrier brackets set-up and tear-down so no CTA leaves while its
// partner may still signal it.
constexpr int P_BM = 256, P_BN = 256;
constexpr uint32_t P_A_BYTES = 128 * BKB;  // this CTA's 128 rows of A
constexpr uint32_t P_B_BYTES = 128 * BKB;  // this CTA's 128 rows of B^T

template <int KIND>
struct PairCfg {
  using SF = SfCfg<KIND>;
  static constexpr uint32_t kSfa = SF::A_SF;  // scale atoms of this CTA's 128 A rows
  static constexpr uint32_t kSfb = SF::B_SF;  // scale atoms of the tile's 256 B^T rows
  static constexpr uint32_t kStageBytes = P_A_BYTES + P_B_BYTES + kSfa + kSfb;
  static constexpr int kNacc = kScaled<KIND> ? 1 : 2;  // accumulator buffers
  static constexpr int kStages = kScaled<KIND> ? (KIND == kMxfp8 ? 6 : 5) : 7;
  static constexpr uint32_t kA = 0;
  static constexpr uint32_t kB = kA + kStages * P_A_BYTES;
  static constexpr uint32_t kSfA = kB + kStages * P_B_BYTES;
  static constexpr uint32_t kSfB = kSfA + kStages * kSfa;
  static constexpr uint32_t kBar = kSfB + kStages * kSfb;
  // stage ring, accumulator barriers, drain, scale-factor ring (sf_full,
  // sf_free) and the copier's drain
  // (+ one more ring: a stage's scale atoms are in shared memory)
  static constexpr uint32_t kNumBars = 5 * kStages + 2 * kNacc + 2;
  static constexpr uint32_t kMisc = kBar + 8 * kNumBars;
  static constexpr uint32_t kTotal = kMisc + 16;
  static constexpr uint32_t kAlloc = kTotal + 1024;  // manual 1024-byte alignment
  static_assert(kAlloc <= 227 * 1024, "pair ring exceeds shared memory");
  static_assert(kNacc * 256 + (!kScaled<KIND> ? 0
                                              : kStages * (SF::SFA_COLS + SF::SFB_COLS)) <=
                    TMEM_COLS,
                "TMEM overflow");
};

// ------------------------------------------------------------ fused activation cast
// Per-tensor FP8 GEMM whose A operand is cast inside the kernel (template
// argument CAST = 1 + the activation's BRC_DTYPE_*; 0 = no cast). Encoding A in each tile's producer would repeat the
// encode once per N tile (32 times at N = 8192) at about 7 instructions per
// element, more than the issue slots a 256 x 256 x 128 FP8 stage leaves.
// Instead kCastWarps extra warps per CTA encode A once, into the codes
// tensor, in the order the tiles consume it: tile group by tile group (the
// kGroupM row blocks of the tile order), K chunk by K chunk, 32-row slab by
// slab. Units are claimed from a global queue, so no caster waits on anyone
// and every unit is taken by whichever CTA is running. After a slab's codes
// are stored the warp adds one to the ready counter of its (256-row block, K
// chunk); the producer waits (bounded) for a block's full count before its
// first TMA load of that chunk. Rows [0, first_rows) are encoded by a cast
// kernel before the launch, so the first tiles start at once; the rest is
// encoded while the tensor cores work on earlier groups.
// The casters keep at most kCastLead groups ahead of the furthest producer:
// running ahead through the whole tensor at launch, their reads and code
// writes crowded the first groups' operand traffic out of HBM and L2 and
// slowed the GEMM by 6-9%. Held back, their traffic spreads over the GEMM
// and a group's codes are still in L2 when its tiles load them. The hold is
// a bounded pause, not a dependency: a unit a producer waits for is never
// held (a producer publishes its group before it waits).
// Letting the eight epilogue warps also encode while they waited for an
// accumulator was measured slower at every width (C2 0.892 vs 0.809 ms for
// the separate apply pass + GEMM; N = 1024: 0.229 vs 0.169 ms).
constexpr int kCastWarps = 2;
constexpr uint32_t kCastLead = 1;
constexpr uint64_t kCastHoldNs = 20000000ull;  // 20 ms, then cast regardless
constexpr int kCastChunk = 1024;  // K elements (code bytes) per ready counter
constexpr int kCastSlab = 32;     // rows per cast unit
constexpr int kKbPerChunk = kCastChunk / BKB;
static_assert(P_BM % kCastSlab == 0, "a slab must not straddle a row block");
template <int KIND, int CAST>
constexpr int kThreadsP = kThreadsG<KIND> + (CAST != 0 ? 32 * kCastWarps : 0);

// Unit u -> (first row of its slab, K chunk); false past the last unit.
__device__ __forceinline__ bool cast_unit(int u, const Params& p, int& row0, int& kc) {
  const int G = p.group_m * P_BM;
  for (int g0 = (p.first_rows / G) * G; g0 < p.M; g0 += G) {
    const int r0 = max(g0, p.first_rows), r1 = min(g0 + G, p.M);
    const int slabs = (r1 - r0 + kCastSlab - 1) / kCastSlab;
    const int n = slabs * p.kchunks;
    if (u < n) {
      kc = u / slabs;
      row0 = r0 + kCastSlab * (u - kc * slabs);
      return true;
    }
    u -= n;
  }
  return false;
}

// Encode one 16-byte vector of A with the per-tensor scale s (r = RN(1/s)):
// the encoders and division of the per-tensor cast kernels, so the codes are
// theirs bit for bit. A vector holding NaN, or a non-finite scale, takes the
// per-element path (NaN -> the NaN code).
template <int XDT, int FMT>
__device__ __forceinline__ void cast_vector(const uint4 v, float s, float r, bool fast,
                                            float& m, uint8_t* dst) {
  constexpr int V = In<XDT>::kVec;
  const float vmax = vec_absmax<XDT>(v);
  m = fmax_nan(m, vmax);
  float f[V];
  unpack<XDT>(v, f);
  uint32_t w[V / 4];
  if (fast && !isnan(vmax)) {
    // packed-pair forms (same roundings, half the FMA-pipe instructions):
    // these warps share their SM's issue slots with the GEMM's
#pragma unroll
    for (int j = 0; j < V / 4; ++j) {
      float q[4];
      div4(f + 4 * j, s, r, q);
      w[j] = enc4p_fp8<FMT>(q[0], q[1], q[2], q[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < V / 4; ++j) {
      uint32_t c = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) c |= enc1_fp8<FMT>(div_ieee(f[4 * j + i], s)) << (8 * i);
      w[j] = c;
    }
  }
  if constexpr (V == 8) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  else *reinterpret_cast<uint32_t*>(dst) = w[0];
}

// Per-warp state of an encoding warp: the scale, its reciprocal, and the
// amax of everything this warp has read.
struct CastState {
  float s, rcp, m;
  bool fast;
  uint64_t pol;
};
__device__ __forceinline__ CastState cast_state(const Params& p) {
  CastState c;
  c.s = *p.a_scale;
  c.fast = isfinite(c.s) && c.s > 0.f;
  c.rcp = __frcp_rn(c.s);
  c.m = 0.f;
  c.pol = l2_evict_first_policy();  // each input line is read once
  return c;
}

// Encode one 32-row slab of one K chunk (the whole warp) and publish it: the
// codes of every lane, a proxy fence, then one release add on the ready
// counter of the slab's 256-row block.
template <int XDT, int AFMT>
__device__ __forceinline__ void cast_slab(const Params& p, int row0, int kc, int lane,
                                          CastState& c) {
  constexpr int V = In<XDT>::kVec;
  constexpr int PER = kCastChunk / V / 32;  // vectors per lane per row of a chunk
  constexpr int R = 16 / PER;               // rows per batch: 16 loads in flight per lane
  constexpr size_t kEsz = XDT == BRC_DTYPE_F32 ? 4 : 2;
  const char* xb = static_cast<const char*>(p.x);
  const int k0 = kc * kCastChunk;
  const int nv = min(kCastChunk, p.K - k0) / V;
  const int rows = min(kCastSlab, p.M - row0);
  for (int r0 = 0; r0 < rows; r0 += R) {
    uint4 v[R][PER];
#pragma unroll
    for (int h = 0; h < R; ++h)
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int j = lane + 32 * q;
        v[h][q] = make_uint4(0u, 0u, 0u, 0u);
        if (r0 + h < rows && j < nv)
          v[h][q] = ldg16_last_use(
              xb + ((size_t)(row0 + r0 + h) * p.K + k0 + (size_t)j * V) * kEsz, c.pol);
      }
#pragma unroll
    for (int h = 0; h < R; ++h)
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int j = lane + 32 * q;
        if (r0 + h < rows && j < nv)
          cast_vector<XDT, AFMT>(v[h][q], c.s, c.rcp, c.fast, c.m,
                                 p.a_codes + (size_t)(row0 + r0 + h) * p.K + k0 +
                                     (size_t)j * V);
      }
  }
  fence_proxy_async_global();
  __threadfence();
  __syncwarp();
  if (lane == 0) red_release_gpu_add(p.cast_ready + (size_t)(row0 / P_BM) * p.kchunks + kc, 1u);
}

// Group (tile-order group of row blocks) of a cast unit's slab.
__device__ __forceinline__ uint32_t cast_group(const Params& p, int row0) {
  return (uint32_t)(row0 / (p.group_m * P_BM));
}

template <int KIND, int AFMT, int BFMT, int OUT, int CAST = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsP<KIND, CAST>, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmap_a,
                const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_sfa,
                const __grid_constant__ CUtensorMap tmap_sfb, const Params p) {
  using C = PairCfg<KIND>;
  using SF = SfCfg<KIND>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* empty = full + S;
  uint64_t* tmem_full = empty + S;
  uint64_t* tmem_empty = tmem_full + C::kNacc;
  uint64_t* drain = tmem_empty + C::kNacc;
  uint64_t* sf_full = drain + 1;    // (leader) a stage's scale factors are in both CTAs' TMEM
  uint64_t* sf_free = sf_full + S;  // (leader) the MMAs reading a stage's TMEM slot are done
  uint64_t* cdrain = sf_free + S;
  uint64_t* sf_loaded = cdrain + 1;  // (leader) both CTAs' scale atoms of a stage have landed
  constexpr bool kCopier = kSfCopier && kScaled<KIND>;
  uint32_t* tmem_base_sh = reinterpret_cast<uint32_t*>(smem + C::kMisc);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int num_tiles = p.num_m * p.num_n;  // 256 x 256 tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kNacc; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&sf_full[s], 1);
      mbar_init(&sf_free[s], 1);
      mbar_init(&sf_loaded[s], 1);
    }
    mbar_init(cdrain, 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    if constexpr (kScaled<KIND>) {
      prefetch_tmap(&tmap_sfa);
      prefetch_tmap(&tmap_sfb);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_sh, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_base_sh;
  const uint32_t full_leader = mapa_shared(smem_u32(full), 0u);
  const uint32_t sf_loaded_leader = mapa_shared(smem_u32(sf_loaded), 0u);
  const uint32_t tmem_empty_leader = mapa_shared(smem_u32(tmem_empty), 0u);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;  // per-stage bits for the drain
      uint32_t published = 0;                  // 1 + the group last published
      uint64_t ready_lo = 0ull, ready_hi = 0ull;  // row blocks < 128 whose codes are all ready
      auto seen_ready = [&](int mb) {
        return mb < 128 && (((mb < 64 ? ready_lo : ready_hi) >> (mb & 63)) & 1ull);
      };
      bool ok = true;
      for (int tile = cluster; ok && tile < num_tiles; tile += nclusters) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        // scale atoms (2-D copies of 512-byte rows; rows past the operand's
        // end read as zeros): this CTA's 128 A rows and the tile's 256 B^T rows
        const int a_atom = 2 * mb + (int)rank;
        if constexpr (CAST != 0) {
          // publish this tile's group before waiting on any of its codes
          const uint32_t grp = (uint32_t)(mb / p.group_m);
          if (grp + 1 > published) {
            atomicMax(p.gemm_group, grp);
            published = grp + 1;
          }
        }
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, 1u)) {
            ok = false;
            break;
          }
          // The leader expects both CTAs' bytes on its own barriers. The
          // scale atoms go first, on their own barrier, so the copier moves
          // them into TMEM while the operand tiles are still in flight; with
          // one barrier for both, copy latency followed operand latency and
          // the ring (about 1 us deep for MXFP8) no longer hid the sum.
          if constexpr (kScaled<KIND>) {
            if (rank == 0) mbar_arrive_expect_tx(&sf_loaded[stage], 2 * (C::kSfa + C::kSfb));
            const uint32_t sb = sf_loaded_leader + 8u * stage;
            const int kcol = kb * (int)SF::kAtomsK;
            tma_load_2d_pair(smem + C::kSfA + stage * C::kSfa, &tmap_sfa, 0,
                             a_atom * (int)p.sf_col_tiles + kcol, sb);
            tma_load_2d_pair(smem + C::kSfB + stage * C::kSfb, &tmap_sfb, 0,
                             (2 * nb) * (int)p.sf_col_tiles + kcol, sb);
            tma_load_2d_pair(smem + C::kSfB + stage * C::kSfb + C::kSfb / 2, &tmap_sfb, 0,
                             (2 * nb + 1) * (int)p.sf_col_tiles + kcol, sb);
          }
          if constexpr (CAST != 0) {
            // A's codes of this K chunk: cast before the launch, or wait for
            // every slab of this row block (once per row block and producer:
            // a block whose chunks were all seen ready is remembered)
            if (kb % kKbPerChunk == 0 && mb * P_BM >= p.first_rows && !seen_ready(mb)) {
              const uint32_t slabs = (min(P_BM, p.M - mb * P_BM) + kCastSlab - 1) / kCastSlab;
              if (!counter_wait(p.cast_ready + (size_t)mb * p.kchunks + kb / kKbPerChunk, slabs,
                                abort_flag, p.status, 1u)) {
                ok = false;
                break;
              }
              fence_proxy_async_global();
            }
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (P_A_BYTES + P_B_BYTES));
          const uint32_t fb = full_leader + 8u * stage;
          tma_load_2d_pair(smem + C::kA + stage * P_A_BYTES, &tmap_a, kb * BKB,
                           mb * P_BM + 128 * (int)rank, fb);
          tma_load_2d_pair(smem + C::kB + stage * P_B_BYTES, &tmap_b, kb * BKB,
                           nb * P_BN + 128 * (int)rank, fb);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if constexpr (CAST != 0) {
          if (ok && mb < 64) ready_lo |= 1ull << mb;
          else if (ok && mb < 128) ready_hi |= 1ull << (mb - 64);
        }
      }
      if (!ok && rank == 0) {
        // the leader's barriers count both CTAs' copies: wait (bounded) for
        // those in flight before the pair leaves
        for (int s = 0; s < S; ++s)
          if (issued & (1u << s)) {
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(&full[s], (issued_parity >> s) & 1u) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
            while (kScaled<KIND> &&
                   !mbar_try_wait(&sf_loaded[s], (issued_parity >> s) & 1u) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA warp (leader)
    // As in the single-CTA kernel: the whole warp runs the loop with
    // warp-uniform addresses and descriptors; lane 0 issues the copies, MMAs
    // and every commit.
    if (rank == 0) {
      int stage = 0, abuf = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem + C::kA), b_base = smem_u32(smem + C::kB);
      const uint64_t dhi = desc_sw128_hi();
      for (int tile = cluster; ok && tile < num_tiles; tile += nclusters) {
        // accumulator buffer abuf: free once both CTAs' epilogues read it
        if (!__all_sync(0xffffffffu,
                        mbar_wait(&tmem_empty[abuf], acc_phase ^ 1u, abort_flag, p.status, 1u))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tmem + 256u * abuf;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag, p.status, 1u))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t alo = desc_sw128_lo(a_base + stage * P_A_BYTES);
          const uint32_t blo = desc_sw128_lo(b_base + stage * P_B_BYTES);
          uint32_t sfa_col = 0, sfb_col = 0;
          if constexpr (kCopier) {
            sfa_col = tmem + SF_COL + stage * SF::SFA_COLS;
            sfb_col = tmem + SF_COL + S * SF::SFA_COLS + stage * SF::SFB_COLS;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&sf_full[stage], phase, abort_flag, p.status, 1u))) {
              ok = false;
              break;
            }
            tc_fence_after();
          } else if constexpr (kScaled<KIND>) {
            sfa_col = tmem + SF_COL + stage * SF::SFA_COLS;
            sfb_col = tmem + SF_COL + S * SF::SFA_COLS + stage * SF::SFB_COLS;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&sf_loaded[stage], phase, abort_flag, p.status, 1u))) {
              ok = false;
              break;
            }
          }
          if (elect_lane()) {
            if constexpr (!kCopier && kScaled<KIND>) {
              const uint32_t sa = smem_u32(smem + C::kSfA + stage * C::kSfa);
              const uint32_t sb = smem_u32(smem + C::kSfB + stage * C::kSfb);
#pragma unroll
              for (uint32_t j = 0; j < SF::kAtomsK; ++j) {
                tc_cp_sf_pair(sfa_col + 4 * j, desc_sf_atom(sa + 512 * j));
                tc_cp_sf_pair(sfb_col + 8 * j, desc_sf_atom(sb + 512 * j));
                tc_cp_sf_pair(sfb_col + 8 * j + 4, desc_sf_atom(sb + C::kSfb / 2 + 512 * j));
              }
            }
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) {
              const uint64_t ad = dhi | (uint64_t)(alo + 2 * k);
              const uint64_t bd = dhi | (uint64_t)(blo + 2 * k);
              const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
              if constexpr (KIND == kPerTensor) {
                mma_f8f6f4_pair(dacc, ad, bd, idesc_f8f6f4(AFMT, BFMT, P_BM, P_BN), acc);
              } else if constexpr (KIND == kBf16) {
                mma_bf16_pair(dacc, ad, bd, idesc_bf16(P_BM, P_BN), acc);
              } else if constexpr (KIND == kMxfp8) {
                mma_mxf8f6f4_pair(dacc, ad, bd,
                                  idesc_block_scaled(AFMT, BFMT, P_BM, P_BN, 1u, k, k),
                                  sfa_col | (k << 30), sfb_col | (k << 30), acc);
              } else {
                mma_mxf4nvf4_4x_pair(dacc, ad, bd,
                                     idesc_block_scaled(1u, 1u, P_BM, P_BN, 0u, 0u, 0u),
                                     sfa_col + 4 * k, sfb_col + 8 * k, acc);
              }
            }
            tc_commit_pair(&empty[stage], 0x3);
            if constexpr (kCopier) tc_commit_pair(&sf_free[stage], 0x1);
          }
          __syncwarp();
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_lane()) tc_commit_pair(&tmem_full[abuf], 0x3);
        __syncwarp();
        if (++abuf == C::kNacc) {
          abuf = 0;
          acc_phase ^= 1u;
        }
      }
      // every MMA lane 0 issued has completed before the pair frees TMEM
      if (elect_lane()) {
        tc_commit_pair(drain, 0x1);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0u) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      __syncwarp();
    }
  } else if (kCopier && warp == 2 + kEpiWarps) {
    // ------------------------------------------------------------ scale-factor copier (leader)
    // The leader's sf_loaded barrier counts both CTAs' atom copies, so once it
    // completes both CTAs' scale atoms of the stage are in shared memory; each
    // tcgen05.cp cta_group::2 moves every CTA's atoms into its own TMEM.
    // The whole warp runs the loop; lane 0 issues the copies and commits.
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < num_tiles; tile += nclusters) {
        for (int kb = 0; kb < p.num_kb; ++kb) {
          const bool w = mbar_wait(&sf_loaded[stage], phase, abort_flag, p.status, 1u) &&
                         mbar_wait(&sf_free[stage], phase ^ 1u, abort_flag, p.status, 1u);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_col = tmem + SF_COL + stage * SF::SFA_COLS;
          const uint32_t sfb_col = tmem + SF_COL + S * SF::SFA_COLS + stage * SF::SFB_COLS;
          // atom j of a stage is 512 bytes (32 descriptor address units) after atom 0
          const uint64_t dsa = desc_sf_atom(smem_u32(smem + C::kSfA + stage * C::kSfa));
          const uint64_t dsb = desc_sf_atom(smem_u32(smem + C::kSfB + stage * C::kSfb));
          const uint64_t dsb2 = dsb + (C::kSfb / 2) / 16;
          if (elect_lane()) {
#pragma unroll
            for (uint32_t j = 0; j < SF::kAtomsK; ++j) {
              tc_cp_sf_pair(sfa_col + 4 * j, dsa + 32 * j);
              tc_cp_sf_pair(sfb_col + 8 * j, dsb + 32 * j);
              tc_cp_sf_pair(sfb_col + 8 * j + 4, dsb2 + 32 * j);
            }
            tc_commit_pair(&sf_full[stage], 0x1);
          }
          __syncwarp();
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every copy lane 0 issued has completed before the pair frees TMEM
      if (elect_lane()) {
        tc_commit_pair(cdrain, 0x1);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(cdrain, 0u) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      __syncwarp();
    }
  } else if (CAST != 0 && warp >= 2 + kEpiWarps) {
    // ------------------------------------------------------------ activation casters
    if constexpr (CAST != 0) {
      constexpr int XDT = CAST - 1;
      CastState c = cast_state(p);
      while (!*abort_flag) {
        uint32_t u = 0;
        if (lane == 0) u = atomicAdd(p.cast_next, 1u);
        u = __shfl_sync(0xffffffffu, u, 0);
        int row0, kc;
        if (!cast_unit((int)u, p, row0, kc)) break;
        if (lane == 0) {
          const uint32_t grp = cast_group(p, row0);
          if (grp > ld_acquire_gpu(p.gemm_group) + kCastLead) {
            const uint64_t t0 = globaltimer();
            do {
              __nanosleep(2000);
            } while (grp > ld_acquire_gpu(p.gemm_group) + kCastLead && !*abort_flag &&
                     globaltimer() - t0 < kCastHoldNs);
          }
        }
        __syncwarp();
        cast_slab<XDT, AFMT>(p, row0, kc, lane, c);
      }
      float m = c.m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0 && __float_as_uint(m) != 0u) atomicMax(p.amax_bits, __float_as_uint(m));
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = ew / 4;    // which 128 accumulator columns
    float scale = 1.f;
    if constexpr (KIND == kPerTensor) scale = __fmul_rn(*p.a_scale, *p.b_scale);
    uint32_t acc_phase = 0;
    int abuf = 0;
    for (int tile = cluster; tile < num_tiles; tile += nclusters) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      if (!mbar_wait(&tmem_full[abuf], acc_phase, abort_flag, p.status, 1u)) break;
      tc_fence_after();
      uint32_t r[4][32];
      const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + 256u * abuf + 128 * half;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + 32 * c, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tmem_empty_leader + 8u * abuf);
      if (++abuf == C::kNacc) {
        abuf = 0;
        acc_phase ^= 1u;
      }
      const int row = mb * P_BM + 128 * (int)rank + 32 * quad + lane;
      const int col0 = nb * P_BN + 128 * half;
      if (row < p.M) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = __uint_as_float(r[c][i]);
            if constexpr (KIND == kPerTensor) v[i] = __fmul_rn(v[i], scale);
          }
          store_row_chunk<OUT>(p.d, p.ldd, row, col0 + 32 * c, p.N, v, 32);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ block FP8
// DeepSeek-v3 style Float8BlockScaling: A with 1 x 128 float32 scales, B with
// 128 x 128 float32 scales. Float32 (non power of two) scales cannot ride in
// the MMA, so each 128-K block is multiplied into its own TMEM partial (two
// partial buffers of 256 columns) and the epilogue warps promote it into
// float32 register accumulators: acc += P_kb * (sa[m, kb] * sb[n / 128, kb]).
// Each epilogue warp owns one 128-column half of the tile, so its B scale is
// one value per K block.
constexpr uint32_t kPartialCols = 256;
// 12 warps: warp 0 producer, warp 1 MMA, warps 2-3 idle, warps 4-11 promotion
// and epilogue. The first warpgroup gives up registers (setmaxnreg) so that
// each promotion thread holds its 128 accumulators and two 32-column TMEM
// loads in flight: 384 threads x 168 registers at launch = 128 x 56 + 256 x 224.
constexpr int kBlockThreads = 32 * (4 + kEpiWarps);
constexpr uint32_t kBlockCtlRegs = 56, kBlockEpiRegs = 224, kBlockLaunchRegs = 168;
static_assert(128 * kBlockCtlRegs + 32 * kEpiWarps * kBlockEpiRegs <=
                  kBlockThreads * kBlockLaunchRegs,
              "register split must fit the launch allocation");
static_assert(kBlockLaunchRegs * kBlockThreads <= 65536 &&
                  65536 / kBlockThreads / 8 * 8 == kBlockLaunchRegs,
              "launch bounds give 168 registers per thread");

template <int AFMT, int BFMT, int OUT>
__global__ void __launch_bounds__(kBlockThreads, 1)
    k_gemm_block(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b, const Params p) {
  using L = Smem<kPerTensor>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;   // 2 partial buffers
  uint64_t* pempty = pfull + 2;
  uint64_t* drain = pempty + 2;
  static_assert(2 * STAGES + 5 <= L::kNumBars, "barrier area too small");
  uint32_t* tmem_base_sh = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.num_m * p.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_sh;
  if (warp < 4) {
  regs_dec<kBlockCtlRegs>();
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(smem + L::kA + stage * A_BYTES, &tmap_a, kb * BKB, mb * BM, &full[stage]);
          tma_load_2d(smem + L::kB + stage * B_BYTES, &tmap_b, kb * BKB, nb * BN, &full[stage]);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(&full[s], (issued_parity >> s) & 1u) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // MMA warp: the whole warp runs the loop with warp-uniform addresses and
    // descriptors; lane 0 issues the MMAs and every commit.
    {
      int stage = 0, pbuf = 0;
      uint32_t phase = 0, pphase = 0;
      bool ok = true;
      const uint32_t idesc = idesc_f8f6f4(AFMT, BFMT, BM, BN);
      const uint32_t a_base = smem_u32(smem + L::kA), b_base = smem_u32(smem + L::kB);
      const uint64_t dhi = desc_sw128_hi();
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        for (int kb = 0; kb < p.num_kb; ++kb) {
          const bool w = mbar_wait(&pempty[pbuf], pphase ^ 1u, abort_flag, p.status, 1u) &&
                         mbar_wait(&full[stage], phase, abort_flag, p.status, 1u);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t alo = desc_sw128_lo(a_base + stage * A_BYTES);
          const uint32_t blo = desc_sw128_lo(b_base + stage * B_BYTES);
          const uint32_t d = tmem + pbuf * kPartialCols;
          if (elect_lane()) {
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k)
              mma_f8f6f4(d, dhi | (uint64_t)(alo + 2 * k), dhi | (uint64_t)(blo + 2 * k), idesc,
                         k > 0 ? 1u : 0u);
            tc_commit(&empty[stage]);
            tc_commit(&pfull[pbuf]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          pbuf ^= 1;
          if (pbuf == 0) pphase ^= 1u;
        }
      }
      if (elect_lane()) {
        tc_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0u) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      __syncwarp();
    }
  }  // warps 2-3: nothing to do
  } else {
    regs_inc<kBlockEpiRegs>();
    const int ew = warp - 4;
    const int quad = warp & 3;
    const int half = ew / 4;
    int pbuf = 0;
    uint32_t pphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int row = mb * BM + 32 * quad + lane;
      const int rs = row < p.M ? row : p.M - 1;  // clamp scale reads for rows past M
      const int bgrp = min(2 * nb + half, (p.N - 1) / 128);
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      // scales for K block kb+1 are loaded while block kb is promoted
      const float* sa_row = p.bsa + (int64_t)rs * p.bs_ld;
      const float* sb_row = p.bsb + (int64_t)bgrp * p.bs_ld;
      float sa_next = sa_row[0], sb_next = sb_row[0];
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const float s = __fmul_rn(sa_next, sb_next);
        if (kb + 1 < p.num_kb) {
          sa_next = sa_row[kb + 1];
          sb_next = sb_row[kb + 1];
        }
        if (!mbar_wait(&pfull[pbuf], pphase, abort_flag, p.status, 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + pbuf * kPartialCols + 128 * half;
        // 32-column TMEM loads issued in pairs (both in flight, one wait per
        // pair: two load latencies per K block instead of four); the partial
        // buffer is handed back once the second pair has landed, before its
        // FMAs. Packed FMAs (fma.rn.f32x2) round each element as one IEEE fma.
        const float2 s2 = make_float2(s, s);
        uint32_t ra[32], rb[32];
        auto promote = [&](const uint32_t (&cur)[32], int c) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 v = __ffma2_rn(
                make_float2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1])), s2,
                make_float2(acc[32 * c + 2 * i], acc[32 * c + 2 * i + 1]));
            acc[32 * c + 2 * i] = v.x;
            acc[32 * c + 2 * i + 1] = v.y;
          }
        };
        tmem_ld32(taddr, ra);
        tmem_ld32(taddr + 32, rb);
        tmem_ld_wait();
        reg_bind32(ra);
        reg_bind32(rb);
        promote(ra, 0);
        promote(rb, 1);
        tmem_ld32(taddr + 64, ra);
        tmem_ld32(taddr + 96, rb);
        tmem_ld_wait();
        reg_bind32(ra);
        reg_bind32(rb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pbuf]);
        promote(ra, 2);
        promote(rb, 3);
        pbuf ^= 1;
        if (pbuf == 0) pphase ^= 1u;
      }
      if (!ok) break;
      if (row < p.M) {
        const int col0 = nb * BN + 128 * half;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          store_row_chunk<OUT>(p.d, p.ldd, row, col0 + 32 * c, p.N, acc + 32 * c, 32);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Row-major uint8 matrix [rows, row_bytes] -> box [box_rows, 128 bytes], 128B swizzle.
int make_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes,
              uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return BRC_ERR_CUDA;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {BKB, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BRC_OK : BRC_ERR_CUDA;
}

template <int KIND, int AFMT, int BFMT, int OUT>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  auto kern = k_gemm<KIND, AFMT, BFMT, OUT>;
  const int smem = (int)Smem<KIND>::kAlloc;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return BRC_ERR_CUDA;
  if (!configured[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (rc) return rc;
    configured[dev] = true;
  }
  const int tiles = p.num_m * p.num_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kern<<<grid, kThreadsG<KIND>, smem, st>>>(ta, tb, p);
  return check_launch();
}

template <int KIND, int AFMT, int BFMT, int OUT, int CAST = 0>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                const CUtensorMap& tsb, const Params& p, cudaStream_t st) {
  auto kern = k_gemm_pair<KIND, AFMT, BFMT, OUT, CAST>;
  const int smem = (int)PairCfg<KIND>::kAlloc;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return BRC_ERR_CUDA;
  if (!configured[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (rc) return rc;
    configured[dev] = true;
  }
  const int tiles = p.num_m * p.num_n;
  const int pairs = sm_count() / 2;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  kern<<<grid, kThreadsP<KIND, CAST>, smem, st>>>(ta, tb, tsa, tsb, p);
  return check_launch();
}

template <int KIND, int AFMT, int BFMT>
int launch_pair_out(int out_dtype, const CUtensorMap& ta, const CUtensorMap& tb,
                    const CUtensorMap& tsa, const CUtensorMap& tsb, const Params& p,
                    cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32)
    return launch_pair<KIND, AFMT, BFMT, BRC_DTYPE_F32>(ta, tb, tsa, tsb, p, st);
  if (out_dtype == BRC_DTYPE_BF16)
    return launch_pair<KIND, AFMT, BFMT, BRC_DTYPE_BF16>(ta, tb, tsa, tsb, p, st);
  return launch_pair<KIND, AFMT, BFMT, BRC_DTYPE_F16>(ta, tb, tsa, tsb, p, st);
}

// Fused-cast pair kernel for (activation dtype, A / B formats, output dtype).
template <int CAST, int AFMT, int BFMT>
int launch_cast_pair_out(int out_dtype, const CUtensorMap& ta, const CUtensorMap& tb,
                         const Params& p, cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32)
    return launch_pair<kPerTensor, AFMT, BFMT, BRC_DTYPE_F32, CAST>(ta, tb, ta, tb, p, st);
  if (out_dtype == BRC_DTYPE_BF16)
    return launch_pair<kPerTensor, AFMT, BFMT, BRC_DTYPE_BF16, CAST>(ta, tb, ta, tb, p, st);
  return launch_pair<kPerTensor, AFMT, BFMT, BRC_DTYPE_F16, CAST>(ta, tb, ta, tb, p, st);
}
template <int CAST>
int launch_cast_pair_fmt(int a_fmt, int b_fmt, int out_dtype, const CUtensorMap& ta,
                         const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  if (a_fmt == BRC_FP8_E4M3 && b_fmt == BRC_FP8_E4M3)
    return launch_cast_pair_out<CAST, 0, 0>(out_dtype, ta, tb, p, st);
  if (a_fmt == BRC_FP8_E4M3) return launch_cast_pair_out<CAST, 0, 1>(out_dtype, ta, tb, p, st);
  if (b_fmt == BRC_FP8_E4M3) return launch_cast_pair_out<CAST, 1, 0>(out_dtype, ta, tb, p, st);
  return launch_cast_pair_out<CAST, 1, 1>(out_dtype, ta, tb, p, st);
}
int launch_cast_pair(int x_dtype, int a_fmt, int b_fmt, int out_dtype, const CUtensorMap& ta,
                     const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  if (x_dtype == BRC_DTYPE_BF16)
    return launch_cast_pair_fmt<1 + BRC_DTYPE_BF16>(a_fmt, b_fmt, out_dtype, ta, tb, p, st);
  if (x_dtype == BRC_DTYPE_F16)
    return launch_cast_pair_fmt<1 + BRC_DTYPE_F16>(a_fmt, b_fmt, out_dtype, ta, tb, p, st);
  return launch_cast_pair_fmt<1 + BRC_DTYPE_F32>(a_fmt, b_fmt, out_dtype, ta, tb, p, st);
}

// Scale atoms (512 bytes each, row group-major) as a 2-D tensor of rows of
// 128 uint32 values; a box is `atoms_k` consecutive atoms.
int make_sf_tmap(CUtensorMap* m, const uint8_t* sf, int row_groups, uint32_t col_tiles,
                 uint32_t atoms_k) {
  return encode_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, sf, 128,
                        (uint64_t)row_groups * col_tiles, 512, 128, atoms_k);
}

// CTA pairs (256 x 256 tiles) when they fill the GPU, single CTAs otherwise.
bool use_pairs(int M, int N) {
  return ((M + P_BM - 1) / P_BM) * ((N + P_BN - 1) / P_BN) >= sm_count() / 2;
}
void to_pair_params(Params& p) {
  p.num_m = (p.M + P_BM - 1) / P_BM;
  p.num_n = (p.N + P_BN - 1) / P_BN;
  p.group_m = kGroupM / 2;  // the same 2048 rows of A per tile group
}

template <int KIND, int AFMT, int BFMT>
int launch_out(int out_dtype, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
               cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32) return launch<KIND, AFMT, BFMT, BRC_DTYPE_F32>(ta, tb, p, st);
  if (out_dtype == BRC_DTYPE_BF16) return launch<KIND, AFMT, BFMT, BRC_DTYPE_BF16>(ta, tb, p, st);
  return launch<KIND, AFMT, BFMT, BRC_DTYPE_F16>(ta, tb, p, st);
}

template <int AFMT, int BFMT, int OUT>
int launch_block(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  auto kern = k_gemm_block<AFMT, BFMT, OUT>;
  const int smem = (int)Smem<kPerTensor>::kAlloc;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return BRC_ERR_CUDA;
  if (!configured[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (rc) return rc;
    configured[dev] = true;
  }
  const int tiles = p.num_m * p.num_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kern<<<grid, kBlockThreads, smem, st>>>(ta, tb, p);
  return check_launch();
}

template <int AFMT, int BFMT>
int launch_block_out(int out_dtype, const CUtensorMap& ta, const CUtensorMap& tb,
                     const Params& p, cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32) return launch_block<AFMT, BFMT, BRC_DTYPE_F32>(ta, tb, p, st);
  if (out_dtype == BRC_DTYPE_BF16) return launch_block<AFMT, BFMT, BRC_DTYPE_BF16>(ta, tb, p, st);
  return launch_block<AFMT, BFMT, BRC_DTYPE_F16>(ta, tb, p, st);
}

int check_common(const void* a, const void* b, void* d, int M, int N, int K, int out_dtype,
                 int k_multiple) {
  if (!a || !b || !d) return BRC_ERR_NULL;
  if (M < 0 || N < 0 || K < 0) return BRC_ERR_SHAPE;
  if (out_dtype != BRC_DTYPE_F32 && out_dtype != BRC_DTYPE_BF16 && out_dtype != BRC_DTYPE_F16)
    return BRC_ERR_DTYPE;
  if (K % k_multiple || N % 16) return BRC_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(d)) & 15)
    return BRC_ERR_ALIGN;
  return BRC_OK;
}


Params base_params(int M, int N, int K, int k_per_stage, void* d) {
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m = (M + BM - 1) / BM;
  p.num_n = (N + BN - 1) / BN;
  p.num_kb = K / k_per_stage;
  p.group_m = kGroupM;
  p.d = d;
  p.ldd = N;
  p.status = nullptr;
  return p;
}

}  // namespace gemm
}  // namespace brc

namespace brc {
int encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  gemm::EncodeTiledFn fn = gemm::encode_fn();
  if (!fn) return BRC_ERR_CUDA;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BRC_OK : BRC_ERR_CUDA;
}

// Device address of the sticky GEMM status word, for kernels in other
// translation units. Looked up once per device (with that device current) and
// cached, so later launches make no runtime lookups.
uint32_t* gemm_status_ptr() {
  static std::mutex mu;
  static uint32_t* cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    uint32_t* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_gemm_status) != cudaSuccess)
      return nullptr;
    cache[dev] = p;
  }
  return cache[dev];
}
}  // namespace brc

using namespace brc;
using namespace brc::gemm;

namespace {
uint32_t* status_word() { return brc::gemm_status_ptr(); }

// ------------------------------------------------------------------ failure-path self-test
// The GEMMs' failure path, run on purpose without a fault: one CTA sets up
// as the GEMMs do (barriers, a TMEM allocation), warp 0 waits on a barrier
// nothing ever arrives at with a short bound, and warp 1 waits on another
// with the GEMMs' normal 2 s bound. Warp 0's wait runs out, records the
// timeout in the status word and raises the CTA's abort flag; warp 1 must
// leave on that flag well before its own bound. Both then take the GEMMs'
// tear-down (fences, CTA barrier, TMEM freed by the warp that allocated it).
// Bit w of g_selftest_roles is set when warp w left its wait without the
// barrier completing.
__device__ uint32_t g_selftest_roles = 0;

__global__ void __launch_bounds__(64, 1) k_selftest_wait_timeout(uint64_t limit_ns,
                                                                 uint32_t* status) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ uint32_t abort_word;
  volatile uint32_t* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const bool done = warp == 0
                        ? __all_sync(0xffffffffu, mbar_wait(&bars[0], 0u, abort_flag, status, 1u,
                                                            limit_ns))
                        : __all_sync(0xffffffffu, mbar_wait(&bars[1], 0u, abort_flag, status, 1u));
  if (lane == 0 && !done) atomicOr(&g_selftest_roles, 1u << warp);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}
}  // namespace

extern "C" {

int brc_gemm_fp8_pertensor(const uint8_t* a, const uint8_t* b, int M, int N, int K, int a_fmt,
                           int b_fmt, const float* a_scale, const float* b_scale, void* d,
                           int d_dtype, void* stream) {
  int rc = check_common(a, b, d, M, N, K, d_dtype, BKB);
  if (rc) return rc;
  if (!a_scale || !b_scale) return BRC_ERR_NULL;
  if ((a_fmt != BRC_FP8_E4M3 && a_fmt != BRC_FP8_E5M2) ||
      (b_fmt != BRC_FP8_E4M3 && b_fmt != BRC_FP8_E5M2))
    return BRC_ERR_DTYPE;
  if ((int64_t)M * N == 0) return BRC_OK;
  if (K == 0) return BRC_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap ta, tb;
  if (use_pairs(M, N)) {
    if ((rc = make_tmap(&ta, a, M, K, 128))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, 128))) return rc;
    Params p = base_params(M, N, K, BKB, d);
    to_pair_params(p);
    // 16 row blocks (4096 rows, a 33.5 MB A panel at K = 8192) per tile group:
    // C2's weight then streams from DRAM 4 times instead of 8 (748.7 -> 730.2
    // us); 32 (a 67 MB panel that no longer stays in L2) measured 809 against
    // 751 us, and the MXFP8 GEMM measured no better with 16 and keeps 8.
    p.group_m = kGroupM;
    p.a_scale = a_scale;
    p.b_scale = b_scale;
    p.status = status_word();
    if (a_fmt == BRC_FP8_E4M3 && b_fmt == BRC_FP8_E4M3)
      return launch_pair_out<kPerTensor, 0, 0>(d_dtype, ta, tb, ta, tb, p, st);
    if (a_fmt == BRC_FP8_E4M3)
      return launch_pair_out<kPerTensor, 0, 1>(d_dtype, ta, tb, ta, tb, p, st);
    if (b_fmt == BRC_FP8_E4M3)
      return launch_pair_out<kPerTensor, 1, 0>(d_dtype, ta, tb, ta, tb, p, st);
    return launch_pair_out<kPerTensor, 1, 1>(d_dtype, ta, tb, ta, tb, p, st);
  }
  if ((rc = make_tmap(&ta, a, M, K, BM))) return rc;
  if ((rc = make_tmap(&tb, b, N, K, BN))) return rc;
  Params p = base_params(M, N, K, BKB, d);
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.status = status_word();
  if (a_fmt == BRC_FP8_E4M3 && b_fmt == BRC_FP8_E4M3)
    return launch_out<kPerTensor, 0, 0>(d_dtype, ta, tb, p, st);
  if (a_fmt == BRC_FP8_E4M3) return launch_out<kPerTensor, 0, 1>(d_dtype, ta, tb, p, st);
  if (b_fmt == BRC_FP8_E4M3) return launch_out<kPerTensor, 1, 0>(d_dtype, ta, tb, p, st);
  return launch_out<kPerTensor, 1, 1>(d_dtype, ta, tb, p, st);
}

int64_t brc_cast_gemm_workspace_bytes(int M, int K) {
  if (M < 0 || K < 0) return -1;
  const int64_t mblocks = (M + P_BM - 1) / P_BM, kchunks = (K + kCastChunk - 1) / kCastChunk;
  return 16 + 4 * mblocks * kchunks;
}

int brc_cast_gemm_pertensor_fp8(const void* x, int x_dtype, int a_fmt, const uint8_t* b,
                                int b_fmt, const float* b_scale, int M, int N, int K,
                                float* history, int history_len, int margin, int use_history,
                                const uint32_t* amax_in, uint8_t* a_codes, float* a_scale_out,
                                void* d, int d_dtype, void* workspace, int64_t workspace_bytes,
                                int prologue_rows, void* stream) {
  if (!a_codes || !a_scale_out || !workspace || !b_scale) return BRC_ERR_NULL;
  int rc = check_common(x, b, d, M, N, K, d_dtype, BKB);
  if (rc) return rc;
  if (x_dtype != BRC_DTYPE_F32 && x_dtype != BRC_DTYPE_BF16 && x_dtype != BRC_DTYPE_F16)
    return BRC_ERR_DTYPE;
  if ((a_fmt != BRC_FP8_E4M3 && a_fmt != BRC_FP8_E5M2) ||
      (b_fmt != BRC_FP8_E4M3 && b_fmt != BRC_FP8_E5M2))
    return BRC_ERR_DTYPE;
  if (reinterpret_cast<uintptr_t>(a_codes) & 15) return BRC_ERR_ALIGN;
  if (history && history_len < 1) return BRC_ERR_SHAPE;
  if (history && amax_in) return BRC_ERR_UNSUPPORTED;
  if (margin < -126 || margin > 127) return BRC_ERR_RANGE;
  if (workspace_bytes < brc_cast_gemm_workspace_bytes(M, K)) return BRC_ERR_SHAPE;
  if (K == 0 && M > 0 && N > 0) return BRC_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = (int64_t)M * K;
  uint32_t* ws = static_cast<uint32_t*>(workspace);
  if ((rc = check_cuda(cudaMemsetAsync(ws, 0, (size_t)brc_cast_gemm_workspace_bytes(M, K), st))))
    return rc;
  // 1. the scale: from the history, from the caller's (all-reduced) amax, or
  //    from the amax of the whole tensor
  if (amax_in) {
    if ((rc = pertensor_fp8_scale(x, x_dtype, n, a_fmt, reinterpret_cast<const float*>(amax_in),
                                  1, 0, true, ws, a_scale_out, st)))
      return rc;
  } else {
    const bool from_history = history && use_history;
    if ((rc = pertensor_fp8_scale(x, x_dtype, n, a_fmt, history, history_len, margin,
                                  from_history, ws, a_scale_out, st)))
      return rc;
  }
  // 2. the first tile group's rows, before the GEMM (all of A when there is
  //    no GEMM to overlap with)
  // tile groups of 16 row blocks, as the plain per-tensor GEMM: the first
  // group's rows are encoded before the launch
  const int group_m = kGroupM;
  int first = M;
  if (N > 0) {
    const int group_rows = group_m * P_BM;
    first = prologue_rows < 0 ? group_rows : prologue_rows / P_BM * P_BM;
    if (first > M) first = M;
  }
  if ((rc = pertensor_fp8_encode(x, x_dtype, (int64_t)first * K, a_fmt, a_scale_out, a_codes, ws,
                                 st)))
    return rc;
  // 3. the GEMM, its casters encoding rows [first, M)
  if (N > 0 && M > 0) {
    CUtensorMap ta, tb;
    if ((rc = make_tmap(&ta, a_codes, M, K, 128))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, 128))) return rc;
    Params p = base_params(M, N, K, BKB, d);
    to_pair_params(p);
    p.group_m = group_m;
    p.a_scale = a_scale_out;
    p.b_scale = b_scale;
    p.status = status_word();
    p.x = x;
    p.a_codes = a_codes;
    p.amax_bits = ws;
    p.cast_next = ws + 1;
    p.gemm_group = ws + 2;
    p.cast_ready = ws + 4;
    p.first_rows = first;
    p.kchunks = (K + kCastChunk - 1) / kCastChunk;
    rc = launch_cast_pair(x_dtype, a_fmt, b_fmt, d_dtype, ta, tb, p, st);
    if (rc) return rc;
  }
  // 4. the history records this tensor's amax
  if (history) return pertensor_fp8_history_push(history, history_len, ws, st);
  return BRC_OK;
}

int brc_gemm_mxfp8(const uint8_t* a, const uint8_t* b, int M, int N, int K, int a_fmt,
                   int b_fmt, const uint8_t* a_sf_mma, const uint8_t* b_sf_mma, void* d,
                   int d_dtype, void* stream) {
  int rc = check_common(a, b, d, M, N, K, d_dtype, BKB);
  if (rc) return rc;
  if (!a_sf_mma || !b_sf_mma) return BRC_ERR_NULL;
  if ((a_fmt != BRC_FP8_E4M3 && a_fmt != BRC_FP8_E5M2) ||
      (b_fmt != BRC_FP8_E4M3 && b_fmt != BRC_FP8_E5M2))
    return BRC_ERR_DTYPE;
  if (((reinterpret_cast<uintptr_t>(a_sf_mma) | reinterpret_cast<uintptr_t>(b_sf_mma)) & 15))
    return BRC_ERR_ALIGN;
  if ((int64_t)M * N == 0) return BRC_OK;
  if (K == 0) return BRC_ERR_UNSUPPORTED;
  CUtensorMap ta, tb;
  cudaStream_t st = (cudaStream_t)stream;
  const uint32_t sf_col_tiles = (uint32_t)((K / 32 + 3) / 4);
  if (use_pairs(M, N)) {
    CUtensorMap tsa, tsb;
    if ((rc = make_tmap(&ta, a, M, K, 128))) return rc;
    if ((rc = make_tmap(&tb, b, N, K, 128))) return rc;
    if ((rc = make_sf_tmap(&tsa, a_sf_mma, (M + 127) / 128, sf_col_tiles, 1))) return rc;
    if ((rc = make_sf_tmap(&tsb, b_sf_mma, (N + 127) / 128, sf_col_tiles, 1))) return rc;
    Params p = base_params(M, N, K, BKB, d);
    to_pair_params(p);
    p.sf_col_tiles = sf_col_tiles;
    p.sfb_row_atoms = (N + 127) / 128;
    p.status = status_word();
    if (a_fmt == BRC_FP8_E4M3 && b_fmt == BRC_FP8_E4M3)
      return launch_pair_out<kMxfp8, 0, 0>(d_dtype, ta, tb, tsa, tsb, p, st);
    if (a_fmt == BRC_FP8_E4M3)
      return launch_pair_out<kMxfp8, 0, 1>(d_dtype, ta, tb, tsa, tsb, p, st);
    if (b_fmt == BRC_FP8_E4M3)
      return launch_pair_out<kMxfp8, 1, 0>(d_dtype, ta, tb, tsa, tsb, p, st);
    return launch_pair_out<kMxfp8, 1, 1>(d_dtype, ta, tb, tsa, tsb, p, st);
  }
  if ((rc = make_tmap(&ta, a, M, K, BM))) return rc;
  if ((rc = make_tmap(&tb, b, N, K, BN))) return rc;
  Params p = base_params(M, N, K, BKB, d);
  p.sfa = a_sf_mma;
  p.sfb = b_sf_mma;
  p.sf_col_tiles = sf_col_tiles;
  p.sfb_row_atoms = (N + 127) / 128;
  p.status = status_word();
  if (a_fmt == BRC_FP8_E4M3 && b_fmt == BRC_FP8_E4M3)
    return launch_out<kMxfp8, 0, 0>(d_dtype, ta, tb, p, st);
  if (a_fmt == BRC_FP8_E4M3) return launch_out<kMxfp8, 0, 1>(d_dtype, ta, tb, p, st);
  if (b_fmt == BRC_FP8_E4M3) return launch_out<kMxfp8, 1, 0>(d_dtype, ta, tb, p, st);
  return launch_out<kMxfp8, 1, 1>(d_dtype, ta, tb, p, st);
}

int brc_gemm_nvfp4(const uint8_t* a_packed, const uint8_t* b_packed, int M, int N, int K,
                   const uint8_t* a_sf_mma, const uint8_t* b_sf_mma, void* d, int d_dtype,
                   void* stream) {
  int rc = check_common(a_packed, b_packed, d, M, N, K, d_dtype, 2 * BKB);
  if (rc) return rc;
  if (!a_sf_mma || !b_sf_mma) return BRC_ERR_NULL;
  if (((reinterpret_cast<uintptr_t>(a_sf_mma) | reinterpret_cast<uintptr_t>(b_sf_mma)) & 15))
    return BRC_ERR_ALIGN;
  if ((int64_t)M * N == 0) return BRC_OK;
  if (K == 0) return BRC_ERR_UNSUPPORTED;
  CUtensorMap ta, tb;
  const uint32_t sf_col_tiles = (uint32_t)((K / 16 + 3) / 4);
  // NVFP4 on CTA pairs: with both kernels' scale-factor copies on copier
  // warps the pair form is ahead (4096 x 28672 x 8192: 0.513 vs 0.527 ms);
  // before the copiers the single-CTA form was (0.599 vs 0.617 ms).
  constexpr bool kNvfp4Pairs = true;
  if (kNvfp4Pairs && use_pairs(M, N)) {
    CUtensorMap tsa, tsb;
    if ((rc = make_tmap(&ta, a_packed, M, K / 2, 128))) return rc;
    if ((rc = make_tmap(&tb, b_packed, N, K / 2, 128))) return rc;
    if ((rc = make_sf_tmap(&tsa, a_sf_mma, (M + 127) / 128, sf_col_tiles, 4))) return rc;
    if ((rc = make_sf_tmap(&tsb, b_sf_mma, (N + 127) / 128, sf_col_tiles, 4))) return rc;
    Params p = base_params(M, N, K, 2 * BKB, d);
    to_pair_params(p);
    // Tile groups of 16 row blocks (4096 rows): 4-bit A rows are half the bytes
    // of FP8 ones, so a group's A panel is the same 16.8 MB at K = 8192, and for
    // M up to 4096 the weight streams from DRAM once instead of once per
    // 2048-row group (C4 read 286 MB per launch with 8 row blocks per group).
    p.group_m = kGroupM;
    p.sf_col_tiles = sf_col_tiles;
    p.sfb_row_atoms = (N + 127) / 128;
    p.status = status_word();
    return launch_pair_out<kNvfp4, 0, 0>(d_dtype, ta, tb, tsa, tsb, p, (cudaStream_t)stream);
  }
  if ((rc = make_tmap(&ta, a_packed, M, K / 2, BM))) return rc;
  if ((rc = make_tmap(&tb, b_packed, N, K / 2, BN))) return rc;
  Params p = base_params(M, N, K, 2 * BKB, d);
  p.sfa = a_sf_mma;
  p.sfb = b_sf_mma;
  p.sf_col_tiles = sf_col_tiles;
  p.sfb_row_atoms = (N + 127) / 128;
  p.status = status_word();
  return launch_out<kNvfp4, 0, 0>(d_dtype, ta, tb, p, (cudaStream_t)stream);
}

int brc_gemm_block_fp8(const uint8_t* a, const uint8_t* b, int M, int N, int K, int a_fmt,
                       int b_fmt, const float* a_scales, const float* b_scales, void* d,
                       int d_dtype, void* stream) {
  int rc = check_common(a, b, d, M, N, K, d_dtype, BKB);
  if (rc) return rc;
  if (!a_scales || !b_scales) return BRC_ERR_NULL;
  if ((a_fmt != BRC_FP8_E4M3 && a_fmt != BRC_FP8_E5M2) ||
      (b_fmt != BRC_FP8_E4M3 && b_fmt != BRC_FP8_E5M2))
    return BRC_ERR_DTYPE;
  if ((int64_t)M * N == 0) return BRC_OK;
  if (K == 0) return BRC_ERR_UNSUPPORTED;
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, a, M, K, BM))) return rc;
  if ((rc = make_tmap(&tb, b, N, K, BN))) return rc;
  Params p = base_params(M, N, K, BKB, d);
  p.bsa = a_scales;
  p.bsb = b_scales;
  p.bs_ld = K / 128;
  p.status = status_word();
  cudaStream_t st = (cudaStream_t)stream;
  if (a_fmt == BRC_FP8_E4M3 && b_fmt == BRC_FP8_E4M3)
    return launch_block_out<0, 0>(d_dtype, ta, tb, p, st);
  if (a_fmt == BRC_FP8_E4M3) return launch_block_out<0, 1>(d_dtype, ta, tb, p, st);
  if (b_fmt == BRC_FP8_E4M3) return launch_block_out<1, 0>(d_dtype, ta, tb, p, st);
  return launch_block_out<1, 1>(d_dtype, ta, tb, p, st);
}

int brc_gemm_bf16(const void* a, const void* b, int M, int N, int K, void* d, int d_dtype,
                  void* stream) {
  int rc = check_common(a, b, d, M, N, K, d_dtype, 8);
  if (rc) return rc;
  if ((int64_t)M * N == 0) return BRC_OK;
  if (K == 0) return BRC_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const uint64_t row_bytes = 2ull * (uint64_t)K;
  // 64 bf16 (128 bytes) of K per stage; a partial last stage reads zeros
  // past the row end (the tensor map's out-of-bounds fill), adding nothing.
  const int num_kb = (int)((row_bytes + BKB - 1) / BKB);
  CUtensorMap ta, tb;
  if (use_pairs(M, N)) {
    if ((rc = make_tmap(&ta, a, M, row_bytes, 128))) return rc;
    if ((rc = make_tmap(&tb, b, N, row_bytes, 128))) return rc;
    Params p = base_params(M, N, K, 64, d);
    p.num_kb = num_kb;
    to_pair_params(p);
    p.status = status_word();
    return launch_pair_out<kBf16, 0, 0>(d_dtype, ta, tb, ta, tb, p, st);
  }
  if ((rc = make_tmap(&ta, a, M, row_bytes, BM))) return rc;
  if ((rc = make_tmap(&tb, b, N, row_bytes, BN))) return rc;
  Params p = base_params(M, N, K, 64, d);
  p.num_kb = num_kb;
  p.status = status_word();
  return launch_out<kBf16, 0, 0>(d_dtype, ta, tb, p, st);
}

int brc_selftest_wait_timeout(int limit_us, int* roles_out, void* stream) {
  if (limit_us <= 0 || limit_us > 1000000) return BRC_ERR_RANGE;
  uint32_t* status = status_word();
  if (!status) return BRC_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  const uint32_t zero = 0;
  int rc = check_cuda(cudaMemcpyToSymbolAsync(g_selftest_roles, &zero, sizeof(zero), 0,
                                              cudaMemcpyHostToDevice, st));
  if (rc) return rc;
  k_selftest_wait_timeout<<<1, 64, 0, st>>>((uint64_t)limit_us * 1000ull, status);
  if ((rc = check_launch())) return rc;
  if ((rc = check_cuda(cudaStreamSynchronize(st)))) return rc;
  uint32_t roles = 0, st_word = 0;
  if ((rc = check_cuda(cudaMemcpyFromSymbol(&roles, g_selftest_roles, sizeof(roles))))) return rc;
  if ((rc = check_cuda(cudaMemcpyFromSymbol(&st_word, g_gemm_status, sizeof(st_word)))))
    return rc;
  if (roles_out) *roles_out = (int)roles;
  return (st_word & 1u) ? BRC_ERR_TIMEOUT : BRC_OK;
}

int brc_gemm_status(int reset) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v)) != cudaSuccess) return BRC_ERR_CUDA;
  if (reset) {
    const uint32_t z = 0;
    if (cudaMemcpyToSymbol(g_gemm_status, &z, sizeof(z)) != cudaSuccess) return BRC_ERR_CUDA;
  }
  return (int)v;
}

}  // extern "C"
