// INT4 weight-only skinny GEMM (decode-shaped: M <= 16 activation rows).
//
//   out[m, n] = sum_g s[n, g] * sum_{k in g} A[m, k] * (q[n, k] - zp[n, g])
//
// A is bfloat16 (M, K); the weight is the INT4 cast of W^T (N, K) in the
// skinny-GEMM tile layout brc_cast_int4 writes (16 rows x one 128-element
// group per 1 KB tile, plus fp32 scales and 128 + zero point per tile row).
// The value (q - zp) is an integer in [-15, 15], exact in bfloat16, so each
// group's inner sum runs on the tensor cores (mma.sync m16n8k16, bf16 x bf16
// -> fp32) with the weight as the 16-row "A" operand and the activations as
// the 8-column "B" operand (one n8 tile for M <= 8, two for M <= 16); the
// group scale is applied to the fp32 partial. This equals the reference's
// dequantize-then-float32-matmul (src/breccia/kernels/reference/matmul.py:
// 123-133 on src/breccia/kernels/reference/cast.py:574-586) up to float32
// rounding order.
//
// The MMA is fed bf16 (128 + code) (one byte permute per pair of codes) and
// the offset is removed per group in float32:
//   sum_k A_k (q_k - zp) = sum_k A_k (128 + q_k) - (128 + zp) * sum_k A_k.
// The per-(activation row, group) sums sum_k A_k come from the tensor cores
// too: one chunk of activations at a time, an MMA against an all-ones
// fragment gives them in exactly the layout the correction needs.
//
// Fragment layout. Thread t of a warp reads bytes 16t..16t+15 of each of its
// two rows' 64-byte group: word i holds elements 32t+8i .. 32t+8i+7, element
// 32t+8i+j (j < 4) in the low nibble of byte j and element 32t+8i+4+j in its
// high nibble. The low nibbles of word i form one k16 MMA step, the high
// nibbles the next: MMA column slots 2t, 2t+1 take elements +0, +1 and slots
// 2t+8, 2t+9 take +2, +3 (+4..+7 for the high nibbles). The matching B
// fragment is 4 consecutive activations, one 8-byte shared-memory load, so
// the activations stay in their natural order and are loaded by bulk copies.
//
// Pipeline. The CTA owns a contiguous range of 16-row blocks. A producer
// warp streams the CTA's tiles (row block by row block, one activation chunk
// at a time; the chunk is the whole K when it fits in shared memory) through
// a ring of large stages of 32 tiles (about 37 KB, three bulk copies when
// the tiles are contiguous), and loads the activation chunks. Two ways to
// split a stage among the 16 consumer warps:
//  * shared (a row block's chunk spans more than a stage: M <= 4 at K = 8192,
//    whole K resident): each warp takes two consecutive tiles (two groups of
//    one row block) of every stage; partial sums of a row block meet in
//    shared memory;
//  * owner (a stage holds whole row blocks of the chunk: the chunked
//    activations of M > 4): each warp owns the CTA's row blocks w and w + 16,
//    keeps their sums in registers across every chunk and writes them at the
//    end. With the shared split a chunk of 8 groups moved each warp to a new
//    row block every stage, and the shared-memory partial-sum atomics took
//    about 30% of the time (C5 M = 16: 84 -> 63 us).
// Stages are released through "empty" mbarriers (one arrival per consumer
// warp in both modes: an owner passes the stages it has no tile in). Every wait is bounded: on a timeout the waiter
// records the status bit and raises the CTA's abort flag; the others see the
// flag, stop, and the producer waits for its copies in flight.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "breccia_b200.h"
#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace brc {

uint32_t* gemm_status_ptr();  // device address of the GEMM status word (gemm_sm100.cu)

namespace int4gemm {

using namespace sm100;

constexpr int G = 128;                   // group size handled by this kernel
constexpr int TILE_BYTES = 16 * 64;      // 16 rows x one group of packed codes
constexpr int TILE_SLOT = TILE_BYTES + 64 + 64;  // + 16 scales + 16 (128 + zero point)
// NC consumer warps (one tile of every stage each) + one producer warp
__host__ __device__ constexpr int threads_for(int NC) { return 32 * (NC + 1); }
constexpr int TPW = 2;  // consecutive tiles per consumer warp per stage (same row block)
__host__ __device__ constexpr int stage_bytes(int NC) { return NC * TPW * TILE_SLOT; }
// 24 consumer warps with one activation n8 tile (M <= 8, fewer registers per
// thread), 16 with two
__host__ __device__ constexpr int consumers_for(int MT) { return MT == 1 ? 16 : 16; }
constexpr int kSmemLimit = 227 * 1024;
constexpr int kApad = 8;    // bf16 elements of padding per activation row in shared memory
constexpr int kMaxRb = 32;  // row blocks per CTA (sizes the partial-sum area)
constexpr int kMaxStages = 16;

struct Params {
  const __nv_bfloat16* a;  // (M, K)
  const uint8_t* w;        // tiles, 1 KB each: tile (n/16) * (K/128) + g
  const float* sc;         // 16 per tile
  const float* zp;         // 16 per tile (128 + zero point), asymmetric only
  void* out;               // (M, N)
  int M, N, K;
  int kc;      // activation columns per chunk (divides K)
  int nb;      // activation buffers: 1 (kc == K) or 2 (double buffered)
  int stages;  // ring stages
  int rbmax;   // row blocks per CTA, at most
  uint32_t* status;
};

struct Layout {  // byte offsets into dynamic shared memory
  uint32_t a, sa, acc, ring, full, empty, afull, aempty, safull, misc, total;
};

__host__ __device__ inline uint32_t take(uint32_t& o, uint32_t bytes) {
  const uint32_t r = o;
  o = (o + bytes + 15u) & ~15u;
  return r;
}
__host__ __device__ inline Layout layout(int NC, int M, int kc, int nb, int stages, int rbmax) {
  Layout L;
  uint32_t o = 0;
  L.a = take(o, (uint32_t)(nb * M * (kc + kApad) * 2));
  L.sa = take(o, (uint32_t)(nb * (kc / G) * 16 * 4));
  L.acc = take(o, (uint32_t)(rbmax * 16 * M * 4));
  L.ring = take(o, (uint32_t)(stages * stage_bytes(NC)));
  L.full = take(o, (uint32_t)(stages * 8));
  L.empty = take(o, (uint32_t)(stages * 8));
  L.afull = take(o, 2 * 8);
  L.aempty = take(o, 2 * 8);
  L.safull = take(o, 2 * 8);
  L.misc = take(o, 16);
  L.total = o;
  return L;
}

// c += A * B (16 x 8 x 16, bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// d = A * B (the first step of an accumulation chain)
__device__ __forceinline__ void mma_bf16_first(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// Two 4-bit codes (bytes 2j and 2j+1 of x, one code per byte) as the bf16
// pair (128 + code): bf16 0x43cc is 128 + cc for cc < 128, so one byte
// permute against the constant 0x43 builds both halves.
template <int J>
__device__ __forceinline__ uint32_t code_pair(uint32_t x) {
  constexpr uint32_t sel = (2 * J) | (4 << 4) | ((2 * J + 1) << 8) | (4 << 12);
  return prmt(x, 0x43434343u, sel);
}

__device__ __forceinline__ void red_shared_add(float* p, float v) {
  asm volatile("red.shared.add.f32 [%0], %1;" ::"r"(smem_u32(p)), "f"(v) : "memory");
}

// Barrier of the NC consumer warps only (the producer warp does not take part).
template <int NC>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory");
}

// One tile's contribution to the running sums: the group's 8 k16 MMA steps
// (low nibbles and high nibbles on two independent accumulator chains),
// then tot += scale * (acc - (128 + zp) * group sum of the activations).
template <int MT, int MODE>
__device__ __forceinline__ void tile_math(float (&tot)[MT][4], const uint4 w0, const uint4 w1,
                                          const float2 sc, const float2 off,
                                          const __nv_bfloat16* const (&brow)[MT],
                                          const float* sa_g, int t) {
  const uint32_t r0[4] = {w0.x, w0.y, w0.z, w0.w};
  const uint32_t r1[4] = {w1.x, w1.y, w1.z, w1.w};
  float acc[2][MT][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t a0 = r0[i], a1 = r1[i];
    if constexpr (MODE == 1) {
      a0 ^= 0x88888888u;  // two's-complement nibble q -> q + 8
      a1 ^= 0x88888888u;
    }
    const uint32_t x0 = a0 & 0x0F0F0F0Fu, y0 = (a0 >> 4) & 0x0F0F0F0Fu;
    const uint32_t x1 = a1 & 0x0F0F0F0Fu, y1 = (a1 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t u0 = h ? y0 : x0, u1 = h ? y1 : x1;
      const uint32_t af[4] = {code_pair<0>(u0), code_pair<0>(u1), code_pair<1>(u0),
                              code_pair<1>(u1)};
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint2 bv = *reinterpret_cast<const uint2*>(brow[mt] + 8 * i + 4 * h);
        if (i == 0) mma_bf16_first(acc[h][mt], af, bv.x, bv.y);
        else mma_bf16(acc[h][mt], af, bv.x, bv.y);
      }
    }
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const float2 sa = *reinterpret_cast<const float2*>(sa_g + mt * 8 + 2 * t);
    const float c0 = acc[0][mt][0] + acc[1][mt][0], c1 = acc[0][mt][1] + acc[1][mt][1];
    const float c2 = acc[0][mt][2] + acc[1][mt][2], c3 = acc[0][mt][3] + acc[1][mt][3];
    tot[mt][0] = __fmaf_rn(sc.x, __fmaf_rn(-off.x, sa.x, c0), tot[mt][0]);
    tot[mt][1] = __fmaf_rn(sc.x, __fmaf_rn(-off.x, sa.y, c1), tot[mt][1]);
    tot[mt][2] = __fmaf_rn(sc.y, __fmaf_rn(-off.y, sa.x, c2), tot[mt][2]);
    tot[mt][3] = __fmaf_rn(sc.y, __fmaf_rn(-off.y, sa.y, c3), tot[mt][3]);
  }
}

// Wait for `parity` of `bar` while also watching the abort flag; bounded.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile uint32_t* abort_flag, uint32_t* status) {
  return mbar_wait(bar, parity, abort_flag, status, 1u);
}

// OWNER (used when a stage holds whole row blocks of a chunk, 32 % gpc == 0):
// consumer warp w owns the CTA's row blocks w, w + NC; it walks every stage
// of every chunk in order (waiting on it and releasing it, so the ring's
// barrier counts are those of the shared mode) but does the math only for
// its own row blocks, keeps their sums in registers across all chunks, and
// writes them to global memory at the end: no shared-memory partial sums.
// Otherwise every warp takes TPW tiles of every stage and row-block partial
// sums meet in shared memory.
template <int MT, int MODE, int OUT, int NC, bool OWNER>  // MODE 0: unsigned sym, 1: signed sym, 2: asym
__global__ void __launch_bounds__(threads_for(NC), 1) k_int4_skinny(const Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int kConsumers = NC, kThreads = threads_for(NC), STAGE_TILES = NC * TPW;
  constexpr int STAGE_BYTES = stage_bytes(NC);
  const Layout L = layout(NC, p.M, p.kc, p.nb, p.stages, p.rbmax);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = p.stages;
  const int groups = p.K / G, gpc = p.kc / G, nchunks = p.K / p.kc;
  const int rs = p.kc + kApad;  // activation row stride in shared memory (elements)

  // this CTA's row blocks; per chunk its tiles i = 0 .. items-1 are
  // (row block i / gpc, group i % gpc), stage k holding i = 16k .. 16k+15
  const int n_rb = p.N / 16;
  const int rb0 = (int)((int64_t)blockIdx.x * n_rb / gridDim.x);
  const int nrb = (int)((int64_t)(blockIdx.x + 1) * n_rb / gridDim.x) - rb0;
  const int items = nrb * gpc;
  const int nst = (items + STAGE_TILES - 1) / STAGE_TILES;  // stages per chunk

  __nv_bfloat16* A_s = reinterpret_cast<__nv_bfloat16*>(smem + L.a);
  float* SA_s = reinterpret_cast<float*>(smem + L.sa);
  float* acc_s = reinterpret_cast<float*>(smem + L.acc);
  uint8_t* ring = smem + L.ring;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
  uint64_t* afull = reinterpret_cast<uint64_t*>(smem + L.afull);
  uint64_t* aempty = reinterpret_cast<uint64_t*>(smem + L.aempty);
  // a chunk buffer's activation group sums are in shared memory (one arrival
  // per warp that computes some of them)
  uint64_t* safull = reinterpret_cast<uint64_t*>(smem + L.safull);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L.misc);

  if (threadIdx.x == 0) {
    for (int i = 0; i < R; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumers);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], kConsumers);
      mbar_init(&safull[b], min(p.kc / G, kConsumers));
    }
    *abort_flag = 0u;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < nrb * 16 * p.M; i += kThreads) acc_s[i] = 0.f;
  __syncthreads();

  if (warp == kConsumers) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    constexpr uint32_t kZp = MODE == 2 ? 64u : 0u;
    int a_next = 0;  // next activation chunk to load
    auto load_a = [&](int c) {
      uint64_t* bar = &afull[c % p.nb];
      __nv_bfloat16* dst = A_s + (size_t)(c % p.nb) * p.M * rs;
      mbar_arrive_expect_tx(bar, (uint32_t)(p.M * p.kc * 2));
      for (int m = 0; m < p.M; ++m)
        bulk_load(dst + (size_t)m * rs, p.a + (int64_t)m * p.K + (int64_t)c * p.kc,
                  (uint32_t)(p.kc * 2), bar);
    };
    // chunk c >= 2 reuses the buffer of chunk c - 2, free once every
    // consumer warp has arrived on its "empty" barrier
    auto try_load_next_a = [&]() {
      if (a_next >= nchunks) return;
      if (a_next >= 2 &&
          !mbar_test_wait(&aempty[a_next % 2], (uint32_t)(((a_next - 2) / 2) & 1)))
        return;
      load_a(a_next++);
    };
    load_a(a_next++);
    if (nchunks > 1) load_a(a_next++);
    int slot = 0, q = 0;  // ring slot and global stage counter
    uint32_t fill = 0;    // parity of the slot's fill being issued
    bool ok = true;
    for (int c = 0; ok && c < nchunks; ++c) {
      int rbl = 0, gl = 0;  // position of the stage's first tile
      for (int k = 0; ok && k < nst; ++k, ++q) {
        if (q >= R) {
          // wait (bounded) for the consumers to release the slot, loading
          // activation chunks as their buffers free up meanwhile (polling
          // without blocking while a chunk load is still pending)
          const uint64_t t0 = globaltimer();
          while (!(a_next < nchunks ? mbar_test_wait(&empty[slot], fill ^ 1u)
                                    : mbar_try_wait(&empty[slot], fill ^ 1u))) {
            try_load_next_a();
            if (*abort_flag || globaltimer() - t0 > kWaitLimitNs) {
              if (!*abort_flag) {
                *abort_flag = 1u;
                if (p.status) atomicOr(p.status, 1u);
              }
              ok = false;
              break;
            }
          }
          if (!ok) break;
        }
        const int n = min(STAGE_TILES, items - k * STAGE_TILES);
        uint8_t* dst = ring + (size_t)slot * STAGE_BYTES;
        uint64_t* bar = &full[slot];
        mbar_arrive_expect_tx(bar, (uint32_t)n * (TILE_BYTES + 64u + kZp));
        // runs of contiguous tiles: a row block's groups of this chunk, and
        // consecutive row blocks too when the chunk is the whole K
        for (int gi = 0; gi < n;) {
          int run = n - gi;
          if (gpc != groups && run > gpc - gl) run = gpc - gl;
          const int64_t tile = (int64_t)(rb0 + rbl) * groups + (int64_t)c * gpc + gl;
          bulk_load(dst + gi * TILE_BYTES, p.w + tile * TILE_BYTES, (uint32_t)(run * TILE_BYTES),
                    bar);
          bulk_load(dst + STAGE_TILES * TILE_BYTES + gi * 64, p.sc + tile * 16,
                    (uint32_t)(run * 64), bar);
          if constexpr (MODE == 2)
            bulk_load(dst + STAGE_TILES * (TILE_BYTES + 64) + gi * 64, p.zp + tile * 16,
                      (uint32_t)(run * 64), bar);
          gi += run;
          gl += run;
          while (gl >= gpc) {
            gl -= gpc;
            ++rbl;
          }
        }
        try_load_next_a();
        if (++slot == R) {
          slot = 0;
          fill ^= 1u;
        }
      }
    }
    // remaining activation chunks (bounded waits)
    while (ok && a_next < nchunks) {
      const uint64_t t0 = globaltimer();
      const int before = a_next;
      while (a_next == before) {
        try_load_next_a();
        if (a_next != before) break;
        if (*abort_flag || globaltimer() - t0 > kWaitLimitNs) {
          if (!*abort_flag) {
            *abort_flag = 1u;
            if (p.status) atomicOr(p.status, 1u);
          }
          ok = false;
          break;
        }
      }
    }
    if (*abort_flag) {
      // wait (bounded) for the copies still in flight: the last fill of
      // every ring slot and the activation chunks issued
      const int filled = q < R ? q : R;
      for (int s = 0; s < filled; ++s) {
        const int last_q = q - 1 - ((q - 1 - s) % R + R) % R;  // last stage in slot s
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&full[s], (uint32_t)((last_q / R) & 1)) &&
               globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      for (int cc = a_next > 2 ? a_next - 2 : 0; cc < a_next; ++cc) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&afull[cc % p.nb], (uint32_t)((cc / p.nb) & 1)) &&
               globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int gid = lane >> 2, t = lane & 3;
  const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
  // activation row of this lane's B fragments. Lanes past the last row read
  // row M - 1 instead of zeros: they only feed output columns m >= M, which
  // no path stores (and no guard or zeroing is needed per fragment).
  const int arow[2] = {min(gid, p.M - 1), min(8 + gid, p.M - 1)};
  float tot[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) tot[mt][i] = 0.f;
  float own[2][MT][4];  // OWNER: sums of this warp's row blocks warp and warp + NC
#pragma unroll
  for (int o = 0; o < 2; ++o)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) own[o][mt][i] = 0.f;

  auto flush = [&](int rbl) {  // this warp's partial sums of row block rbl -> shared
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = mt * 8 + 2 * t + (i & 1);
        if (m < p.M) red_shared_add(&acc_s[(rbl * 16 + gid + (i >> 1) * 8) * p.M + m], tot[mt][i]);
        tot[mt][i] = 0.f;
      }
  };

  bool ok = true;
  int slot = 0;        // ring slot being read
  uint32_t phase = 0;  // parity of its current fill
  for (int c = 0; c < nchunks; ++c) {
    const int b = c % p.nb;
    const __nv_bfloat16* As = A_s + (size_t)b * p.M * rs;
    float* SAs = SA_s + (size_t)b * gpc * 16;
    if (ok) ok = wait_or_abort(&afull[b], (uint32_t)((c / p.nb) & 1), abort_flag, p.status);
    // per-(activation row, group) sums of the chunk: ones x activations
    if (ok) {
      for (int g = warp; g < gpc; g += kConsumers) {
        float s2[2][MT][4];
#pragma unroll
        for (int kt = 0; kt < 8; ++kt) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint2 bv = *reinterpret_cast<const uint2*>(As + (size_t)arow[mt] * rs + g * G +
                                                             32 * t + 4 * kt);
            if (kt < 2) mma_bf16_first(s2[kt & 1][mt], ones, bv.x, bv.y);
            else mma_bf16(s2[kt & 1][mt], ones, bv.x, bv.y);
          }
        }
        if (gid == 0) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            *reinterpret_cast<float2*>(SAs + g * 16 + mt * 8 + 2 * t) =
                make_float2(s2[0][mt][0] + s2[1][mt][0], s2[0][mt][1] + s2[1][mt][1]);
        }
      }
      if (warp < gpc) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&safull[b]);
      }
    }
    // The chunk's sums are visible once every warp that computes some has
    // arrived. (An mbarrier rather than a barrier of all consumer warps: no
    // warp waits for the others to finish the previous chunk. The sum buffer
    // is free again when its activation buffer is refilled, which waits for
    // every warp's "done" arrival on aempty.)
    if (ok) ok = wait_or_abort(&safull[b], (uint32_t)((c / p.nb) & 1), abort_flag, p.status);

    if constexpr (OWNER) {
      const int rbs = STAGE_TILES / gpc;  // row blocks per stage
      for (int k = 0; ok && k < nst; ++k) {
        if (!wait_or_abort(&full[slot], phase, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const uint8_t* sp = ring + (size_t)slot * STAGE_BYTES;
#pragma unroll
        for (int o = 0; o < 2; ++o) {
          const int rb = warp + o * NC;
          if (rb < nrb && rb / rbs == k) {
            const int base = (rb - k * rbs) * gpc;  // first tile of the row block in the stage
            // two tiles per iteration: their MMA chains are independent and
            // interleave (C5 M = 16: 61.5 -> 60.3 us)
#pragma unroll 2
            for (int j = 0; j < gpc; ++j) {
              const int pos = base + j;
              const uint4 w0 = *reinterpret_cast<const uint4*>(sp + pos * TILE_BYTES + gid * 64 +
                                                               16 * t);
              const uint4 w1 = *reinterpret_cast<const uint4*>(sp + pos * TILE_BYTES +
                                                               (gid + 8) * 64 + 16 * t);
              const float2 sc = *reinterpret_cast<const float2*>(sp + STAGE_TILES * TILE_BYTES +
                                                                 pos * 64 + gid * 8);
              float2 off;
              if constexpr (MODE == 2)
                off = *reinterpret_cast<const float2*>(sp + STAGE_TILES * (TILE_BYTES + 64) +
                                                       pos * 64 + gid * 8);
              else
                off = MODE == 1 ? make_float2(136.f, 136.f) : make_float2(128.f, 128.f);
              const __nv_bfloat16* bg[MT];
#pragma unroll
              for (int mt = 0; mt < MT; ++mt)
                bg[mt] = As + (size_t)arow[mt] * rs + 32 * t + j * G;
              tile_math<MT, MODE>(own[o], w0, w1, sc, off, bg, SAs + j * 16, t);
            }
          }
        }
        __syncwarp();  // every lane is done reading the slot
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == R) {
          slot = 0;
          phase ^= 1u;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&aempty[b]);  // done with this chunk's activations
      continue;
    }

    const __nv_bfloat16* brow[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) brow[mt] = As + (size_t)arow[mt] * rs + 32 * t;
    // this warp's tiles of stage k: i = k * STAGE_TILES + TPW * warp + j, j < TPW,
    // consecutive groups of one row block (gpc is a multiple of 8)
    int rbl = TPW * warp / gpc, gl = TPW * warp - (TPW * warp / gpc) * gpc, cur_rbl = rbl;
    for (int k = 0; ok && k < nst; ++k) {
      if (!wait_or_abort(&full[slot], phase, abort_flag, p.status)) {
        ok = false;
        break;
      }
      const int i0 = k * STAGE_TILES + TPW * warp;
      const int nmine = min(TPW, max(0, items - i0));
      const uint8_t* sp = ring + (size_t)slot * STAGE_BYTES;
      uint4 w0[TPW], w1[TPW];
      float2 sc[TPW], off[TPW];
#pragma unroll
      for (int j = 0; j < TPW; ++j) {
        if (j < nmine) {
          const int pos = TPW * warp + j;
          w0[j] = *reinterpret_cast<const uint4*>(sp + pos * TILE_BYTES + gid * 64 + 16 * t);
          w1[j] = *reinterpret_cast<const uint4*>(sp + pos * TILE_BYTES + (gid + 8) * 64 + 16 * t);
          sc[j] = *reinterpret_cast<const float2*>(sp + STAGE_TILES * TILE_BYTES + pos * 64 +
                                                   gid * 8);
          if constexpr (MODE == 2)
            off[j] = *reinterpret_cast<const float2*>(sp + STAGE_TILES * (TILE_BYTES + 64) +
                                                      pos * 64 + gid * 8);
          else
            off[j] = MODE == 1 ? make_float2(136.f, 136.f) : make_float2(128.f, 128.f);
        }
      }
      __syncwarp();  // every lane has read its part of the slot
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == R) {
        slot = 0;
        phase ^= 1u;
      }
      if (nmine > 0) {
        if (rbl != cur_rbl) {
          flush(cur_rbl);
          cur_rbl = rbl;
        }
#pragma unroll
        for (int j = 0; j < TPW; ++j) {
          if (j < nmine) {
            const __nv_bfloat16* bg[MT];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) bg[mt] = brow[mt] + (gl + j) * G;
            tile_math<MT, MODE>(tot, w0[j], w1[j], sc[j], off[j], bg, SAs + (gl + j) * 16, t);
          }
        }
      }
      gl += STAGE_TILES;
      while (gl >= gpc) {
        gl -= gpc;
        ++rbl;
      }
    }
    if (items > TPW * warp) flush(cur_rbl);
    __syncwarp();
    if (lane == 0) mbar_arrive(&aempty[b]);  // done with this chunk's activations
  }
  if constexpr (OWNER) {
    if (!ok || *abort_flag) return;
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      const int rb = warp + o * NC;
      if (rb >= nrb) continue;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int m = mt * 8 + 2 * t + (i & 1);
          if (m >= p.M) continue;
          const int64_t o_ = (int64_t)m * p.N + (int64_t)(rb0 + rb) * 16 + gid + (i >> 1) * 8;
          const float v = own[o][mt][i];
          if constexpr (OUT == BRC_DTYPE_F32) static_cast<float*>(p.out)[o_] = v;
          else if constexpr (OUT == BRC_DTYPE_BF16)
            static_cast<__nv_bfloat16*>(p.out)[o_] = __float2bfloat16_rn(v);
          else static_cast<__half*>(p.out)[o_] = __float2half_rn(v);
        }
    }
    return;
  }
  consumers_sync<NC>();  // all partial sums are in shared memory
  if (*abort_flag) return;
  const int cols = nrb * 16;
  for (int i = threadIdx.x; i < p.M * cols; i += kConsumers * 32) {
    const int m = i / cols, nl = i - m * cols;
    const float v = acc_s[nl * p.M + m];
    const int64_t o = (int64_t)m * p.N + (int64_t)rb0 * 16 + nl;
    if constexpr (OUT == BRC_DTYPE_F32) static_cast<float*>(p.out)[o] = v;
    else if constexpr (OUT == BRC_DTYPE_BF16)
      static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
    else static_cast<__half*>(p.out)[o] = __float2half_rn(v);
  }
}

// ------------------------------------------------------------------ host
template <int MT, int MODE, int OUT, bool OWNER>
int launch(const Params& p, int grid, size_t smem, cudaStream_t st) {
  constexpr int NC = consumers_for(MT);
  auto kern = k_int4_skinny<MT, MODE, OUT, NC, OWNER>;
  // the opt-in shared-memory size is set once per device (to the maximum)
  static bool configured[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BRC_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSmemLimit));
      if (rc) return rc;
      configured[dev] = true;
    }
  }
  kern<<<grid, threads_for(NC), smem, st>>>(p);
  return check_launch();
}

template <int MT, int MODE, bool OWNER>
int launch_out(int out_dtype, const Params& p, int grid, size_t smem, cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32) return launch<MT, MODE, BRC_DTYPE_F32, OWNER>(p, grid, smem, st);
  if (out_dtype == BRC_DTYPE_BF16)
    return launch<MT, MODE, BRC_DTYPE_BF16, OWNER>(p, grid, smem, st);
  return launch<MT, MODE, BRC_DTYPE_F16, OWNER>(p, grid, smem, st);
}

template <int MT, bool OWNER>
int launch_mode(int mode, int out_dtype, const Params& p, int grid, size_t smem,
                cudaStream_t st) {
  if (mode == 0) return launch_out<MT, 0, OWNER>(out_dtype, p, grid, smem, st);
  if (mode == 1) return launch_out<MT, 1, OWNER>(out_dtype, p, grid, smem, st);
  return launch_out<MT, 2, OWNER>(out_dtype, p, grid, smem, st);
}

// Shared-memory plan for one call: activation chunk and ring depth.
struct Plan {
  int kc, nb, stages;
  Layout L;
};

int plan(int M, int K, int rbmax, Plan& out) {
  const int NC = consumers_for(M <= 8 ? 1 : 2);
  // Activations: the whole K when that leaves room for 4 ring stages, else
  // double-buffered chunks (the largest multiple of 1024 dividing K that
  // does); then as many stages as fit, up to 16.
  auto ring_room = [&](int kc, int nb) -> long {
    const Layout L0 = layout(NC, M, kc, nb, 0, rbmax);
    return (long)kSmemLimit - (long)L0.total;
  };
  const long kStageCost = stage_bytes(NC) + 16;
  int kc = 0, nb = 1;
  for (int cand = K; cand >= 1024; cand -= 1024) {
    if (K % cand) continue;
    const int cnb = cand == K ? 1 : 2;
    if (ring_room(cand, cnb) >= 4 * kStageCost || cand == 1024) {
      kc = cand;
      nb = cnb;
      break;
    }
  }
  if (kc == 0) return BRC_ERR_UNSUPPORTED;
  int stages = (int)(ring_room(kc, nb) / kStageCost);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return BRC_ERR_UNSUPPORTED;
  out.kc = kc;
  out.nb = nb;
  out.stages = stages;
  out.L = layout(NC, M, kc, nb, stages, rbmax);
  return out.L.total <= (uint32_t)kSmemLimit ? BRC_OK : BRC_ERR_UNSUPPORTED;
}

}  // namespace int4gemm
}  // namespace brc

extern "C" int brc_gemm_int4(const void* a_bf16, int M, int K, const uint8_t* w_tiles, int N,
                             int is_signed, int symmetric, const float* scale_tiles,
                             const float* zp_tiles, void* d, int d_dtype, void* stream) {
  using namespace brc::int4gemm;
  if (!a_bf16 || !w_tiles || !scale_tiles || !d) return BRC_ERR_NULL;
  if (!symmetric && !zp_tiles) return BRC_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? BRC_OK : BRC_ERR_SHAPE;
  if (d_dtype != BRC_DTYPE_F32 && d_dtype != BRC_DTYPE_BF16 && d_dtype != BRC_DTYPE_F16)
    return BRC_ERR_DTYPE;
  if (M > 16 || K % 1024 || N % 16 || (!symmetric && is_signed)) return BRC_ERR_UNSUPPORTED;
  if (((uintptr_t)a_bf16 | (uintptr_t)w_tiles | (uintptr_t)scale_tiles |
       (uintptr_t)(zp_tiles ? zp_tiles : scale_tiles)) & 15)
    return BRC_ERR_ALIGN;
  const int n_rb = N / 16;
  int grid = brc::sm_count();
  if (grid > n_rb) grid = n_rb;
  if ((n_rb + grid - 1) / grid > kMaxRb) grid = (n_rb + kMaxRb - 1) / kMaxRb;
  const int rbmax = (n_rb + grid - 1) / grid;
  Plan pl;
  int rc = plan(M, K, rbmax, pl);
  if (rc) return rc;

  Params p{};
  p.a = static_cast<const __nv_bfloat16*>(a_bf16);
  p.w = w_tiles;
  p.sc = scale_tiles;
  p.zp = zp_tiles;
  p.out = d;
  p.M = M;
  p.N = N;
  p.K = K;
  p.kc = pl.kc;
  p.nb = pl.nb;
  p.stages = pl.stages;
  p.rbmax = rbmax;
  p.status = brc::gemm_status_ptr();
  const int mode = symmetric ? (is_signed ? 1 : 0) : 2;
  cudaStream_t st = (cudaStream_t)stream;
  // row-block owners when a stage holds whole row blocks of a chunk (and a
  // warp owns at most two row blocks)
  const int gpc = pl.kc / G;
  const bool owner = (consumers_for(M <= 8 ? 1 : 2) * TPW) % gpc == 0 &&
                     rbmax <= 2 * consumers_for(M <= 8 ? 1 : 2);
  if (owner)
    return M <= 8 ? launch_mode<1, true>(mode, d_dtype, p, grid, pl.L.total, st)
                  : launch_mode<2, true>(mode, d_dtype, p, grid, pl.L.total, st);
  return M <= 8 ? launch_mode<1, false>(mode, d_dtype, p, grid, pl.L.total, st)
                : launch_mode<2, false>(mode, d_dtype, p, grid, pl.L.total, st);
}
