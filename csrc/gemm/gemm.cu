// Persistent warp-specialised tcgen05 GEMM for sm_100a: C = epilogue(A · B^T).
//
//   A: [M, K] bf16, K-major (row-major activations) or MN-major (A = X^T of a
//      row-major X[K, M], used for weight gradients dY^T · X).
//   B: [N, K] bf16, K-major (nn.Linear weights [out, in]) or MN-major
//      (B = W^T of a row-major W[K, N], used for input gradients dY · W).
//   Accumulation in fp32 in tensor memory (TMEM).
//
// Roles (192 threads): warp 0 issues TMA tile loads (128-byte swizzle, no
// multicast) into a STAGES-deep shared-memory ring; warp 1 issues
// tcgen05.mma (M=128, N=BN, K=16) from one elected thread and commits each
// stage back to the producer; warps 2-5 drain the double-buffered TMEM
// accumulator (tcgen05.ld 32x32b) and run the epilogue while the next tile
// accumulates. One CTA per SM walks tiles M-fastest so the CTAs running at
// the same time share B tiles through L2.
//
// Epilogues: bf16 store, fp32 store, fp32 accumulate (C += alpha * acc, for
// gradient accumulation into the flat fp32 buffers), and SwiGLU with two B
// operands (out = silu(A·Bg^T) * (A·Bu^T), bf16).
//
// Stream-K mode (single-B epilogues): when the tile count leaves the last wave
// of the persistent grid mostly idle (e.g. 160 tiles of a 1024 x 5120 output on
// 148 SMs), the tiles x k-blocks iteration space is split evenly over the CTAs.
// CTA c owns the contiguous iterations [start(c), start(c+1)) and walks them
// from the END, so the piece it finishes first is the one that ends mid-tile:
// that piece is stored as an fp32 partial in slot c of a workspace and
// counted on the tile's flag. The piece holding a tile's last k-block is the
// first piece of its owner's range, processed last; its epilogue waits (bounded)
// for the lower-index CTAs that hold the tile's earlier k-blocks, adds their
// partials from the workspace and stores the tile, then clears the flag. Waits
// only ever point at lower-index CTAs, which finished those pieces first.
//
// Grouped launches: up to three problems of one shape and layout (the TimeMix r, k and v projections) share
// the persistent grid, the tile numbering and the stream-K iteration space, each with its own tensor maps and
// output pointer.
//
// 256-row tiles (tuner candidates, store / accumulate / SwiGLU epilogues): the MMA warp issues two M = 128 MMAs
// per k-step into two TMEM accumulators, both reading the same B tile, which halves the B traffic from L2 per
// FLOP (what a CTA pair does with cta_group::2, without a cluster). With 512 accumulator columns the TMEM holds
// one accumulator, so the epilogue of a tile does not overlap the next tile's main loop.
//
// All waits are bounded (sm100.cuh); on timeout the kernel records status 1
// in *status and unwinds, freeing its TMEM.
#include <cuda.h>
#include <algorithm>
#include <map>
#include <vector>
#include <mutex>
#include <atomic>
#include <cstring>
#include <cstdlib>
#include <tuple>
#include "../common/common.cuh"
#include "../common/sm100.cuh"

namespace {

enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_F32_ACCUM = 2, EPI_SWIGLU = 3, EPI_ATOMIC_T = 4, EPI_NMSE = 5 };

constexpr int BM = 128, BK = 64, STAGES = 4, THREADS = 192;
constexpr int MN_CHUNK_BYTES = 64 * BK * 2;  // one 64-wide MN-major chunk: BK rows x 128 B

// MT = 2: a 256-row tile per CTA as two M = 128 MMAs per k-step that read the same B tile in shared memory, so each
// B tile crosses L2 half as often per FLOP (the single-CTA counterpart of a CTA-pair tile; no cluster is needed).
template <int BN, bool A_MN, bool B_MN, int EPI, int MT = 1>
struct Cfg {
  static_assert(MT == 1 || (MT == 2 && EPI != EPI_ATOMIC_T && EPI != EPI_NMSE),
                "256-row tiles take the store, accumulate and SwiGLU epilogues");
  static constexpr int NB = EPI == EPI_SWIGLU ? 2 : 1;
  static constexpr int ROWS = MT * BM;  // tile rows
  static constexpr int A_HALF = BM * BK * 2;
  static constexpr int A_BYTES = MT * A_HALF;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + NB * B_BYTES;
  // Pipeline depth: 4 stages for the compute-bound tiles (3 where a stage is over 50 KB: 256-row tiles of 192+
  // columns and the 256-row SwiGLU tile);
  // the skinny split-K tiles (weight streaming for decode) are memory-bound and keep 8 stages of 20 KB in flight.
  static constexpr int ST = EPI == EPI_ATOMIC_T ? 8 : STAGES * STAGE_BYTES <= 200 * 1024 ? STAGES : 3;
  static constexpr int ACC_COLS = NB * BN * MT;
  // accumulators: two (the epilogue drains one while the next tile accumulates) when they fit in the 512 TMEM
  // columns, else one; the column count is rounded up to the power of two tcgen05.alloc takes
  static constexpr int NACC = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = NACC * ACC_COLS <= 64 ? 64 : NACC * ACC_COLS <= 128 ? 128
                                   : NACC * ACC_COLS <= 256 ? 256 : 512;
  static constexpr uint32_t IDESC = sm100::idesc_bf16(BM, BN, A_MN, B_MN);
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = ST * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(TMEM_COLS == 64 || TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512,
                "TMEM columns must be a power of 2 (>= 32)");
};

// Operand tensor maps. A group of G <= MAX_GROUPS problems of one shape and layout (e.g. the r, k and v projections
// of a TimeMix layer) runs as one launch: problem g reads a[g] and b[g] and writes C[g]. The SwiGLU epilogue (G = 1)
// reads its two B operands from b[0] (gate) and b[1] (up).
constexpr int MAX_GROUPS = 3;
struct GemmMaps {
  CUtensorMap a[MAX_GROUPS];
  CUtensorMap b[MAX_GROUPS];
};

struct GemmArgs {
  int M, N, K;
  void* C[MAX_GROUPS];
  long ldc;
  int groups;  // problems in the launch; tiles are numbered M-fastest, then N, then problem, then split
  int tiles_m, tiles_n;
  int splits, kchunk;  // split-K: tile t covers k-blocks [ks * kchunk, (ks + 1) * kchunk), ks = t / (tiles_m * tiles_n)
  float alpha;
  int* status;
  // stream-K (sk = 1): CTA c owns iterations [c q + min(c, rem), (c + 1) q + min(c + 1, rem)) of tiles x k-blocks
  int sk, q, rem;
  // parallel split-K (splitp = S > 1): CTA c computes k-part c % S of tile c / S, publishes it as an fp32 partial,
  // and after all S parts of the tile are published reduces rows [part BM / S, (part + 1) BM / S) of the tile
  int splitp;
  float* ws;   // fp32 partial tiles, one BM x BN slot per CTA
  int* flags;  // per tile: partial warps published (4 per contributing CTA); reset by the tile's final CTA
  // EPI_NMSE: target [M, N] bf16 (row stride N) and per-row sums [M, 4] = {sum t^2 (given), sum (p-t)^2, sum p^2,
  // sum p t}; C receives d loss / d p = 2 (p - t) / (N max(mean t^2, eps)) in bf16.
  const __nv_bfloat16* target;
  float* rowsum;
  float eps;
};

// Work of one CTA: whole (or split-K) tiles strided over the grid, or its stream-K pieces, last first.
struct WorkIter {
  int next_tile, total, stride, per_split, kchunk, kblocks;
  bool sk;
  int lo, cur;  // stream-K range still to walk: [lo, cur)
  __device__ WorkIter(const GemmArgs& a, int kblocks_) {
    kblocks = kblocks_;
    per_split = a.tiles_m * a.tiles_n * a.groups;
    total = per_split * a.splits;
    next_tile = blockIdx.x;
    stride = gridDim.x;
    kchunk = a.kchunk;
    sk = a.sk != 0;
    const int c = blockIdx.x;
    lo = c * a.q + min(c, a.rem);
    cur = (c + 1) * a.q + min(c + 1, a.rem);
    splitp = a.splitp;
    sp_done = 0;
  }
  int splitp, sp_done;
  __device__ bool next(int& tile, int& k0, int& k1) {
    if (splitp > 1) {
      if (sp_done) return false;
      sp_done = 1;
      const int part = blockIdx.x % splitp;
      tile = blockIdx.x / splitp;
      k0 = (int)((long)kblocks * part / splitp);
      k1 = (int)((long)kblocks * (part + 1) / splitp);
      return true;
    }
    if (sk) {
      if (cur <= lo) return false;
      tile = (cur - 1) / kblocks;
      const int ts = tile * kblocks, p0 = max(lo, ts);
      k0 = p0 - ts;
      k1 = cur - ts;
      cur = p0;
      return true;
    }
    if (next_tile >= total) return false;
    tile = next_tile;
    next_tile += stride;
    k0 = (tile / per_split) * kchunk;
    k1 = min(kblocks, k0 + kchunk);
    return true;
  }
};

// Stream-K owner of iteration i (inverse of the range formula above).
__device__ __forceinline__ int sk_owner(int i, int q, int rem) {
  const int big = rem * (q + 1);
  return i < big ? i / (q + 1) : rem + (i - big) / q;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Partial-tile slot layout: for 32-column chunk c and float4 q of a row, the 128 rows are contiguous, so a
// warp's 32 rows move as one 512-byte run.
__device__ __forceinline__ float4* sk_slot(float* ws, int slot, int bn, int c, int q, int row, int rows = BM) {
  return reinterpret_cast<float4*>(ws) + (long)slot * rows * (bn / 4) + ((long)(c * 8 + q) * rows + row);
}

__device__ __forceinline__ void store_row(float (&v)[32], int epi, void* C, long ldc, int row, int col, int N,
                                          float alpha) {
  if (epi == EPI_BF16 || epi == EPI_SWIGLU) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(C) + (long)row * ldc + col;
    if (col + 32 <= N && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
      uint4* dst = reinterpret_cast<uint4*>(out);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __nv_bfloat162 p0 = __floats2bfloat162_rn(v[8 * q + 0], v[8 * q + 1]);
        __nv_bfloat162 p1 = __floats2bfloat162_rn(v[8 * q + 2], v[8 * q + 3]);
        __nv_bfloat162 p2 = __floats2bfloat162_rn(v[8 * q + 4], v[8 * q + 5]);
        __nv_bfloat162 p3 = __floats2bfloat162_rn(v[8 * q + 6], v[8 * q + 7]);
        uint4 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&p0);
        pk.y = *reinterpret_cast<uint32_t*>(&p1);
        pk.z = *reinterpret_cast<uint32_t*>(&p2);
        pk.w = *reinterpret_cast<uint32_t*>(&p3);
        dst[q] = pk;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < N) out[i] = __float2bfloat16_rn(v[i]);
    }
    return;
  }
  float* out = reinterpret_cast<float*>(C) + (long)row * ldc + col;
  const bool vec = col + 32 <= N && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  if (epi == EPI_F32) {
    if (vec) {
      float4* dst = reinterpret_cast<float4*>(out);
#pragma unroll
      for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < N) out[i] = v[i];
    }
  } else if (epi == EPI_ATOMIC_T) {  // transposed fp32 partial sums: C[col + i][row] += v[i] (split-K)
    float* base = reinterpret_cast<float*>(C) + row;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col + i < N) atomicAdd(base + (long)(col + i) * ldc, v[i]);
  } else {  // EPI_F32_ACCUM
    if (vec) {
      float4* dst = reinterpret_cast<float4*>(out);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 o = dst[q];
        o.x += alpha * v[4 * q]; o.y += alpha * v[4 * q + 1]; o.z += alpha * v[4 * q + 2]; o.w += alpha * v[4 * q + 3];
        dst[q] = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < N) out[i] += alpha * v[i];
    }
  }
}

// Distillation-loss epilogue for one row's 32 columns: dpred to C, partial sums of (p-t)^2, p^2, p t.
__device__ __forceinline__ void loss_row(const float (&v)[32], const GemmArgs& a, int row, int col, float& se,
                                         float& pp, float& pt) {
  const float tt = a.rowsum[4 * (long)row];
  const float k = 2.f / (a.N * fmaxf(tt / a.N, a.eps));
  const __nv_bfloat16* trow = a.target + (long)row * a.N + col;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.C[0]) + (long)row * a.ldc + col;
  if (col + 32 <= a.N && ((reinterpret_cast<uintptr_t>(trow) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float t[8], d[8];
      rt::unpack8(__ldg(reinterpret_cast<const uint4*>(trow) + q), t);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float p = v[8 * q + u], e = p - t[u];
        se += e * e;
        pp += p * p;
        pt += p * t[u];
        d[u] = k * e;
      }
      reinterpret_cast<uint4*>(out)[q] = rt::pack8(d);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (col + i < a.N) {
        const float p = v[i], t = __bfloat162float(trow[i]), e = p - t;
        se += e * e;
        pp += p * p;
        pt += p * t;
        out[i] = __float2bfloat16_rn(k * e);
      }
    }
  }
}

// Problem, row tile and column tile of a tile index (split index excluded).
__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& g, int& tm, int& tn) {
  const int per_problem = a.tiles_m * a.tiles_n;
  const int t = tile % (per_problem * a.groups);
  g = t / per_problem;
  tm = t % a.tiles_m;
  tn = (t % per_problem) / a.tiles_m;
}

// Set by a launch without a status word whose bounded wait gave up (read and cleared by rt_gemm_fault).
__device__ int gemm_fault_word = 0;

template <int BN, bool A_MN, bool B_MN, int EPI, int MT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ GemmMaps maps, const GemmArgs args) {
  using C_ = Cfg<BN, A_MN, B_MN, EPI, MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = sm100::align_smem_1024(smem_raw);
  constexpr int ST = C_::ST;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST * C_::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* tfull = bars + 2 * ST;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  constexpr int NACC = C_::NACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NACC; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 128);
    }
    sm100::mbar_init(drain, 1);
    *abort = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int g = 0; g < args.groups; ++g) {
      sm100::prefetch_tmap(&maps.a[g]);
      sm100::prefetch_tmap(&maps.b[g]);
    }
    if (C_::NB == 2) sm100::prefetch_tmap(&maps.b[1]);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C_::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (sm100::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      WorkIter work(args, kblocks);
      int tile, k0, k1;
      while (!*abort && work.next(tile, k0, k1)) {
        int g, tm, tn;
        tile_coords(args, tile, g, tm, tn);
        const CUtensorMap* ta = &maps.a[g];
        for (int kb = k0; kb < k1; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1, abort)) break;
          uint8_t* a_dst = smem + stage * C_::STAGE_BYTES;
          sm100::mbar_expect_tx(&full[stage], C_::STAGE_BYTES);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            uint8_t* a_half = a_dst + mt * C_::A_HALF;
            const int m0 = tm * C_::ROWS + mt * BM;
            if (!A_MN) {
              sm100::tma_load_2d(a_half, ta, &full[stage], kb * BK, m0);
            } else {
              sm100::tma_load_2d(a_half, ta, &full[stage], m0, kb * BK);
              sm100::tma_load_2d(a_half + MN_CHUNK_BYTES, ta, &full[stage], m0 + 64, kb * BK);
            }
          }
#pragma unroll
          for (int j = 0; j < C_::NB; ++j) {
            uint8_t* b_dst = a_dst + C_::A_BYTES + j * C_::B_BYTES;
            const CUtensorMap* tb = &maps.b[C_::NB == 2 ? j : g];
            if (!B_MN) {
              sm100::tma_load_2d(b_dst, tb, &full[stage], kb * BK, tn * BN);
            } else {
#pragma unroll
              for (int c = 0; c < BN / 64; ++c)
                sm100::tma_load_2d(b_dst + c * MN_CHUNK_BYTES, tb, &full[stage], tn * BN + c * 64, kb * BK);
            }
          }
          ++issued;
          if (++stage == ST) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: every issued stage must have been consumed before shared memory goes away.
      (void)issued;
      for (int s = 0; s < ST; ++s) {
        if (!sm100::mbar_wait_bounded(&empty[stage], phase ^ 1)) break;
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (sm100::elect_one()) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      WorkIter work(args, kblocks);
      int tile, k0, k1;
      while (!*abort && work.next(tile, k0, k1)) {
        if (!sm100::mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) break;
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C_::ACC_COLS;
        bool ok = true;
        for (int kb = k0; kb < k1; ++kb) {
          if (!sm100::mbar_wait(&full[stage], phase, abort)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(smem + stage * C_::STAGE_BYTES);
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint32_t a_half = a_base + mt * C_::A_HALF;
              const uint64_t adesc = A_MN ? sm100::smem_desc(a_half + ks * 2048, MN_CHUNK_BYTES, 1024)
                                          : sm100::smem_desc(a_half + ks * 32, 16, 1024);
#pragma unroll
              for (int j = 0; j < C_::NB; ++j) {
                const uint32_t b_base = a_base + C_::A_BYTES + j * C_::B_BYTES;
                const uint64_t bdesc = B_MN ? sm100::smem_desc(b_base + ks * 2048, MN_CHUNK_BYTES, 1024)
                                            : sm100::smem_desc(b_base + ks * 32, 16, 1024);
                sm100::mma_bf16(d_tmem + (mt * C_::NB + j) * BN, adesc, bdesc, C_::IDESC, (kb != k0) || (ks != 0));
              }
            }
          }
          sm100::mma_commit(&empty[stage]);
          if (++stage == ST) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        sm100::mma_commit(&tfull[acc]);
        if (++acc == NACC) { acc = 0; acc_phase ^= 1; }
      }
      sm100::mma_commit(drain);
      sm100::mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    WorkIter work(args, kblocks);
    int tile, k0, k1;
    while (!*abort && work.next(tile, k0, k1)) {
      int g, tm, tn;
      tile_coords(args, tile, g, tm, tn);
      void* const Cg = args.C[g];
      if (!sm100::mbar_wait(&tfull[acc], acc_phase, abort)) break;
      sm100::tc_fence_after();
      const int row = tm * C_::ROWS + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * C_::ACC_COLS;
      if (MT == 1 && C_::NB == 1 && EPI != EPI_NMSE && EPI != EPI_ATOMIC_T && args.splitp > 1) {
        // ---- parallel split-K: publish this part, wait for the tile's other parts, reduce this CTA's row band
        const int S = args.splitp, part = blockIdx.x % S;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          sm100::tmem_ld32(t_row + c * 32, v);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(sk_slot(args.ws, blockIdx.x, BN, c, q, row_in_tile),
                   make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
        }
        sm100::tc_fence_before();
        sm100::mbar_arrive(&tempty[acc]);
        if (++acc == NACC) { acc = 0; acc_phase ^= 1; }
        int* arrive = args.flags + 4 * tile;
        int* depart = arrive + 1;
        __threadfence();
        __syncwarp();
        bool ok = true;
        if (lane == 0) {
          atomicAdd(arrive, 1);
          const uint64_t t0 = sm100::globaltimer();
          for (uint32_t spin = 0; ld_acquire_gpu(arrive) < 4 * S; ++spin) {
            if ((spin & 63u) == 63u && (sm100::globaltimer() - t0 > RT_WAIT_LIMIT_NS || *abort)) {
              ok = false;
              break;
            }
          }
          if (!ok) *abort = 1;
        }
        __syncwarp();
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        // rows [r0, r1) of the tile, all BN columns, summed over the S parts' slots (4 warps share the band)
        const int r0 = BM * part / S, r1 = BM * (part + 1) / S, rows = r1 - r0;
        const int etid = threadIdx.x - 64;  // 0..127 over the epilogue warps
        for (int e = etid; e < rows * (BN / 4); e += 128) {
          const int r = r0 + e % rows, cq = e / rows;
          float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int s2 = 0; s2 < S; ++s2) {
            const float4 p4 = __ldcg(sk_slot(args.ws, tile * S + s2, BN, cq >> 3, cq & 7, r));
            acc4.x += p4.x; acc4.y += p4.y; acc4.z += p4.z; acc4.w += p4.w;
          }
          const int grow = tm * BM + r, gcol = tn * BN + 4 * cq;
          if (grow >= args.M || gcol >= args.N) continue;
          const float vals[4] = {acc4.x, acc4.y, acc4.z, acc4.w};
          if (EPI == EPI_BF16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(Cg) + (long)grow * args.ldc + gcol;
            if (gcol + 4 <= args.N && (reinterpret_cast<uintptr_t>(o) & 7) == 0) {
              __nv_bfloat162 a2 = __floats2bfloat162_rn(vals[0], vals[1]), b2 = __floats2bfloat162_rn(vals[2], vals[3]);
              uint2 pk;
              pk.x = *reinterpret_cast<uint32_t*>(&a2);
              pk.y = *reinterpret_cast<uint32_t*>(&b2);
              *reinterpret_cast<uint2*>(o) = pk;
            } else {
              for (int u = 0; u < 4 && gcol + u < args.N; ++u) o[u] = __float2bfloat16_rn(vals[u]);
            }
          } else {
            float* o = reinterpret_cast<float*>(Cg) + (long)grow * args.ldc + gcol;
            for (int u = 0; u < 4 && gcol + u < args.N; ++u) {
              if (EPI == EPI_F32) o[u] = vals[u];
              else o[u] += args.alpha * vals[u];
            }
          }
        }
        __syncwarp();
        if (lane == 0 && atomicAdd(depart, 1) == 4 * S - 1) {  // last warp out: every wait has passed
          *arrive = 0;
          *depart = 0;
        }
        continue;
      }
      // stream-K roles of this piece (uniform over the warp; each warp syncs on its own)
      const bool partial = C_::NB == 1 && args.sk && k1 < kblocks;          // ends mid-tile: publish fp32 partial
      const bool fixup = C_::NB == 1 && args.sk && k1 == kblocks && k0 > 0;  // final piece: add earlier partials
      int first_slot = 0;
      int* flag = args.flags + 4 * tile + quarter;  // one counter per row quarter: warps sync pairwise
      float se = 0.f, pp = 0.f, pt = 0.f;           // EPI_NMSE row sums over this tile's columns
      if (fixup) {
        first_slot = sk_owner(tile * kblocks, args.q, args.rem);
        const int need = (int)blockIdx.x - first_slot;
        bool ok = true;
        if (lane == 0) {
          const uint64_t t0 = sm100::globaltimer();
          for (uint32_t spin = 0; ld_acquire_gpu(flag) < need; ++spin) {
            if ((spin & 63u) == 63u && (sm100::globaltimer() - t0 > RT_WAIT_LIMIT_NS || *abort)) {
              ok = false;
              break;
            }
          }
          if (!ok) *abort = 1;
        }
        __syncwarp();
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      }
#pragma unroll 1
      for (int cc = 0; cc < MT * (BN / 32); ++cc) {  // MT = 2: rows 128..255 of the tile sit BN columns further
        const int mt = cc / (BN / 32), c = cc % (BN / 32);
        const int srow = mt * BM + row_in_tile, grow = row + mt * BM;
        float v[32];
        const uint32_t t_half = t_row + mt * C_::NB * BN;  // this row half's accumulator (gate, then up for SwiGLU)
        sm100::tmem_ld32(t_half + c * 32, v);
        if (EPI == EPI_SWIGLU) {
          float u[32];
          sm100::tmem_ld32(t_half + BN + c * 32, u);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = rt::siluf_(v[i]) * u[i];
        } else {
          sm100::tmem_wait_ld();
        }
        if (partial) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(sk_slot(args.ws, blockIdx.x, BN, c, q, srow, C_::ROWS),
                   make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
          continue;
        }
        if (fixup) {
          for (int slot = first_slot; slot < (int)blockIdx.x; ++slot) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 p = __ldcg(sk_slot(args.ws, slot, BN, c, q, srow, C_::ROWS));
              v[4 * q] += p.x; v[4 * q + 1] += p.y; v[4 * q + 2] += p.z; v[4 * q + 3] += p.w;
            }
          }
        }
        if (grow < args.M) {
          if (EPI == EPI_NMSE)
            loss_row(v, args, grow, tn * BN + c * 32, se, pp, pt);
          else
            store_row(v, EPI, Cg, args.ldc, grow, tn * BN + c * 32, args.N, args.alpha);
        }
      }
      if (EPI == EPI_NMSE && !partial && row < args.M) {
        atomicAdd(args.rowsum + 4 * (long)row + 1, se);
        atomicAdd(args.rowsum + 4 * (long)row + 2, pp);
        atomicAdd(args.rowsum + 4 * (long)row + 3, pt);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tempty[acc]);
      if (++acc == NACC) { acc = 0; acc_phase ^= 1; }
      if (partial) {  // publish this warp's 32 rows (both halves of a 256-row tile)
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(flag, 1);
      } else if (fixup && lane == 0) {
        *flag = 0;  // all contributions to this quarter arrived and were read; the next launch is stream-ordered
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort) atomicExch(args.status ? args.status : &gemm_fault_word, 1);
}

// The driver's tensor-map encoder, resolved through the runtime so the extension does not link libcuda
// (it must import on machines without a driver).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

bool make_tmap(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
               uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn encode = encode_fn();
  if (!encode) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms_cached() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

// Stream-K workspace of one device and issue lane: a 256 x 256 fp32 partial slot per SM (the widest tile) and 4
// counters per tile. Allocated on the first stream-K launch of the lane outside stream capture and kept (graphs
// hold its address); the counters are zeroed once and every launch leaves them zero again. Launches that use one
// workspace therefore must not run concurrently: a lane is a sequence of GEMMs issued in order on one stream (the
// teacher's forward is lane 0, the students' micro-steps lane 1 when they run beside it), and the host thread
// selects the lane of its next launches with rt_gemm_set_lane.
constexpr int SK_MAX_FLAGS = 4 * 32768;
constexpr int SK_LANES = 2;
struct SkWorkspace {
  float* ws = nullptr;
  int* flags = nullptr;
};
std::map<std::pair<int, int>, SkWorkspace> g_sk_spaces;  // (device, lane)
std::mutex g_sk_mutex;
thread_local int g_lane = 0;
// Set while GEMMs of two lanes may run at the same time. Parallel split-K (whose S parts wait for each other and
// so need all of them resident at once) then runs as stream-K, whose waits only point at lower-index CTAs that
// were dispatched earlier: two concurrent GEMMs can delay each other's CTAs but never wait on each other.
std::atomic<bool> g_concurrent{false};
SkWorkspace* sk_workspace(cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_sk_mutex);
  SkWorkspace& w = g_sk_spaces[{dev, g_lane}];
  if (w.ws) return &w;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return nullptr;
  float* ws = nullptr;
  int* flags = nullptr;
  if (cudaMalloc(&ws, (size_t)num_sms_cached() * 2 * BM * 256 * sizeof(float)) != cudaSuccess) return nullptr;
  if (cudaMalloc(&flags, SK_MAX_FLAGS * sizeof(int)) != cudaSuccess ||
      cudaMemsetAsync(flags, 0, SK_MAX_FLAGS * sizeof(int), stream) != cudaSuccess) {
    cudaFree(ws);
    return nullptr;
  }
  w.ws = ws;
  w.flags = flags;
  return &w;
}

struct LossArgs {
  const void* target = nullptr;
  float* rowsum = nullptr;
  float eps = 0.f;
};

// The problems of one launch: G of the same shape and layouts (A[g] . B[g]^T -> C[g]); B1 is the SwiGLU up operand.
struct Prob {
  int G = 1;
  const void* A[MAX_GROUPS] = {};
  const void* B[MAX_GROUPS] = {};
  const void* B1 = nullptr;
  void* C[MAX_GROUPS] = {};
  long lda = 0, ldb = 0, ldc = 0;
  int M = 0, N = 0, K = 0;
};

Prob single(const void* A, long lda, const void* B, long ldb, void* C, long ldc, int M, int N, int K) {
  Prob p;
  p.A[0] = A;
  p.B[0] = B;
  p.C[0] = C;
  p.lda = lda; p.ldb = ldb; p.ldc = ldc;
  p.M = M; p.N = N; p.K = K;
  return p;
}

// cudaFuncSetAttribute once per device for the kernel instantiation that owns `done` (it is a per-device attribute;
// the host cost of repeating it on every launch showed on the eagerly issued short-chunk student steps).
template <typename Kern>
cudaError_t set_smem_once(std::atomic<uint64_t>& done, Kern kern, int bytes) {
  int dev = 0;
  RT_CUDA_CHECK(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? 1ull << dev : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  RT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return cudaSuccess;
}

template <int BN, bool A_MN, bool B_MN, int EPI, int MT = 1>
cudaError_t launch(const Prob& p, float alpha, int* status, cudaStream_t stream, int splits = 1, bool sk = false,
                   LossArgs loss = LossArgs(), int splitp = 0) {
  using C_ = Cfg<BN, A_MN, B_MN, EPI, MT>;
  if (p.G < 1 || p.G > MAX_GROUPS || (C_::NB == 2 && p.G != 1)) return cudaErrorInvalidValue;
  const int M = p.M, N = p.N, K = p.K;
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool ok = true;
  for (int g = 0; g < p.G && ok; ++g) {
    ok = A_MN ? make_tmap(&maps.a[g], p.A[g], M, K, p.lda * 2, 64, BK) : make_tmap(&maps.a[g], p.A[g], K, M, p.lda * 2, BK, BM);
    ok = ok && (B_MN ? make_tmap(&maps.b[g], p.B[g], N, K, p.ldb * 2, 64, BK)
                     : make_tmap(&maps.b[g], p.B[g], K, N, p.ldb * 2, BK, BN));
  }
  if (C_::NB == 2)
    ok = ok && (B_MN ? make_tmap(&maps.b[1], p.B1, N, K, p.ldb * 2, 64, BK)
                     : make_tmap(&maps.b[1], p.B1, K, N, p.ldb * 2, BK, BN));
  if (!ok) return cudaErrorInvalidValue;
  GemmArgs args;
  args.M = M; args.N = N; args.K = K; args.ldc = p.ldc; args.alpha = alpha; args.status = status;
  args.groups = p.G;
  for (int g = 0; g < MAX_GROUPS; ++g) args.C[g] = g < p.G ? p.C[g] : p.C[0];
  args.tiles_m = (M + C_::ROWS - 1) / C_::ROWS;
  args.tiles_n = (N + BN - 1) / BN;
  args.splits = splits;
  args.kchunk = ((K + BK - 1) / BK + splits - 1) / splits;
  const int tiles = args.tiles_m * args.tiles_n * p.G;
  const int total = tiles * splits;
  args.sk = 0; args.q = 0; args.rem = 0; args.ws = nullptr; args.flags = nullptr; args.splitp = 0;
  args.target = static_cast<const __nv_bfloat16*>(loss.target);
  args.rowsum = loss.rowsum;
  args.eps = loss.eps;
  int grid = total < num_sms_cached() ? total : num_sms_cached();
  if (splitp > 1 && g_concurrent.load(std::memory_order_relaxed)) {  // see g_concurrent
    splitp = 0;
    sk = true;
  }
  if (splitp > 1 && MT == 1 && C_::NB == 1 && splits == 1 && EPI != EPI_ATOMIC_T && EPI != EPI_NMSE) {
    const int kb = (K + BK - 1) / BK;
    int S = splitp;
    while (S > 1 && (tiles * S > num_sms_cached() || kb < 2 * S)) --S;  // co-resident CTAs, >= 2 k-blocks each
    SkWorkspace* w = S > 1 && 4L * tiles <= SK_MAX_FLAGS ? sk_workspace(stream) : nullptr;
    if (w) {
      grid = tiles * S;
      args.splitp = S;
      args.ws = w->ws;
      args.flags = w->flags;
    }
  } else if (sk && C_::NB == 1 && splits == 1 && EPI != EPI_ATOMIC_T) {
    const long iters = (long)tiles * ((K + BK - 1) / BK);
    SkWorkspace* w = 4L * tiles <= SK_MAX_FLAGS && iters >= num_sms_cached() && iters < (1L << 30)
                         ? sk_workspace(stream) : nullptr;
    if (w) {
      grid = num_sms_cached();
      args.sk = 1;
      args.q = (int)(iters / grid);
      args.rem = (int)(iters % grid);
      args.ws = w->ws;
      args.flags = w->flags;
    }
  }
  auto kern = gemm_kernel<BN, A_MN, B_MN, EPI, MT>;
  static std::atomic<uint64_t> smem_set{0};  // one per instantiation of this launcher, i.e. per kernel
  RT_CUDA_CHECK(set_smem_once(smem_set, kern, C_::SMEM_BYTES));
  kern<<<grid, THREADS, C_::SMEM_BYTES, stream>>>(maps, args);
  return cudaGetLastError();
}

// Tile width: the one whose tile count fills the persistent grid best (fraction of the last wave that is
// busy), preferring wider tiles (less L2 traffic per FLOP) when two are within 3%. Widths that are not a
// multiple of 64 need a K-major B operand.
int pick_bn(int M, int N, int G, bool swiglu, bool b_mn) {
  if (swiglu) return 128;
  const int sms = num_sms_cached();
  const long tm = (M + BM - 1) / BM;
  int best = 64;
  double best_eff = -1.0;
  for (int bn : {256, 224, 192, 160, 128, 64}) {
    if (b_mn && bn % 64) continue;
    if (N < bn / 2 && bn != 64) continue;
    const long tiles = tm * ((N + bn - 1) / bn) * G;
    const long waves = (tiles + sms - 1) / sms;
    // useful fraction: filled slots, and the padding of the last (partial) column tile
    const double fill = (double)tiles / (double)(waves * sms);
    const double pad = (double)N / (double)(((N + bn - 1) / bn) * bn);
    const double eff = fill * pad * (bn >= 128 ? 1.0 : 0.85);  // narrow tiles: lower MMA and L2 efficiency
    if (eff > best_eff * 1.03) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}

// Tile choice: width bn, plus SK_FLAG for the stream-K schedule and M2_FLAG for 256-row tiles (widths 256 and 128,
// store and accumulate epilogues).
constexpr int SK_FLAG = 1 << 16;
constexpr int M2_FLAG = 1 << 17;
constexpr int SP_SHIFT = 20;  // choice bits 20..27: parallel split-K factor S (0 = off)

template <bool A_MN, bool B_MN, int EPI>
cudaError_t dispatch_bn(int choice, const Prob& p, float alpha, int* status, cudaStream_t s) {
  const int bn = choice & (SK_FLAG - 1);
  const bool sk = (choice & SK_FLAG) != 0;
  const int sp = (choice >> SP_SHIFT) & 255;
  if (choice & M2_FLAG) {
    if (bn == 256) return launch<256, A_MN, B_MN, EPI, 2>(p, alpha, status, s, 1, sk);
    if (bn == 128) return launch<128, A_MN, B_MN, EPI, 2>(p, alpha, status, s, 1, sk);
    return cudaErrorInvalidValue;
  }
#define RT_L(W) return launch<W, A_MN, B_MN, EPI>(p, alpha, status, s, 1, sk, LossArgs(), sp)
  if (bn == 256) RT_L(256);
  if (bn == 192) RT_L(192);
  if (bn == 128) RT_L(128);
  if constexpr (!B_MN) {
    if (bn == 224) RT_L(224);
    if (bn == 160) RT_L(160);
  }
  RT_L(64);
#undef RT_L
}

cudaError_t gemm_with_bn(int choice, const Prob& p, int a_mn, int b_mn, int epi, float alpha, int* status,
                         cudaStream_t stream);

// Tile width per problem shape, measured once: the first call of a shape with a store epilogue (outside stream
// capture) runs every candidate width on the real operands and keeps the fastest (every width computes each
// output with the same MMA sequence over K, so the result does not depend on the choice). Accumulating calls
// and calls under capture use the measured width of the shape when known, else the wave-fill estimate.
struct TileKey {
  int M, N, K, a_mn, b_mn, G;
  bool operator<(const TileKey& o) const {
    return std::tie(M, N, K, a_mn, b_mn, G) < std::tie(o.M, o.N, o.K, o.a_mn, o.b_mn, o.G);
  }
};
std::map<TileKey, int>& tile_cache() {
  static std::map<TileKey, int> cache;
  return cache;
}
std::mutex& tile_mutex() {
  static std::mutex m;
  return m;
}

// 256-row tiles among the measured candidates (THESEUS_GEMM_M2=0 leaves them out, for comparisons).
bool m2_enabled() {
  static const bool on = [] {
    const char* e = getenv("THESEUS_GEMM_M2");
    return !(e && e[0] == '0');
  }();
  return on;
}

int measured_bn(const TileKey& key, const Prob& p, int epi, float alpha, int* status, cudaStream_t stream) {
  {
    std::lock_guard<std::mutex> lock(tile_mutex());
    auto it = tile_cache().find(key);
    if (it != tile_cache().end()) return it->second;
    // A shorter chunk of a measured GEMM: same N and layouts, fewer token rows (K-major A: M is the token count)
    // or a shallower K (MN-major A, weight gradients: K is the token count), at most 8x smaller. Reuse the choice
    // of the nearest larger measured bucket instead of timing again in the middle of training.
    // Further than 8x from every measured bucket of the shape, the wave-fill estimate is used (still no timing).
    int best = -1;
    long best_size = 0;
    bool larger_known = false;
    for (const auto& [k, choice] : tile_cache()) {
      if (k.N != key.N || k.a_mn != key.a_mn || k.b_mn != key.b_mn || k.G != key.G) continue;
      const bool rows_any = !key.a_mn && k.K == key.K && k.M > key.M;
      const bool depth_any = key.a_mn && k.M == key.M && k.K > key.K;
      larger_known = larger_known || rows_any || depth_any;
      const bool rows = rows_any && k.M <= 8 * key.M;
      const bool depth = depth_any && k.K <= 8 * key.K;
      const long size = (long)k.M * k.K;
      if ((rows || depth) && (best < 0 || size < best_size)) {
        best = choice;
        best_size = size;
      }
    }
    if (best < 0 && larger_known) best = pick_bn(key.M, key.N, key.G, false, key.b_mn != 0);
    if (best >= 0) {
      tile_cache()[key] = best;
      return best;
    }
  }
  const int guess = pick_bn(key.M, key.N, key.G, false, key.b_mn != 0);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (epi == EPI_F32_ACCUM || epi == EPI_NMSE || cudaStreamIsCapturing(stream, &cap) != cudaSuccess ||
      cap != cudaStreamCaptureStatusNone)
    return guess;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return guess;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return guess;
  }
  int best = guess;
  float best_ms = 1e30f;
  const long kblocks = (key.K + BK - 1) / BK;
  std::vector<int> choices = {256, 224, 192, 160, 128, 64, 256 | SK_FLAG, 224 | SK_FLAG, 192 | SK_FLAG, 128 | SK_FLAG};
  if (key.M >= 2 * BM && epi != EPI_NMSE && m2_enabled())
    for (int c : {256 | M2_FLAG, 128 | M2_FLAG, 256 | M2_FLAG | SK_FLAG, 128 | M2_FLAG | SK_FLAG}) choices.push_back(c);
  {  // parallel split-K where the tiles fill under half of the SMs and K is deep
    const int sms = num_sms_cached();
    for (int bn : {64, 128, 192, 256}) {
      const long tiles = (long)((key.M + BM - 1) / BM) * ((key.N + bn - 1) / bn) * key.G;
      if (tiles * 2 > sms || (key.N < bn / 2 && bn != 64) || (key.b_mn && bn % 64)) continue;
      const long smax = std::min<long>({sms / tiles, kblocks / 2, 255});
      for (long S : {smax, smax / 2})
        if (S >= 2) choices.push_back(bn | (int)(S << SP_SHIFT));
    }
  }
  for (int choice : choices) {
    const int bn = choice & (SK_FLAG - 1);
    if (key.b_mn && bn % 64) continue;
    if (key.N < bn / 2 && bn != 64) continue;
    if (choice & SK_FLAG) {  // stream-K only where the whole-tile schedule leaves a wave partly idle
      const int rows = (choice & M2_FLAG) ? 2 * BM : BM;
      const long tiles = (long)((key.M + rows - 1) / rows) * ((key.N + bn - 1) / bn) * key.G;
      const int sms = num_sms_cached();
      if (tiles % sms == 0 || tiles * kblocks < 2L * sms || kblocks < 8) continue;
    }
    // one warm-up launch, then the best of two batches of four back-to-back launches (short kernels: the
    // batch amortises the event and launch jitter that dominates a single 10-20 us launch)
    float ms = 1e30f;
    bool failed = gemm_with_bn(choice, p, key.a_mn, key.b_mn, epi, alpha, status, stream) != cudaSuccess;
    for (int rep = 0; rep < 2 && !failed; ++rep) {
      cudaEventRecord(e0, stream);
      for (int l = 0; l < 4 && !failed; ++l)
        failed = gemm_with_bn(choice, p, key.a_mn, key.b_mn, epi, alpha, status, stream) != cudaSuccess;
      cudaEventRecord(e1, stream);
      if (failed || cudaEventSynchronize(e1) != cudaSuccess) break;
      float t = 0.f;
      cudaEventElapsedTime(&t, e0, e1);
      ms = std::min(ms, t / 4);
    }
    if (failed) {
      cudaGetLastError();  // a candidate the shape cannot take (e.g. alignment): skip it
      continue;
    }
    // the estimate wins unless a candidate is more than 3% faster (single-launch timings are noisy)
    const float score = choice == guess ? 0.97f * ms : ms;
    if (score < best_ms) {
      best_ms = score;
      best = choice;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  std::lock_guard<std::mutex> lock(tile_mutex());
  tile_cache()[key] = best;
  return best;
}

bool bad_operands(const Prob& p) {
  if ((p.lda & 7) || (p.ldb & 7)) return true;
  for (int g = 0; g < p.G; ++g)
    if (!p.A[g] || !p.B[g] || !p.C[g] || (reinterpret_cast<uintptr_t>(p.A[g]) & 15) ||
        (reinterpret_cast<uintptr_t>(p.B[g]) & 15))
      return true;
  return false;
}

// Shapes share a measured tile choice per bucket: M by 128-row tiles and K by 512 (the token count of a partial
// chunk varies from call to call; the choice affects speed only, never the result).
cudaError_t gemm_measured(const Prob& p, int a_mn, int b_mn, int epi, float alpha, int* status, cudaStream_t stream) {
  const TileKey key{(p.M + BM - 1) / BM * BM, p.N, (p.K + 511) / 512 * 512, a_mn != 0, b_mn != 0, p.G};
  const int bn = measured_bn(key, p, epi, alpha, status, stream);
  return gemm_with_bn(bn, p, a_mn, b_mn, epi, alpha, status, stream);
}

cudaError_t gemm_fixed(const Prob& p, int a_mn, int b_mn, int epi, float alpha, int choice, int* status,
                       cudaStream_t stream) {
  const int bn = choice & (SK_FLAG - 1);
  if (bn != 64 && bn != 128 && bn != 160 && bn != 192 && bn != 224 && bn != 256) return cudaErrorInvalidValue;
  if (b_mn && bn % 64) return cudaErrorInvalidValue;
  if ((choice & M2_FLAG) && ((bn != 128 && bn != 256) || (choice >> SP_SHIFT))) return cudaErrorInvalidValue;
  return gemm_with_bn(choice, p, a_mn, b_mn, epi, alpha, status, stream);
}

}  // namespace

// C[M,N] (ldc) = epi(A · B^T); A K-major [M,K] (lda) or MN-major [K,M] (lda); B K-major [N,K] (ldb) or
// MN-major [K,N] (ldb). bf16 operands; lda/ldb/ldc multiples of 8 elements, 16-byte aligned bases.
extern "C" cudaError_t rt_gemm_bf16(const void* A, long lda, int a_mn, const void* B, long ldb, int b_mn, void* C,
                                    long ldc, int M, int N, int K, int epi, float alpha, int* status,
                                    cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  const Prob p = single(A, lda, B, ldb, C, ldc, M, N, K);
  if (bad_operands(p)) return cudaErrorInvalidValue;
  return gemm_measured(p, a_mn, b_mn, epi, alpha, status, stream);
}

// G (1..3) GEMMs of one shape and layout in one launch: C[g] = epi(A[g] · B[g]^T), with the layouts, strides and
// epilogues of rt_gemm_bf16 (every problem uses the same lda / ldb / ldc). The tiles of all problems share one
// persistent grid and one stream-K iteration space, so three 1024 x 5120 x 5120 projections fill the machine like
// one 1024 x 15360 x 5120 GEMM. choice < 0: the measured tile choice of the shape; else a fixed one (tests).
extern "C" cudaError_t rt_gemm_bf16_group(int G, const void* const* A, long lda, int a_mn, const void* const* B,
                                          long ldb, int b_mn, void* const* C, long ldc, int M, int N, int K, int epi,
                                          float alpha, int choice, int* status, cudaStream_t stream) {
  if (G < 1 || G > MAX_GROUPS || !A || !B || !C) return cudaErrorInvalidValue;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  Prob p = single(A[0], lda, B[0], ldb, C[0], ldc, M, N, K);
  p.G = G;
  for (int g = 1; g < G; ++g) {
    p.A[g] = A[g];
    p.B[g] = B[g];
    p.C[g] = C[g];
  }
  if (bad_operands(p)) return cudaErrorInvalidValue;
  return choice < 0 ? gemm_measured(p, a_mn, b_mn, epi, alpha, status, stream)
                    : gemm_fixed(p, a_mn, b_mn, epi, alpha, choice, status, stream);
}

namespace {
cudaError_t nmse_dispatch(int choice, const Prob& p, const LossArgs& loss, int* status, cudaStream_t s) {
  const int bn = choice & (SK_FLAG - 1);
  const bool sk = (choice & SK_FLAG) != 0;
#define RT_L(W) return launch<W, false, false, EPI_NMSE>(p, 1.f, status, s, 1, sk, loss)
  if (bn == 256) RT_L(256);
  if (bn == 224) RT_L(224);
  if (bn == 192) RT_L(192);
  if (bn == 160) RT_L(160);
  if (bn == 128) RT_L(128);
  RT_L(64);
#undef RT_L
}
}  // namespace

// Student output projection with the distillation loss in the epilogue: p = A B^T (A [M, K], B [N, K], both K-major)
// is never stored; dpred [M, N] (ldc) = 2 (p - t) / (N max(mean_row t^2, eps)) in bf16, and rowsum [M, 4] (whose
// column 0 holds sum_row t^2 on entry) gains the row's sums of (p - t)^2, p^2 and p t. Tile choice: the one measured
// for this shape bucket by a store-epilogue call, else the wave-fill estimate (timing would repeat the sums).
extern "C" cudaError_t rt_gemm_nmse_bf16(const void* A, long lda, const void* B, long ldb, void* dpred, long ldc,
                                         const void* target, float* rowsum, int M, int N, int K, float eps,
                                         int* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((ldc & 7)) return cudaErrorInvalidValue;
  const Prob p = single(A, lda, B, ldb, dpred, ldc, M, N, K);
  if (bad_operands(p)) return cudaErrorInvalidValue;
  const TileKey key{(M + BM - 1) / BM * BM, N, (K + 511) / 512 * 512, 0, 0, 1};
  const int choice = measured_bn(key, p, EPI_NMSE, 1.f, status, stream);
  LossArgs loss;
  loss.target = target;
  loss.rowsum = rowsum;
  loss.eps = eps;
  return nmse_dispatch(choice, p, loss, status, stream);
}

// 1 if a GEMM launched without a status word gave up a wait since the last call (synchronizes the device).
// A launch that gave up a wait leaves its tile's split-K arrive/depart counters and stream-K quarter flags
// nonzero (only the success path clears them); later launches would then pass their waits early on the stale
// counts. So a fault also zeroes the current device's schedule counters, after the device is idle.
extern "C" int rt_gemm_fault() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, gemm_fault_word, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    cudaMemcpyToSymbol(gemm_fault_word, &zero, sizeof(int));
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(g_sk_mutex);
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    for (int lane = 0; lane < SK_LANES; ++lane) {
      auto it = g_sk_spaces.find({dev, lane});
      if (it != g_sk_spaces.end() && it->second.flags &&
          cudaMemset(it->second.flags, 0, SK_MAX_FLAGS * sizeof(int)) != cudaSuccess)
        return -1;
    }
  }
  return v;
}

// Issue lane of this host thread's next GEMM launches (0 or 1; each lane has its own stream-K workspace).
extern "C" cudaError_t rt_gemm_set_lane(int lane) {
  if (lane < 0 || lane >= SK_LANES) return cudaErrorInvalidValue;
  g_lane = lane;
  return cudaSuccess;
}

// 1 while GEMMs of both lanes may overlap on the device (parallel split-K choices then run as stream-K).
extern "C" void rt_gemm_set_concurrent(int on) { g_concurrent.store(on != 0); }

// Asynchronous form of rt_gemm_fault for a per-step metrics snapshot: on `stream`, copy the fault word to `dst`
// (pinned host or device memory) and clear it. A nonzero copy means a launch before it gave up a wait; the
// schedule counters are then reset by a later rt_gemm_fault call (the host raises and stops launching first).
extern "C" cudaError_t rt_gemm_fault_async(int* dst, cudaStream_t stream) {
  void* word = nullptr;
  RT_CUDA_CHECK(cudaGetSymbolAddress(&word, gemm_fault_word));
  RT_CUDA_CHECK(cudaMemcpyAsync(dst, word, sizeof(int), cudaMemcpyDefault, stream));
  return cudaMemsetAsync(word, 0, sizeof(int), stream);
}

// Same with a fixed tile choice (width | 1 << 16 for stream-K); for tests and benchmarks of one schedule.
extern "C" cudaError_t rt_gemm_bf16_tile(const void* A, long lda, int a_mn, const void* B, long ldb, int b_mn,
                                         void* C, long ldc, int M, int N, int K, int epi, float alpha, int choice,
                                         int* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  const Prob p = single(A, lda, B, ldb, C, ldc, M, N, K);
  if (bad_operands(p)) return cudaErrorInvalidValue;
  return gemm_fixed(p, a_mn, b_mn, epi, alpha, choice, status, stream);
}

namespace {

cudaError_t gemm_with_bn(int choice, const Prob& p, int a_mn, int b_mn, int epi, float alpha, int* status,
                         cudaStream_t stream) {
#define RT_G(AM, BMN)                                                                       \
  switch (epi) {                                                                            \
    case EPI_BF16:                                                                          \
      return dispatch_bn<AM, BMN, EPI_BF16>(choice, p, alpha, status, stream);              \
    case EPI_F32:                                                                           \
      return dispatch_bn<AM, BMN, EPI_F32>(choice, p, alpha, status, stream);               \
    default:                                                                                \
      return dispatch_bn<AM, BMN, EPI_F32_ACCUM>(choice, p, alpha, status, stream);         \
  }
  if (!a_mn && !b_mn) { RT_G(false, false) }
  if (!a_mn && b_mn) { RT_G(false, true) }
  if (a_mn && !b_mn) { RT_G(true, false) }
  RT_G(true, true)
#undef RT_G
}

}  // namespace

namespace {

// ws [M, N] fp32 partial sums -> out [M, N] bf16 (ldo), or silu(ws_g) * ws_u when ws_u is given.
__global__ void skinny_finish_kernel(const float* __restrict__ ws, const float* __restrict__ ws_u,
                                     __nv_bfloat16* __restrict__ out, long ldo, int M, int N) {
  const long total = (long)M * N;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
    const int m = (int)(e / N), n = (int)(e % N);
    float v = ws[e];
    if (ws_u) v = rt::siluf_(v) * ws_u[e];
    out[(long)m * ldo + n] = __float2bfloat16_rn(v);
  }
}

// Split count for the skinny path: enough 128-row weight tiles to cover every SM twice, at least 4 k-blocks
// (256 of K) per split.
int skinny_splits(int N, int K) {
  const int tiles = (N + BM - 1) / BM, kblocks = (K + BK - 1) / BK;
  int splits = (2 * num_sms_cached() + tiles - 1) / tiles;
  splits = splits < kblocks / 4 ? splits : kblocks / 4;
  return splits < 1 ? 1 : splits;
}

}  // namespace

// Decode-sized (M <= 32) y[M, N] = X[M, K] · W[N, K]^T as weight streaming: the tcgen05 tiles run swapped
// (128 weight rows x 32 token rows per MMA, weights as the A operand), K is split across CTAs so every SM
// streams weights, partial sums are added (fp32 atomics) into `ws` [M, N] (zeroed here), then converted.
// With Wu given: out = silu(X·W^T) * (X·Wu^T) (ws holds 2 * M * N floats).
extern "C" cudaError_t rt_gemm_skinny_bf16(const void* X, long ldx, const void* W, const void* Wu, long ldw,
                                           float* ws, void* out, long ldo, int M, int N, int K, int* status,
                                           cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if (M > 32 || (ldx & 7) || (ldw & 7) || (reinterpret_cast<uintptr_t>(X) & 15) ||
      (reinterpret_cast<uintptr_t>(W) & 15) || (Wu && (reinterpret_cast<uintptr_t>(Wu) & 15)))
    return cudaErrorInvalidValue;
  const int parts = Wu ? 2 : 1;
  RT_CUDA_CHECK(cudaMemsetAsync(ws, 0, sizeof(float) * (size_t)parts * M * N, stream));
  const int splits = skinny_splits(N, K);
  for (int p = 0; p < parts; ++p)
    RT_CUDA_CHECK((launch<32, false, false, EPI_ATOMIC_T>(single(p ? Wu : W, ldw, X, ldx, ws + (size_t)p * M * N, N,
                                                                 N, M, K),
                                                          1.f, status, stream, splits)));
  const long total = (long)M * N;
  const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  skinny_finish_kernel<<<grid, 256, 0, stream>>>(ws, Wu ? ws + (size_t)M * N : nullptr,
                                                 reinterpret_cast<__nv_bfloat16*>(out), ldo, M, N);
  return cudaGetLastError();
}

namespace {
cudaError_t swiglu_launch(int choice, const Prob& p, int* status, cudaStream_t stream) {
  if (choice & M2_FLAG) return launch<128, false, false, EPI_SWIGLU, 2>(p, 1.f, status, stream);
  return launch<128, false, false, EPI_SWIGLU>(p, 1.f, status, stream);
}

// SwiGLU tile rows per shape bucket (128, or 256 with M2_FLAG), measured once outside stream capture like the
// single-B tile widths: one warm-up launch and the best of two batches of four per candidate; 128 rows unless the
// 256-row tile is more than 3% faster. Both compute every output with the same MMA sequence over K.
int swiglu_choice(const Prob& p, int* status, cudaStream_t stream) {
  const TileKey key{(p.M + BM - 1) / BM * BM, p.N, (p.K + 511) / 512 * 512, 2, 2, 1};  // layouts 2: SwiGLU
  {
    std::lock_guard<std::mutex> lock(tile_mutex());
    auto it = tile_cache().find(key);
    if (it != tile_cache().end()) return it->second;
    // A shorter chunk of a measured shape (same N and K, fewer rows) reuses the nearest larger bucket's choice
    // (256-row tiles only while it keeps at least two row tiles) instead of timing in the middle of training.
    int reuse = -1, reuse_m = 0;
    for (const auto& [k, choice] : tile_cache())
      if (k.a_mn == 2 && k.N == key.N && k.K == key.K && k.M > key.M && (reuse < 0 || k.M < reuse_m)) {
        reuse = choice;
        reuse_m = k.M;
      }
    if (reuse >= 0) {
      if (key.M < 2 * 2 * BM) reuse = 128;
      tile_cache()[key] = reuse;
      return reuse;
    }
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (p.M < 2 * BM || !m2_enabled() || cudaStreamIsCapturing(stream, &cap) != cudaSuccess ||
      cap != cudaStreamCaptureStatusNone)
    return 128;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return 128;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return 128;
  }
  int best = 128;
  float best_ms = 1e30f;
  for (int choice : {128, 128 | M2_FLAG}) {
    float ms = 1e30f;
    bool failed = swiglu_launch(choice, p, status, stream) != cudaSuccess;
    for (int rep = 0; rep < 2 && !failed; ++rep) {
      cudaEventRecord(e0, stream);
      for (int l = 0; l < 4 && !failed; ++l) failed = swiglu_launch(choice, p, status, stream) != cudaSuccess;
      cudaEventRecord(e1, stream);
      if (failed || cudaEventSynchronize(e1) != cudaSuccess) break;
      float t = 0.f;
      cudaEventElapsedTime(&t, e0, e1);
      ms = std::min(ms, t / 4);
    }
    if (failed) {
      cudaGetLastError();
      continue;
    }
    const float score = choice == 128 ? 0.97f * ms : ms;
    if (score < best_ms) {
      best_ms = score;
      best = choice;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  std::lock_guard<std::mutex> lock(tile_mutex());
  tile_cache()[key] = best;
  return best;
}
}  // namespace

// out[M,N] bf16 = silu(A · Bg^T) * (A · Bu^T); A, Bg, Bu K-major. choice < 0: measured tile rows; else 128
// (choice 128) or 256 (128 | 1 << 17) rows per tile (tests).
extern "C" cudaError_t rt_gemm_swiglu_bf16(const void* A, long lda, const void* Bg, const void* Bu, long ldb, void* C,
                                           long ldc, int M, int N, int K, int choice, int* status,
                                           cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((lda & 7) || (ldb & 7)) return cudaErrorInvalidValue;
  Prob p = single(A, lda, Bg, ldb, C, ldc, M, N, K);
  p.B1 = Bu;
  if (bad_operands(p) || !Bu || (reinterpret_cast<uintptr_t>(Bu) & 15)) return cudaErrorInvalidValue;
  if (choice >= 0 && choice != 128 && choice != (128 | M2_FLAG)) return cudaErrorInvalidValue;
  return swiglu_launch(choice < 0 ? swiglu_choice(p, status, stream) : choice, p, status, stream);
}
