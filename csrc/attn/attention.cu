// Causal GQA flash-attention forward for head_dim 256 on sm_100a (tcgen05 + TMA),
// with the gated-attention output gate fused into the epilogue.
//
// One CTA = 128 queries of one query head (grid: query tiles x q-heads x batch).
// Keys/values come from the KV cache [B, cap, Hkv, 256] in blocks of 64.
// Roles (192 threads):
//   warp 0     TMA producer: Q tile once (4 x 64-dim chunks), K and V blocks
//              into a 2-stage ring (no multicast);
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//              score buffers (M=128, N=64, K=256), then O += P_j V_j
//              (M=128, N=256, K=64) with V read MN-major straight from the
//              cache layout;
//   warps 2-5  softmax: one query row per thread (its TMEM lane); causal mask
//              against the absolute position offset + t; online softmax in
//              base 2 with a lazily updated row maximum (the O accumulator in
//              TMEM is rescaled only when the maximum grows by more than 2^8);
//              P_j written as bf16 into a 128B-swizzled K-major tile; at the
//              end O / l times sigmoid(gate) is stored as bf16.
// TMEM: O in columns [0, 256), score buffers in [256, 320) and [320, 384).
// All waits are bounded (sm100.cuh); a timeout records status 1 and unwinds.
#include <cuda.h>
#include "../common/common.cuh"
#include "../common/sm100.cuh"

namespace {

using bf16 = __nv_bfloat16;
constexpr int BQ = 128, BKV = 64, D = 256, DCH = D / 64, THREADS = 192;
constexpr int QCH_BYTES = BQ * 128;              // one 64-dim chunk of the Q tile
constexpr int Q_BYTES = DCH * QCH_BYTES;         // 64 KB
constexpr int KCH_BYTES = BKV * 128;             // one 64-dim chunk of a K or V block
constexpr int KV_BYTES = 2 * DCH * KCH_BYTES;    // K + V of one stage: 64 KB
constexpr int P_BYTES = BQ * 128;                // 128 rows x 64 keys bf16
constexpr int SMEM_BYTES = Q_BYTES + 2 * KV_BYTES + 2 * P_BYTES + 256 + 1024;
constexpr uint32_t IDESC_S = sm100::idesc_bf16(BQ, BKV, false, false);
constexpr uint32_t IDESC_O = sm100::idesc_bf16(BQ, D, false, true);
constexpr uint32_t TMEM_O = 0, TMEM_S = 256;
constexpr float RESCALE_THRESHOLD = 8.f;          // log2 units

struct AttnArgs {
  int B, T, Hq, Hkv, offset, cap;
  float scale_log2;
  const bf16* gate;
  long gate_row, gate_head;
  bf16* out;
  int* status;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(sm100::smem_u32(dst)),
      "l"(tmap), "r"(sm100::smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 2^x by the hardware approximation (flush-to-zero): the softmax probabilities it feeds are rounded to bf16
// right after, far coarser than its error; arguments are <= 0 (x - running max) or -inf (masked keys, giving 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__global__ void __launch_bounds__(THREADS, 1)
flash_attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = sm100::align_smem_1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + Q_BYTES;                  // stage s: K at s*KV_BYTES, V at s*KV_BYTES + DCH*KCH_BYTES
  uint8_t* sP = sKV + 2 * KV_BYTES;             // buffer b at b*P_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_full = bars + 7;    // [2]
  uint64_t* o_done = bars + 9;    // [2]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Longest first: the 1-D grid walks query tiles from the last (most keys under the causal mask) to the first,
  // all heads and batches of one tile before the next, so the shortest tiles fill the tail of the launch.
  const int tiles = (args.T + BQ - 1) / BQ, per = args.Hq * args.B;
  const int tile = tiles - 1 - (int)blockIdx.x / per, rem = (int)blockIdx.x % per;
  const int q0 = tile * BQ, h = rem % args.Hq, b = rem / args.Hq;
  const int g = h / (args.Hq / args.Hkv);
  const int t_last = min(q0 + BQ, args.T) - 1;
  const int nblk = (args.offset + t_last) / BKV + 1;

  if (threadIdx.x == 0) {
    sm100::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&kv_full[i], 1);
      sm100::mbar_init(&kv_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&p_full[i], 128);
      sm100::mbar_init(&o_done[i], 1);
    }
    sm100::mbar_init(drain, 1);
    *abort = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (sm100::elect_one()) {
      sm100::prefetch_tmap(&tq);
      sm100::prefetch_tmap(&tk);
      sm100::prefetch_tmap(&tv);
      sm100::mbar_expect_tx(q_full, Q_BYTES);
      for (int c = 0; c < DCH; ++c) tma_load_3d(sQ + c * QCH_BYTES, &tq, q_full, c * 64, h, b * args.T + q0);
      for (int j = 0; j < nblk && !*abort; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, abort)) break;
        sm100::mbar_expect_tx(&kv_full[st], KV_BYTES);
        uint8_t* k = sKV + st * KV_BYTES;
        uint8_t* v = k + DCH * KCH_BYTES;
        const int row = b * args.cap + j * BKV;
        for (int c = 0; c < DCH; ++c) {
          tma_load_3d(k + c * KCH_BYTES, &tk, &kv_full[st], c * 64, g, row);
          tma_load_3d(v + c * KCH_BYTES, &tv, &kv_full[st], c * 64, g, row);
        }
      }
      for (int j = nblk; j < nblk + 2; ++j)  // both stages consumed before shared memory goes away
        if (j >= 2) sm100::mbar_wait_bounded(&kv_empty[j & 1], ((j >> 1) & 1) ^ 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (sm100::elect_one()) {
      bool ok = sm100::mbar_wait(q_full, 0, abort);
      const uint32_t qb = sm100::smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_full[st], (j >> 1) & 1, abort)) return false;
        sm100::tc_fence_after();
        const uint32_t kb = sm100::smem_u32(sKV + st * KV_BYTES);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int c = ks >> 2, o = (ks & 3) * 32;
          const uint64_t ad = sm100::smem_desc(qb + c * QCH_BYTES + o, 16, 1024);
          const uint64_t bd = sm100::smem_desc(kb + c * KCH_BYTES + o, 16, 1024);
          sm100::mma_bf16(tmem + TMEM_S + st * BKV, ad, bd, IDESC_S, ks > 0);
        }
        sm100::mma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nblk > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nblk; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&p_full[st], (j >> 1) & 1, abort)) break;
        sm100::tc_fence_after();
        const uint32_t pb = sm100::smem_u32(sP + st * P_BYTES);
        const uint32_t vb = sm100::smem_u32(sKV + st * KV_BYTES + DCH * KCH_BYTES);
#pragma unroll
        for (int ks = 0; ks < BKV / 16; ++ks) {
          const uint64_t ad = sm100::smem_desc(pb + ks * 32, 16, 1024);
          const uint64_t bd = sm100::smem_desc(vb + ks * 2048, KCH_BYTES, 1024);
          sm100::mma_bf16(tmem + TMEM_O, ad, bd, IDESC_O, (j > 0 || ks > 0) ? 1u : 0u);
        }
        sm100::mma_commit(&o_done[st]);
        sm100::mma_commit(&kv_empty[st]);
        if (j + 2 < nblk) ok = issue_s(j + 2);
      }
      sm100::mma_commit(drain);
      sm100::mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax / epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int t = q0 + r;
    const int qpos = args.offset + t;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      const int st = j & 1;
      if (!sm100::mbar_wait(&s_full[st], (j >> 1) & 1, abort)) { ok = false; break; }
      sm100::tc_fence_after();
      float s[64];
      {
        float a[32], c2[32];
        sm100::tmem_ld32(lane_base + TMEM_S + st * BKV, a);
        sm100::tmem_ld32(lane_base + TMEM_S + st * BKV + 32, c2);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { s[i] = a[i]; s[32 + i] = c2[i]; }
      }
      const int k0 = j * BKV;
      // Blocks that end at or before the warp's first query position need no causal mask (a warp-uniform test).
      // The block maximum is taken over four independent chains (max is exact, so the order does not matter).
      const bool unmasked = k0 + BKV - 1 <= args.offset + q0 + quarter * 32;
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (unmasked) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          s[i] *= args.scale_log2;
          m4[i & 3] = fmaxf(m4[i & 3], s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          s[i] = (k0 + i <= qpos) ? s[i] * args.scale_log2 : -INFINITY;
          m4[i & 3] = fmaxf(m4[i & 3], s[i]);
        }
      }
      const float mb = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float m_new = fmaxf(m_run, mb);
      if (j == 0) {
        m_run = m_new;
      } else {
        const bool need = m_new > m_run + RESCALE_THRESHOLD;
        if (__any_sync(0xffffffffu, need)) {
          // O must hold P_{j-1} V_{j-1} before it is rescaled.
          if (!sm100::mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort)) { ok = false; break; }
          sm100::tc_fence_after();
          const float alpha = need ? exp2f(m_run - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            sm100::tmem_ld32(lane_base + TMEM_O + c * 32, o);
            sm100::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(lane_base + TMEM_O + c * 32, o);
          }
          tmem_wait_st();
          if (need) {
            l_run *= alpha;
            m_run = m_new;
          }
        }
      }
      float ps[4] = {0.f, 0.f, 0.f, 0.f};  // four independent partial sums of the block's probabilities
      uint32_t packed[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = ex2_approx(s[2 * i] - m_run), p1 = ex2_approx(s[2 * i + 1] - m_run);
        ps[i & 3] += p0 + p1;
        __nv_bfloat162 pk = __floats2bfloat162_rn(p0, p1);
        packed[i] = *reinterpret_cast<uint32_t*>(&pk);
      }
      l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      // P buffer st was last read by the MMA of block j-2.
      if (j >= 2 && !sm100::mbar_wait(&o_done[st], ((j - 2) >> 1) & 1, abort)) { ok = false; break; }
      uint8_t* prow = sP + st * P_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = packed[4 * c]; v.y = packed[4 * c + 1]; v.z = packed[4 * c + 2]; v.w = packed[4 * c + 3];
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&p_full[st]);
    }
    if (ok && sm100::mbar_wait(&o_done[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, abort)) {
      sm100::tc_fence_after();
      const float inv_l = 1.f / l_run;
      const bool store = t < args.T;
      const long bt = (long)b * args.T + t;
      const bf16* gate = args.gate + bt * args.gate_row + (long)h * args.gate_head;
      bf16* out = args.out + (bt * args.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        sm100::tmem_ld32(lane_base + TMEM_O + c * 32, o);
        sm100::tmem_wait_ld();
        if (store) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float g0 = rt::sigmoidf_(__bfloat162float(gate[c * 32 + 2 * i]));
            const float g1 = rt::sigmoidf_(__bfloat162float(gate[c * 32 + 2 * i + 1]));
            __nv_bfloat162 pk = __floats2bfloat162_rn(o[2 * i] * inv_l * g0, o[2 * i + 1] * inv_l * g1);
            w[i] = *reinterpret_cast<uint32_t*>(&pk);
          }
          uint4* dst = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort && args.status) atomicExch(args.status, 1);
}

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

// 3-D map over [rows][heads][256] bf16 with a box of 64 dims x 1 head x box_rows rows.
bool make_map(CUtensorMap* map, const void* base, uint64_t heads, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn encode = encode_fn();
  if (!encode) return false;
  cuuint64_t dims[3] = {D, heads, rows};
  cuuint64_t strides[2] = {D * 2, heads * D * 2};
  cuuint32_t box[3] = {64, 1, box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// q: [B, T, Hq, 256] bf16; keys/values: [B, cap, Hkv, 256] bf16 (positions 0 .. offset+T-1 valid);
// gate: element (b, t, h, d) at gate[(b*T + t) * gate_row + h * gate_head + d]; out: [B, T, Hq, 256] bf16
// = softmax(q k^T / 16, causal at absolute position offset + t) v * sigmoid(gate).
extern "C" cudaError_t rt_flash_attention_fwd(const void* q, const void* keys, const void* values, const void* gate,
                                              long gate_row, long gate_head, void* out, int B, int T, int Hq,
                                              int Hkv, int offset, int cap, int* status, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  if (Hq % Hkv || offset + T > cap) return cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, q, Hq, (uint64_t)B * T, BQ) || !make_map(&tk, keys, Hkv, (uint64_t)B * cap, BKV) ||
      !make_map(&tv, values, Hkv, (uint64_t)B * cap, BKV))
    return cudaErrorInvalidValue;
  AttnArgs args;
  args.B = B; args.T = T; args.Hq = Hq; args.Hkv = Hkv; args.offset = offset; args.cap = cap;
  args.scale_log2 = 0.0625f * 1.4426950408889634f;
  args.gate = (const bf16*)gate; args.gate_row = gate_row; args.gate_head = gate_head;
  args.out = (bf16*)out; args.status = status;
  RT_CUDA_CHECK(cudaFuncSetAttribute(flash_attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  const unsigned ctas = (unsigned)(((T + BQ - 1) / BQ) * Hq * B);
  flash_attn_fwd_kernel<<<ctas, THREADS, SMEM_BYTES, stream>>>(tq, tk, tv, args);
  return cudaGetLastError();
}
