// Fused int4-KV attention for sm_100a (tcgen05 tensor cores, TMEM accumulators).
//
// Computes, per (stream b, head h), O = softmax(Q K^T * scale) V over the cache
// window [lo, hi), reading K and V in packed form: the reference dequantizes the
// window to bf16 (QuantKVTensor.__getitem__, quant_kv.py:189-199) and hands it to
// the upstream attention() (hooked at probe_attention.py:102-124). Tokens below
// sink_tokens are read from the exact bf16 sink copy, as the reference's read
// overlays them (quant_kv.py:196-198). The dequantized values are bit-identical
// to the reference's (fp32 q * scale, rounded to bf16).
//
// One CTA per (128-row Q tile, head, stream); 288 threads, warp-specialised:
//   warps 0-3  converters: load Q once; per KV tile of 128 tokens load codes and
//              scales (or sink rows), dequantize to bf16 and store K and V into
//              double-buffered, 128B-swizzled shared-memory tiles;
//   warps 4-7  softmax: thread r owns Q row r (= TMEM lane r); reads S from TMEM,
//              online softmax in base 2 with lazy rescaling (O is rescaled only
//              when the running max grows by more than 2^8), writes P (bf16) to
//              shared memory, finally normalises O and stores it;
//   warp 8     TMEM allocation and the single thread that issues tcgen05.mma:
//              S_j = Q K_j^T (M=128, N=128, K=128) into one of two TMEM buffers,
//              O += P_j V_j (M=128, N=128, K=128) into the TMEM O accumulator.
// Synchronisation is by mbarriers; every wait gives up after about a second,
// raising a device status word read back by kvq_device_status().
#include <utility>

#include "kvq_common.cuh"
#include "kvq_sm100.cuh"

namespace kvq {
using namespace sm100;

__device__ int g_attn_status = 0;

namespace attn {

constexpr int BM = 128, BN = 128, D = 128;
constexpr int kConvThreads = 128, kSoftThreads = 128;
constexpr int kThreads = kConvThreads + kSoftThreads + 32;
constexpr int kMmaWarp = 8;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // S buffers at columns 0 and 128
constexpr uint32_t kColO = 256;  // O accumulator

// shared memory map (bytes from a 1024-aligned base)
constexpr int kTile = BM * D * 2;  // 32 KB bf16 tile, two 16 KB swizzle atoms
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;       // 2 buffers
constexpr int kOffV = kOffK + 2 * kTile;   // 2 buffers
constexpr int kOffP = kOffV + 2 * kTile;
constexpr int kOffBar = kOffP + kTile;
constexpr int kNumBars = 12;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack

enum Bar { kQFull = 0, kKVFull0 = 1, kKVEmpty0 = 3, kSFull0 = 5, kSEmpty0 = 7, kPFull = 9, kPVDone = 10, kFinal = 11 };

struct Args {
  const uint16_t* q;
  int64_t q_tok_stride, q_batch_stride;
  const uint8_t* kc;
  const uint16_t* ks;
  const uint16_t* ksink;
  const uint8_t* vc;
  const uint16_t* vs;
  const uint16_t* vsink;
  int64_t cache_tokens, sink_tokens, lo;
  int Lk, Lq, H, G;
  uint16_t* out;
  int64_t o_tok_stride, o_batch_stride;
  float scale_log2;
  GroupMap map;
};

// byte offset of 16-byte chunk c (8 bf16 columns) of row r in a 128x128 bf16 tile
// stored as two K-major SWIZZLE_128B atoms (columns 0-63 and 64-127).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * (BM * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

template <class L>
__host__ __device__ constexpr int group_of(int ch) {
  int g = 0;
  while (g + 1 < L::G && ch >= L::E[g + 1]) ++g;
  return g;
}

// 8 channels (one 32-bit word of nibbles) -> 8 bf16, bit-identical to the
// reference dequant: bf16(float(code - 8) * float(scale)).
template <class L, int C>
__device__ __forceinline__ uint4 deq_chunk(uint32_t w, const float (&sf)[L::G]) {
  constexpr int g0 = group_of<L>(8 * C + 0), g1 = group_of<L>(8 * C + 1), g2 = group_of<L>(8 * C + 2),
                g3 = group_of<L>(8 * C + 3), g4 = group_of<L>(8 * C + 4), g5 = group_of<L>(8 * C + 5),
                g6 = group_of<L>(8 * C + 6), g7 = group_of<L>(8 * C + 7);
  auto q = [&](int k) { return static_cast<float>(static_cast<int>((w >> (4 * k)) & 0xFu) - 8); };
  return make_uint4(pack_bf16x2(__fmul_rn(q(0), sf[g0]), __fmul_rn(q(1), sf[g1])),
                    pack_bf16x2(__fmul_rn(q(2), sf[g2]), __fmul_rn(q(3), sf[g3])),
                    pack_bf16x2(__fmul_rn(q(4), sf[g4]), __fmul_rn(q(5), sf[g5])),
                    pack_bf16x2(__fmul_rn(q(6), sf[g6]), __fmul_rn(q(7), sf[g7])));
}

template <class L, int... Cs>
__device__ __forceinline__ void deq_row_store(const uint32_t (&w)[16], const float (&sf)[L::G], uint32_t row_base,
                                              int r, std::integer_sequence<int, Cs...>) {
  (st_shared_v4(row_base + tile_off(r, Cs), deq_chunk<L, Cs>(w[Cs], sf)), ...);
}

template <class L>
__device__ __forceinline__ void load_scales(const uint16_t* p, float (&sf)[L::G]) {
  constexpr int G = L::G;
  if constexpr ((G * 2) % 8 == 0) {
#pragma unroll
    for (int i = 0; i < G / 4; ++i) {
      uint2 v = *reinterpret_cast<const uint2*>(p + 4 * i);
      sf[4 * i + 0] = bf16lo_to_f32(v.x);
      sf[4 * i + 1] = bf16hi_to_f32(v.x);
      sf[4 * i + 2] = bf16lo_to_f32(v.y);
      sf[4 * i + 3] = bf16hi_to_f32(v.y);
    }
  } else if constexpr ((G * 2) % 4 == 0) {
#pragma unroll
    for (int i = 0; i < G / 2; ++i) {
      uint32_t v = *reinterpret_cast<const uint32_t*>(p + 2 * i);
      sf[2 * i + 0] = bf16lo_to_f32(v);
      sf[2 * i + 1] = bf16hi_to_f32(v);
    }
  } else {
#pragma unroll
    for (int i = 0; i < G; ++i) sf[i] = bf16_bits_to_f32(p[i]);
  }
}

// Writes row r (one token of one head) of a K or V tile: zeros past the window,
// the exact bf16 sink copy below sink_tokens, else the dequantized codes.
template <class L>
__device__ __forceinline__ void convert_row(const Args& a, const uint8_t* codes, const uint16_t* scales,
                                            const uint16_t* sink, int b, int h, int jt, uint32_t tile_base,
                                            int r) {
  if (jt >= a.Lk) {
#pragma unroll
    for (int c = 0; c < 16; ++c) st_shared_v4(tile_base + tile_off(r, c), make_uint4(0, 0, 0, 0));
    return;
  }
  const int64_t tok = a.lo + jt;
  if (tok < a.sink_tokens) {
    const uint16_t* src = sink + ((static_cast<int64_t>(b) * a.sink_tokens + tok) * a.H + h) * D;
    uint4 v[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) v[c] = ld_global_nc_v4(src + 8 * c);
#pragma unroll
    for (int c = 0; c < 16; ++c) st_shared_v4(tile_base + tile_off(r, c), v[c]);
    return;
  }
  const int64_t row = (static_cast<int64_t>(b) * a.cache_tokens + tok) * a.H + h;
  const uint4* cp = reinterpret_cast<const uint4*>(codes + row * (D / 2));
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 v = ld_global_nc_v4(cp + i);
    w[4 * i + 0] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
  float sf[L::G];
  load_scales<L>(scales + row * L::G, sf);
  deq_row_store<L>(w, sf, tile_base, r, std::make_integer_sequence<int, 16>{});
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <class L>
__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const __grid_constant__ Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * BM;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int nkv = (a.Lk + BN - 1) / BN;

  if (tid == 0) {
    mbar_init(&bars[kQFull], kConvThreads);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kKVFull0 + i], kConvThreads);
      mbar_init(&bars[kKVEmpty0 + i], 1);
      mbar_init(&bars[kSFull0 + i], 1);
      mbar_init(&bars[kSEmpty0 + i], kSoftThreads);
    }
    mbar_init(&bars[kPFull], kSoftThreads);
    mbar_init(&bars[kPVDone], 1);
    mbar_init(&bars[kFinal], 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // ------------------------------------------------------------ converters
    const int r = tid;
    {
      const int qi = q0 + r;
      const uint32_t qb = sbase + kOffQ;
      if (qi < a.Lq) {
        const uint16_t* src = a.q + b * a.q_batch_stride + static_cast<int64_t>(qi) * a.q_tok_stride +
                              static_cast<int64_t>(h) * D;
        uint4 v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = ld_global_nc_v4(src + 8 * c);
#pragma unroll
        for (int c = 0; c < 16; ++c) st_shared_v4(qb + tile_off(r, c), v[c]);
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) st_shared_v4(qb + tile_off(r, c), make_uint4(0, 0, 0, 0));
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars[kQFull]);
    }
    for (int j = 0; j < nkv; ++j) {
      const int buf = j & 1;
      if (j >= 2 && !mbar_wait_warp(&bars[kKVEmpty0 + buf], ((j >> 1) - 1) & 1, abort, &g_attn_status)) break;
      const int jt = j * BN + r;
      convert_row<L>(a, a.kc, a.ks, a.ksink, b, h, jt, sbase + kOffK + buf * kTile, r);
      convert_row<L>(a, a.vc, a.vs, a.vsink, b, h, jt, sbase + kOffV + buf * kTile, r);
      fence_proxy_async_smem();
      mbar_arrive(&bars[kKVFull0 + buf]);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax
    const int r = tid - kConvThreads;                 // Q row = TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t pb = sbase + kOffP;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      const int buf = j & 1;
      if (!mbar_wait_warp(&bars[kSFull0 + buf], (j >> 1) & 1, abort, &g_attn_status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sb = lane_base + kColS + buf * 128;
      const int valid = min(BN, a.Lk - j * BN);
      // pass 1: row max of S (64 columns per TMEM round trip)
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t s0[32], s1[32];
        tmem_ld32(sb + 64 * k, s0);
        tmem_ld32(sb + 64 * k + 32, s1);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (64 * k + c < valid) mx = fmaxf(mx, __uint_as_float(s0[c]));
          if (64 * k + 32 + c < valid) mx = fmaxf(mx, __uint_as_float(s1[c]));
        }
      }
      const float mt = mx * a.scale_log2;
      // P_j goes to the single P buffer and O may be rescaled: PV_{j-1} must be done
      if (j > 0 && !mbar_wait_warp(&bars[kPVDone], (j - 1) & 1, abort, &g_attn_status)) { ok = false; break; }
      bool rescale = false;
      float alpha = 1.0f;
      if (j == 0) {
        m = mt;
      } else if (mt > m + 8.0f) {
        rescale = true;
        alpha = ex2(m - mt);
        m = mt;
        l *= alpha;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        tc_fence_after();
#pragma unroll 1
        for (int k = 0; k < 4; ++k) {
          uint32_t o[32];
          tmem_ld32(lane_base + kColO + 32 * k, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(lane_base + kColO + 32 * k, o);
        }
        tmem_wait_st();
      }
      // pass 2: P = exp2(S * scale_log2 - m), bf16 into the swizzled P tile
      const float nm = -m;
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t s0[32], s1[32];
        tmem_ld32(sb + 64 * k, s0);
        tmem_ld32(sb + 64 * k + 32, s1);
        tmem_wait_ld();
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float p[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const int cc = 8 * c8 + t;  // column within this 64-column half
            const float sv = __uint_as_float(cc < 32 ? s0[cc] : s1[cc - 32]);
            const float e = ex2(fmaf(sv, a.scale_log2, nm));
            p[t] = (64 * k + cc < valid) ? e : 0.0f;
            sum += p[t];
          }
          st_shared_v4(pb + tile_off(r, 8 * k + c8),
                       make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]), pack_bf16x2(p[4], p[5]),
                                  pack_bf16x2(p[6], p[7])));
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kSEmpty0 + buf]);
      l += sum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[kPFull]);
    }
    if (ok && nkv > 0 && mbar_wait_warp(&bars[kPVDone], (nkv - 1) & 1, abort, &g_attn_status)) {
      tc_fence_after();
      const int qi = q0 + r;
      const float inv = 1.0f / l;
      uint16_t* dst = a.out + b * a.o_batch_stride + static_cast<int64_t>(qi) * a.o_tok_stride +
                      static_cast<int64_t>(h) * D;
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {
        uint32_t o[32];
        tmem_ld32(lane_base + kColO + 32 * k, o);
        tmem_wait_ld();
        if (qi < a.Lq) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            st_global_v4(dst + 32 * k + 8 * c,
                         make_uint4(pack_bf16x2(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                                    pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                                    pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                                    pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv)));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(BM, BN, 0);
      constexpr uint32_t idPV = idesc_bf16(BM, D, 1);
      const uint32_t qaddr = sbase + kOffQ, paddr = sbase + kOffP;
      bool ok = mbar_wait(&bars[kQFull], 0, abort, &g_attn_status);
      auto issue_s = [&](int j) -> bool {
        const int buf = j & 1;
        if (!mbar_wait(&bars[kKVFull0 + buf], (j >> 1) & 1, abort, &g_attn_status)) return false;
        if (j >= 2 && !mbar_wait(&bars[kSEmpty0 + buf], ((j >> 1) - 1) & 1, abort, &g_attn_status)) return false;
        tc_fence_after();
        const uint32_t kaddr = sbase + kOffK + buf * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          mma_bf16_ss(tmem + kColS + buf * 128, smem_desc_sw128(qaddr + off, 16, 1024),
                      smem_desc_sw128(kaddr + off, 16, 1024), idS, kk > 0);
        }
        mma_commit(&bars[kSFull0 + buf]);
        return true;
      };
      if (ok && nkv > 0) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !(ok = issue_s(j + 1))) break;
        if (!(ok = mbar_wait(&bars[kPFull], j & 1, abort, &g_attn_status))) break;
        tc_fence_after();
        const uint32_t vaddr = sbase + kOffV + (j & 1) * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // A = P (K-major over tokens), B = V (MN-major: rows are tokens, d contiguous)
          const uint32_t aoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t boff = kk * 2048;  // 16 tokens = two 8-row groups
          mma_bf16_ss(tmem + kColO, smem_desc_sw128(paddr + aoff, 16, 1024),
                      smem_desc_sw128(vaddr + boff, BN * 128, 1024), idPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars[kPVDone]);
        mma_commit(&bars[kKVEmpty0 + (j & 1)]);
      }
      // all MMAs issued by this thread have completed before TMEM is released
      mma_commit(&bars[kFinal]);
      mbar_wait(&bars[kFinal], 0, abort, &g_attn_status);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <class L>
int launch(const Args& a, int n_qtiles, int batch, cudaStream_t st) {
  static bool configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(attention): %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    configured[dev] = true;
  }
  dim3 grid(n_qtiles, a.H, batch);
  attention_kernel<L><<<grid, kThreads, kSmemBytes, st>>>(a);
  return check_launch("kvq_attention");
}

}  // namespace attn
}  // namespace kvq

using namespace kvq;

extern "C" int kvq_attention(const void* q, int64_t q_token_stride, const void* k_codes, const void* k_scales,
                             const void* k_sink, const void* v_codes, const void* v_scales, const void* v_sink,
                             int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi, void* out,
                             int64_t out_token_stride, int batch, int64_t n_q, int n_heads, int head_dim,
                             const int32_t* chan_band, int n_groups, int k_bits, int v_bits, float softmax_scale,
                             void* stream) {
  clear_error();
  KVQ_REQUIRE(head_dim == 128, KVQ_ERR_UNSUPPORTED, "attention supports head_dim 128, got %d", head_dim);
  KVQ_REQUIRE(k_bits == 4 && v_bits == 4, KVQ_ERR_UNSUPPORTED, "attention reads int4 K and V (got %d/%d bits)",
              k_bits, v_bits);
  KVQ_REQUIRE(batch >= 1 && n_heads >= 1 && n_q >= 0 && cache_tokens >= 1, KVQ_ERR_ARG, "bad shape");
  KVQ_REQUIRE(n_heads <= 65535 && batch <= 65535, KVQ_ERR_ARG, "too many heads or streams");
  KVQ_REQUIRE(0 <= lo && lo < hi && hi <= cache_tokens, KVQ_ERR_ARG,
              "window [%lld, %lld) is empty or outside the cache of %lld tokens", (long long)lo, (long long)hi,
              (long long)cache_tokens);
  KVQ_REQUIRE(hi - lo <= (int64_t)1 << 30 && n_q <= (int64_t)1 << 30, KVQ_ERR_ARG, "sequence too long");
  KVQ_REQUIRE(sink_tokens >= 0 && sink_tokens <= cache_tokens, KVQ_ERR_ARG, "bad sink_tokens");
  KVQ_REQUIRE(sink_tokens == 0 || (k_sink && v_sink), KVQ_ERR_ARG, "sink_tokens > 0 needs both sink buffers");
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  KVQ_REQUIRE(layout != kLayoutGeneric, KVQ_ERR_UNSUPPORTED,
              "attention supports the bands, bands2, bands4, blind32 and blind64 group maps");
  if (n_q == 0) return KVQ_OK;
  KVQ_REQUIRE(q && k_codes && k_scales && v_codes && v_scales && out, KVQ_ERR_ARG, "NULL data pointer");
  KVQ_REQUIRE(q_token_stride >= (int64_t)n_heads * head_dim && out_token_stride >= (int64_t)n_heads * head_dim,
              KVQ_ERR_ARG, "token strides must be >= n_heads*head_dim");
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KVQ_REQUIRE(al16(q) && al16(out) && q_token_stride % 8 == 0 && out_token_stride % 8 == 0, KVQ_ERR_ALIGN,
              "q and out must be 16-byte aligned with token strides that are multiples of 8");
  KVQ_REQUIRE(al16(k_codes) && al16(v_codes) && (!k_sink || al16(k_sink)) && (!v_sink || al16(v_sink)),
              KVQ_ERR_ALIGN, "codes and sink buffers must be 16-byte aligned");
  const int sa = (n_groups * 2) % 8 == 0 ? 8 : (n_groups * 2) % 4 == 0 ? 4 : 2;
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(k_scales) % sa) == 0 && (reinterpret_cast<uintptr_t>(v_scales) % sa) == 0,
              KVQ_ERR_ALIGN, "scales must be %d-byte aligned for %d groups", sa, n_groups);
  int rc = require_sm100();
  if (rc) return rc;
  attn::Args a;
  a.q = static_cast<const uint16_t*>(q);
  a.q_tok_stride = q_token_stride;
  a.q_batch_stride = q_token_stride * n_q;
  a.kc = static_cast<const uint8_t*>(k_codes);
  a.ks = static_cast<const uint16_t*>(k_scales);
  a.ksink = static_cast<const uint16_t*>(k_sink);
  a.vc = static_cast<const uint8_t*>(v_codes);
  a.vs = static_cast<const uint16_t*>(v_scales);
  a.vsink = static_cast<const uint16_t*>(v_sink);
  a.cache_tokens = cache_tokens;
  a.sink_tokens = sink_tokens;
  a.lo = lo;
  a.Lk = static_cast<int>(hi - lo);
  a.Lq = static_cast<int>(n_q);
  a.H = n_heads;
  a.G = n_groups;
  a.out = static_cast<uint16_t*>(out);
  a.o_tok_stride = out_token_stride;
  a.o_batch_stride = out_token_stride * n_q;
  const float sc = softmax_scale > 0.0f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  a.scale_log2 = sc * 1.4426950408889634f;
  a.map = map;
  const int tiles = static_cast<int>((n_q + attn::BM - 1) / attn::BM);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (layout) {
    case kLayoutBands: return attn::launch<LayoutBands>(a, tiles, batch, st);
    case kLayoutBands2: return attn::launch<LayoutBands2>(a, tiles, batch, st);
    case kLayoutBands4: return attn::launch<LayoutBands4>(a, tiles, batch, st);
    case kLayoutBlind32: return attn::launch<LayoutBlind32>(a, tiles, batch, st);
    case kLayoutBlind64: return attn::launch<LayoutBlind64>(a, tiles, batch, st);
    default: break;
  }
  set_error("internal: unhandled layout %d", layout);
  return KVQ_ERR_UNSUPPORTED;
}

extern "C" int kvq_device_status(int reset) {
  clear_error();
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    set_error("cudaDeviceSynchronize: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  e = cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int));
  if (e != cudaSuccess) {
    set_error("reading the device status: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  if (reset && v != 0) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_attn_status, &z, sizeof(int));
    if (e != cudaSuccess) {
      set_error("resetting the device status: %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
  }
  return v;
}
