// Fused int4-KV attention for sm_100a (tcgen05 tensor cores, TMEM, TMA).
//
// Computes, per (stream b, head h), O = softmax(Q K^T * scale) V over the cache
// window [lo, hi), reading K and V in packed form. The reference dequantizes the
// window to bf16 (QuantKVTensor.__getitem__, quant_kv.py:189-199) and hands it to
// the upstream attention() (hooked at probe_attention.py:102-124); tokens below
// sink_tokens come from the exact bf16 sink copy, as the reference's read
// overlays them (quant_kv.py:196-198).
//
// One CTA per (pair of 128-row Q tiles, head, stream); the two Q tiles share
// every dequantized K/V tile. 512 threads, warp-specialised:
//   warps 0-3 / 4-7  softmax for Q tile 0 / 1: thread r owns Q row r (TMEM lane
//                    r). Per KV tile reads S (64
//                    columns) from TMEM, online base-2 softmax with lazy
//                    rescaling of O (only when the row max grows by > 2^8),
//                    writes P as bf16 back into TMEM over S; finally normalises O
//                    and stores it: staged in the Q buffer and written by two TMA
//                    tensor stores per destination (kvq_attention, the gather), or
//                    with per-thread stores (kvq_attention_stats).
//   warps 8-11       converters: per KV tile of 64 tokens, warps 8-9 dequantize
//                    the K rows and 10-11 the V rows (one row per thread) from
//                    the TMA-staged codes into 128B-swizzled bf16 tiles, with
//                    packed bf16x2 arithmetic (bit-identical to the reference).
//                    A row's scales of the next tile are loaded while the
//                    current tile is converted.
//   warps 12 / 15    TMA producers for K / V: packed codes (SWIZZLE_64B staging)
//                    and, for tiles that reach into the sink, the bf16 sink rows
//                    straight into the bf16 tiles (SWIZZLE_128B, the MMA's
//                    layout). Warp 12 first loads the Q tiles by TMA (the S
//                    MMA's 128B-swizzled K-major layout; rows past n_q read 0):
//                    per-thread Q loads had made each CTA's start ~2.5x slower.
//   warps 13 / 14    one thread each issuing the tcgen05.mma of Q tile 0 / 1:
//                    S_x = Q_x K^T (M=128, N=64, K=128, Q and K in shared
//                    memory) and O_x += P_x V (M=128, N=128, K=64, P in TMEM, V
//                    an MN-major shared-memory operand). Warp 13 also owns the
//                    TMEM allocation.
// Pipelining (measured on B200, drives the layout):
//  - S is double-buffered per Q tile and S_x(j+2) is issued right behind
//    PV_x(j) (one thread's MMAs run in issue order, so it overwrites P_x(j)
//    only after PV_x(j) has read it): S_x(j+1) has a whole softmax step to
//    complete and the softmax warps go from one KV tile to the next without
//    waiting for the tensor pipe or for a straggling warp of their Q tile.
//  - One issuing thread per Q tile: a single thread issues a tcgen05.mma only
//    every ~60-100 cycles and blocks ~250 cycles on each tcgen05.commit, which
//    leaves the tensor pipe half idle; two threads keep it fed.
//  - One commit per KV tile and thread (S_x full). Everything else is derived
//    from it: the softmax that sees S_x(j) releases K stage j (read by S_x(j)
//    only) and V stage j-2 (S_x(j) was issued behind PV_x(j-2)); a rescale of O
//    at tile j waits for S_x(j+1) (issued behind PV_x(j-1)).
//  - K and V run as two streams (own code stages, bf16 stages, barriers and
//    producer): K stages come free two KV tiles before V stages, so the K rows
//    of tile j+2 are converted well before S_x(j+2) is issued and their
//    conversion is off the per-tile chain P_x(j) -> PV_x(j) -> S_x(j+2).
// TMEM columns: O_0 [0,128) O_1 [128,256), S_0 [256,320) [320,384), S_1
// [384,448) [448,512) (P over the first 32 columns of its S buffer).
// Synchronisation is by mbarriers with one arrival per warp; every wait gives up
// after about a second, raising the device status word (kvq_device_status()).
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <queue>
#include <vector>
#include <type_traits>
#include <utility>

#include "kvq_common.cuh"
#include "kvq_sm100.cuh"

namespace kvq {
using namespace sm100;

__device__ int g_attn_status = 0;

namespace attn {

constexpr int BM = 128;   // rows per Q tile
constexpr int BN = 64;    // KV tokens per tile
constexpr int D = 128;
constexpr int NS_KV = 4;  // bf16 K/V tile stages
constexpr int kThreads = 16 * 32;
constexpr int kConvWarp0 = 8, kProdWarp = 12, kMmaWarp = 13;  // MMA issuers: warps 13 (Q tile 0), 14 (Q tile 1)
constexpr int kProdWarpV = 15;                                  // warp 12 produces K, warp 15 V
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256;  // S_x buffer u at kColS + 128x + 64u

constexpr int kKVTile = BN * D * 2;     // 16 KB: two 8 KB SWIZZLE_128B atoms (d 0-63, 64-127)
constexpr int kAtom = BN * 128;         // 8 KB
constexpr int kQTile = BM * D * 2;  // 32 KB: Q_x as two 16 KB SWIZZLE_128B atoms (d 0-63, 64-127)
constexpr int kQAtom = BM * 128;    // 16 KB

// Shared-memory geometry for int4 (KB = 4) or int8 (KB = 8) K codes; V codes
// are int4. Code tiles are 64 tokens x 64 B (int4, SWIZZLE_64B) or x 128 B
// (int8, SWIZZLE_128B); int8 K keeps two code stages instead of four so that
// everything fits the 227 KB of one CTA.
template <int KB>
struct Geo {
  static constexpr int NS_LD = KB == 4 ? 4 : 2;  // packed-code stages
  static constexpr int kCodeTileK = BN * (KB == 4 ? 64 : 128);
  static constexpr int kCodeTileV = BN * 64;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + NS_KV * kKVTile;
  static constexpr int kOffKC = kOffV + NS_KV * kKVTile;
  static constexpr int kOffVC = kOffKC + NS_LD * kCodeTileK;
  static constexpr int kOffQ = kOffVC + NS_LD * kCodeTileV;
  static constexpr int kOffBar = kOffQ + 2 * kQTile;
  // barrier indices (S/P full: 2x + buffer)
  // code stages and bf16 stages per tensor: index + NS_LD (NS_KV) for V
  static constexpr int bLdFull = 0, bLdEmpty = bLdFull + 2 * NS_LD, bKvFull = bLdEmpty + 2 * NS_LD,
                       bKvEmpty = bKvFull + 2 * NS_KV, bQReady = bKvEmpty + 2 * NS_KV, bSFull = bQReady + 2,
                       bPFull = bSFull + 4, bOReady = bPFull + 4, bOFinal = bOReady + 2, bMmaDone = bOFinal + 2,
                       bEpi = bMmaDone + 2, kNumBars = bEpi + 2;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack
  static_assert(kOffQ % 1024 == 0 && kOffKC % 1024 == 0, "SWIZZLE_128B operands need 1024-byte alignment");
  static_assert(kSmemBytes <= 227 * 1024, "one CTA per SM must fit");
};

constexpr int kMaxOut = 8;

struct alignas(64) Args {
  CUtensorMap tm_kc, tm_vc;  // codes [B*S rows, H*64 B (int8 K: H*128 B)], box 64 (128) x 64, SWIZZLE_64B (128B)
  CUtensorMap tm_ks, tm_vs;  // sinks [B*sink rows, H*128 bf16], box 64 x 64, SWIZZLE_128B
  CUtensorMap tm_q;          // q as [batch][n_q][H * D] bf16, box 64 x 128 x 1, SWIZZLE_128B (rows past n_q read 0)
  const uint16_t* q;
  int64_t q_tok_stride, q_batch_stride;
  const uint16_t* ks;
  const uint16_t* vs;
  int64_t cache_tokens, sink_tokens, lo;
  int Lk, Lq, H;
  uint16_t* out[kMaxOut];  // n_out destinations of identical layout (this GPU's and peers')
  int n_out, out_head0;     // heads of this launch land at heads out_head0.. of each destination
  int tma_out;              // store through tm_out (one TMA store per Q tile and destination)
  float* stats;             // STATS kernels: [batch][n_q][n_heads][4] fp32 row statistics
  CUtensorMap tm_out[kMaxOut];  // destination d as [batch][n_q][out_heads * D] bf16, box 64 x 128 x 1, SWIZZLE_128B
  int64_t o_tok_stride, o_batch_stride;
  float scale_log2;
  long long wait_cycles;  // limit of every bounded wait (kWaitCycles unless a test asks for less)
  int stall_tile;         // >= 0 only in the abort test: the K producer stops before this KV tile
  // Work units (see attention_kernel): n_hb = heads x streams; the last split_full
  // two-tile units run as two halves of their KV window, every one-tile unit as
  // split_single parts (1 = whole); parts exchange partial results through ws and
  // count in ctr[unit]. ws holds slots of float4 [33][128 rows] (a Q tile's O
  // rows in 32 chunks of 4 channels, then (m, l)): split two-tile unit u, part p,
  // Q tile x at slot (2u + p) 2 + x; one-tile unit s (unit split_full + s), part p
  // at slot 4 split_full + s split_single + p.
  int n_hb, split_full, split_single;
  float4* ws;
  unsigned* ctr;
};

// byte offset of 16-byte chunk c (8 bf16 columns) of row r in a 64 x 128 bf16
// tile stored as two K-major SWIZZLE_128B atoms (columns 0-63 and 64-127).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * kAtom + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

template <class L>
__host__ __device__ constexpr int group_of(int ch) {
  int g = 0;
  while (g + 1 < L::G && ch >= L::E[g + 1]) ++g;
  return g;
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Channels 8C..8C+7 (one 32-bit word of nibbles, w; ws = w >> 4) -> 8 bf16.
// Pair i = channels (8C+2i, 8C+2i+1) = byte i: bf16x2 (128 + lo, 128 + hi) by a
// byte permute and one mask/or, minus 136 (exact), times (s_g, s_g): the exact
// product rounded to bf16, i.e. the reference's bf16(float(q) * float(scale)).
template <class L, int C>
__device__ __forceinline__ uint4 deq8(uint32_t w, uint32_t ws, const uint32_t (&sp)[L::G]) {
  constexpr uint32_t k136 = 0x43084308u;  // bf16x2 (136, 136)
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t t = __byte_perm(w, ws, static_cast<uint32_t>(((4 + i) << 8) | i));
    t = (t & 0x000F000Fu) | 0x43004300u;
    o[i] = t;
  }
  constexpr int g0 = group_of<L>(8 * C + 0), g1 = group_of<L>(8 * C + 2), g2 = group_of<L>(8 * C + 4),
                g3 = group_of<L>(8 * C + 6);
  return make_uint4(bf2_mul(bf2_sub(o[0], k136), sp[g0]), bf2_mul(bf2_sub(o[1], k136), sp[g1]),
                    bf2_mul(bf2_sub(o[2], k136), sp[g2]), bf2_mul(bf2_sub(o[3], k136), sp[g3]));
}

template <class L, int... Cs>
__device__ __forceinline__ void deq_row(const uint32_t (&w)[16], const uint32_t (&sp)[L::G], uint32_t dst, int r,
                                        std::integer_sequence<int, Cs...>) {
  (st_shared_v4(dst + tile_off(r, Cs), deq8<L, Cs>(w[Cs], w[Cs] >> 4, sp)), ...);
}

// int8 channels 16C..16C+15 (one 16-byte chunk v of codes q + 128) -> 16 bf16:
// each byte goes into the low mantissa of 2^23 (exact), minus 2^23 + 128 gives q
// (exact), times the group's fp32 scale (exact: 8 x 8 significant bits), and one
// round to bf16 (cvt.rn.bf16x2): the reference's bf16(float(q) * float(scale)).
// one pair of int8 codes (bytes 2p, 2p+1 of w) times the scale s -> bf16x2
__device__ __forceinline__ uint32_t deq_pair_i8(uint32_t w, uint32_t sel, float s) {
  const float2 f = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, sel)),
                               __uint_as_float(__byte_perm(w, 0x4B000000u, sel + 1)));
  const float2 q = __fadd2_rn(f, make_float2(-8388736.0f, -8388736.0f));
  const float2 y = __fmul2_rn(q, make_float2(s, s));
  return pack_bf16x2(y.x, y.y);
}

template <class L, int C>
__device__ __forceinline__ void deq16_i8(uint4 v, const float (&sf)[L::G], uint32_t dst, int r) {
  constexpr int g0 = group_of<L>(16 * C + 0), g1 = group_of<L>(16 * C + 2), g2 = group_of<L>(16 * C + 4),
                g3 = group_of<L>(16 * C + 6), g4 = group_of<L>(16 * C + 8), g5 = group_of<L>(16 * C + 10),
                g6 = group_of<L>(16 * C + 12), g7 = group_of<L>(16 * C + 14);
  st_shared_v4(dst + tile_off(r, 2 * C),
               make_uint4(deq_pair_i8(v.x, 0x7540u, sf[g0]), deq_pair_i8(v.x, 0x7542u, sf[g1]),
                          deq_pair_i8(v.y, 0x7540u, sf[g2]), deq_pair_i8(v.y, 0x7542u, sf[g3])));
  st_shared_v4(dst + tile_off(r, 2 * C + 1),
               make_uint4(deq_pair_i8(v.z, 0x7540u, sf[g4]), deq_pair_i8(v.z, 0x7542u, sf[g5]),
                          deq_pair_i8(v.w, 0x7540u, sf[g6]), deq_pair_i8(v.w, 0x7542u, sf[g7])));
}

template <class L, int... Cs>
__device__ __forceinline__ void deq_row_i8(uint32_t src, const float (&sf)[L::G], uint32_t dst, int r,
                                           std::integer_sequence<int, Cs...>) {
  (deq16_i8<L, Cs>(ld_shared_v4(src + ((Cs ^ (r & 7)) << 4)), sf, dst, r), ...);
}

// Raw scale words of one row (bf16 pairs, or single bf16 values for odd G).
template <class L>
struct ScaleWords {
  static constexpr int N = (L::G * 2) % 4 == 0 ? L::G / 2 : L::G;
  uint32_t v[N];
};

template <class L>
__device__ __forceinline__ void load_scale_words(const uint16_t* p, ScaleWords<L>& s) {
  constexpr int G = L::G;
  if constexpr ((G * 2) % 8 == 0) {
#pragma unroll
    for (int i = 0; i < G / 4; ++i) {
      uint2 v = __ldg(reinterpret_cast<const uint2*>(p + 4 * i));
      s.v[2 * i] = v.x;
      s.v[2 * i + 1] = v.y;
    }
  } else if constexpr ((G * 2) % 4 == 0) {
#pragma unroll
    for (int i = 0; i < G / 2; ++i) s.v[i] = __ldg(reinterpret_cast<const uint32_t*>(p + 2 * i));
  } else {
#pragma unroll
    for (int i = 0; i < G; ++i) s.v[i] = __ldg(p + i);
  }
}

// (s_g, s_g) bf16x2 per group
template <class L>
__device__ __forceinline__ void scale_pairs(const ScaleWords<L>& s, uint32_t (&sp)[L::G]) {
  constexpr int G = L::G;
  if constexpr ((G * 2) % 4 == 0) {
#pragma unroll
    for (int i = 0; i < G / 2; ++i) {
      sp[2 * i] = __byte_perm(s.v[i], 0, 0x1010);
      sp[2 * i + 1] = __byte_perm(s.v[i], 0, 0x3232);
    }
  } else {
#pragma unroll
    for (int i = 0; i < G; ++i) sp[i] = __byte_perm(s.v[i], 0, 0x1010);
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Most parts a one-tile unit is cut into (at window 3 eight parts measured slower
// than four: each part pays a CTA's fill and a partial store).
constexpr int kMaxParts = 4;

// Workspace slot (float4 [33][128] each) of Q tile x of part p of split unit u.
__host__ __device__ __forceinline__ int64_t ws_slot(const Args& a, int u, int p, int x) {
  return u < a.split_full ? (static_cast<int64_t>(u) * 2 + p) * 2 + x
                          : static_cast<int64_t>(4) * a.split_full +
                                static_cast<int64_t>(u - a.split_full) * a.split_single + p;
}

template <class L, int KB, bool STATS>
__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const __grid_constant__ Args a) {
  using GEO = Geo<KB>;
  constexpr int NS_LD = GEO::NS_LD, kCodeTileK = GEO::kCodeTileK, kCodeTileV = GEO::kCodeTileV;
  constexpr int kOffK = GEO::kOffK, kOffV = GEO::kOffV, kOffKC = GEO::kOffKC, kOffVC = GEO::kOffVC,
                kOffQ = GEO::kOffQ, kOffBar = GEO::kOffBar, kOffMisc = GEO::kOffMisc;
  constexpr int bLdFull = GEO::bLdFull, bLdEmpty = GEO::bLdEmpty, bKvFull = GEO::bKvFull,
                bKvEmpty = GEO::bKvEmpty, bQReady = GEO::bQReady, bSFull = GEO::bSFull, bPFull = GEO::bPFull,
                bOReady = GEO::bOReady, bOFinal = GEO::bOFinal, bMmaDone = GEO::bMmaDone, bEpi = GEO::bEpi;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const long long lim = a.wait_cycles;
  pdl_wait();
  pdl_launch_dependents();
  // One CTA per (pair of Q tiles, head, stream), 1-D grid. The CTAs with two Q
  // tiles come first, pairs fastest (a head's packed K/V stays in L2 across its
  // pairs); the last pairs that hold at most BM queries (one Q tile, about half
  // the work) come after all of them, so that they fill the last wave instead of
  // leaving a partial wave of full-length CTAs at the end.
  //
  // Wave balance: the last split_full two-tile units are each run by two CTAs,
  // one per half of the KV window (consecutive block indices), and every one-tile
  // unit by split_single CTAs (one per part of the KV window): finer pieces for
  // the last wave. A part is an ordinary CTA on a sub-window of whole KV tiles; it
  // leaves its unnormalised O, row max and row sum in the workspace, and the part
  // that finishes last merges them (after the CTA's final barrier, below).
  const int n_pairs = (a.Lq + 2 * BM - 1) / (2 * BM);
  const int n_full = a.Lq - (n_pairs - 1) * 2 * BM > BM ? n_pairs : n_pairs - 1;
  const int n_hb = a.n_hb;  // heads x streams
  const int n_ft = n_full * n_hb;
  const int n_a = n_ft - a.split_full;  // two-tile units run whole
  const int bid = static_cast<int>(blockIdx.x);
  int pair, hb, part = 0, parts = 1, unit = -1;
  if (bid < n_a) {
    hb = bid / n_full;
    pair = bid - hb * n_full;
  } else if (bid < n_ft + a.split_full) {
    const int v = bid - n_a, u = n_a + (v >> 1);
    hb = u / n_full;
    pair = u - hb * n_full;
    part = v & 1;
    parts = 2;
    unit = v >> 1;
  } else {
    const int w = bid - (n_ft + a.split_full);
    hb = w / a.split_single;
    part = w - hb * a.split_single;
    parts = a.split_single;
    pair = n_pairs - 1;
    if (parts > 1) unit = a.split_full + hb;
  }
  const int q0 = pair * (2 * BM);
  const int h = hb % a.H;
  const int b = hb / a.H;
  const int nq = a.Lq - q0 > BM ? 2 : 1;  // Q tiles with queries
  // this CTA's KV window: tiles [jb, je) of the launch's window of a.Lk tokens from a.lo
  const int nkv_all = (a.Lk + BN - 1) / BN;
  const int jb = part * nkv_all / parts, je = (part + 1) * nkv_all / parts;
  const int64_t lo = a.lo + static_cast<int64_t>(jb) * BN;
  const int Lk = min(je * BN, a.Lk) - jb * BN;
  const int nkv = je - jb;

  if (tid == 0) {
    for (int i = 0; i < 2 * NS_LD; ++i) {
      mbar_init(&bars[bLdFull + i], 1);
      mbar_init(&bars[bLdEmpty + i], 2);  // the tensor's two converter warps
    }
    for (int i = 0; i < 2 * NS_KV; ++i) {
      mbar_init(&bars[bKvFull + i], 2);
      mbar_init(&bars[bKvEmpty + i], nq);  // one arrival per Q tile (softmax warp 4x)
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars[bQReady + x], 1);  // the K producer's expect_tx; Q arrives by TMA
      mbar_init(&bars[bSFull + 2 * x], 1);
      mbar_init(&bars[bSFull + 2 * x + 1], 1);
      mbar_init(&bars[bPFull + 2 * x], 4);
      mbar_init(&bars[bPFull + 2 * x + 1], 4);
      mbar_init(&bars[bOReady + x], 1);
      mbar_init(&bars[bOFinal + x], 1);
    }
    mbar_init(&bars[bMmaDone], 1);
    mbar_init(&bars[bMmaDone + 1], 1);
    mbar_init(&bars[bEpi], 4);
    mbar_init(&bars[bEpi + 1], 4);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if ((warp == kProdWarp || warp == kProdWarpV) && lane == 0) {
    const bool pv = warp != kProdWarp;
    if (!pv) prefetch_tmap(&a.tm_q);
    prefetch_tmap(pv ? &a.tm_vc : &a.tm_kc);
    if (a.sink_tokens > 0) prefetch_tmap(pv ? &a.tm_vs : &a.tm_ks);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4 * nq) {
    // ------------------------------------------------------------ softmax (Q tile x)
    const int x = warp >> 2;
    const int r = tid - x * BM;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + lane_off + kColO + 128 * x;
    const uint32_t tS0 = tmem + lane_off + kColS + 128 * x;
    const int qi = q0 + x * BM + r;
    float m = -INFINITY, l = 0.0f;
    // STATS: with e = 2^(t - m) (t = scaled logit in log2 units), lb = sum e (t - m),
    // ls = sum of e over sink tokens, mtrue = the row's true max of t (m may lag it
    // by up to 8). Entropy = ln2 (log2 l - lb / l), max weight = 2^(mtrue - m) / l,
    // sink mass = ls / l, log-sum-exp = ln2 (m + log2 l).
    float lb = 0.0f, ls = 0.0f, mtrue = -INFINITY;
    bool ok = true;
    // One KV tile. PART (the window's last tile when it holds fewer than BN
    // tokens) is a separate instantiation: the column masking then costs nothing
    // on the full tiles, where per-column selects would be issued every time.
    auto step = [&](const int j, const int valid, auto part) -> bool {
      constexpr bool PART = decltype(part)::value;
      const uint32_t tS = tS0 + 64 * (j & 1);
      if (!mbar_wait_warp(&bars[bSFull + 2 * x + (j & 1)], (j >> 1) & 1, abort, &g_attn_status, lim)) return false;
      // S_x(j) complete => this Q tile no longer reads K stage j, and PV_x(j-2)
      // (issued before it) is complete: nor V stage j-2
      if ((warp & 3) == 0 && lane == 0) {
        mbar_arrive(&bars[bKvEmpty + j % NS_KV]);
        if (j >= 2) mbar_arrive(&bars[bKvEmpty + NS_KV + (j - 2) % NS_KV]);
      }
      tc_fence_after();
      uint32_t s0[32], s1[32];
      tmem_ld32x2_wait(tS, tS + 32, s0, s1);
      if constexpr (PART) {
        // columns past the window: a finite logit so low that its weight is 0
        // (finite, so that the entropy sum's p * t stays 0)
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c >= valid) s0[c] = __float_as_uint(-1.0e30f);
          if (32 + c >= valid) s1[c] = __float_as_uint(-1.0e30f);
        }
      }
      // row max: 8 independent chains of three-input maxima
      float pm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pm[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) pm[c & 7] = fmax3(pm[c & 7], __uint_as_float(s0[c]), __uint_as_float(s1[c]));
      const float mt =
          fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) * a.scale_log2;
      bool rescale = false;
      float alpha = 1.0f;
      if (j == 0) {
        m = mt;
      } else if (mt > m + 8.0f) {
        rescale = true;
        alpha = ex2(m - mt);
        if (STATS) {
          lb = alpha * (lb - (mt - m) * l);
          ls *= alpha;
        }
        m = mt;
        l *= alpha;
      }
      if (STATS) mtrue = fmaxf(mtrue, mt);
      const float nm = -m;
      float sum = 0.0f, sumb = 0.0f;
      uint32_t pw[32];
      // P for tokens 0-31 of the tile (S columns 0-31) then 32-63: the first half's
      // TMEM store runs while the second half is computed
      // paired f32x2 operations for the scaling and the row sum: half the issue
      // slots of scalar ones, on sub-partitions shared with the converters
      const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(nm, nm);
      float2 sum2 = make_float2(0.0f, 0.0f), sumb2 = make_float2(0.0f, 0.0f);
      auto half = [&](const uint32_t (&sv)[32], int base) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float2 xx =
              __ffma2_rn(make_float2(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1])), sc2, nm2);
          const float p0 = ex2(xx.x), p1 = ex2(xx.y);
          sum2 = __fadd2_rn(sum2, make_float2(p0, p1));
          if (STATS) sumb2 = __ffma2_rn(make_float2(p0, p1), xx, sumb2);
          pw[base / 2 + c] = pack_bf16x2(p0, p1);
        }
      };
      half(s0, 0);
      tmem_st16(tS, pw);
      half(s1, 32);
      tmem_st16(tS + 16, pw + 16);
      sum = sum2.x + sum2.y;
      if (STATS) sumb = sumb2.x + sumb2.y;
      l += sum;
      if (STATS) {
        lb += sumb;
        // columns whose cache token is below sink_tokens
        const int64_t t0 = lo + static_cast<int64_t>(j) * BN;
        const int ns = static_cast<int>(max(static_cast<int64_t>(0), min(static_cast<int64_t>(valid), a.sink_tokens - t0)));
        if (ns == valid) {
          ls += sum;
        } else if (ns > 0) {
          // the border tile's sink part, recomputed (one tile per row)
          float part = 0.0f;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            if (c < ns) part += ex2(fmaf(__uint_as_float(s0[c]), a.scale_log2, nm));
            if (32 + c < ns) part += ex2(fmaf(__uint_as_float(s1[c]), a.scale_log2, nm));
          }
          ls += part;
        }
      }
      // The rescale of O comes after P: the tile's 64 logits are dead here (with
      // them live, O's registers made the compiler spill). PV_x(j), which
      // accumulates into the rescaled O, is issued only after this warp's arrival.
      if (__any_sync(0xffffffffu, rescale)) {
        // O_x must hold every product up to PV_x(j-1) before it is rescaled:
        // wait for S_x(j+1), issued behind PV_x(j-1) (the next commit into that
        // buffer, S_x(j+3), follows PV_x(j+1), so the phase is unambiguous), or,
        // at the last tile, for the commit that follows PV_x(j-1).
        const bool last = j + 1 == nkv;
        if (!mbar_wait_warp(&bars[last ? bOReady + x : bSFull + 2 * x + ((j + 1) & 1)],
                            last ? 0u : static_cast<uint32_t>(((j + 1) >> 1) & 1), abort, &g_attn_status, lim))
          return false;
        tc_fence_after();
#pragma unroll 1
        for (int k = 0; k < 8; ++k) {
          uint32_t o[16];
          tmem_ld16_wait(tO + 16 * k, o);
#pragma unroll
          for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st16(tO + 16 * k, o);
        }
        tmem_wait_st();
      }
      tmem_wait_st();  // P_x(j), 64 bf16 = 32 columns, over S_x(j)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[bPFull + 2 * x + (j & 1)]);
      return true;
    };
    for (int j = 0; j < nkv; ++j) {
      const int valid = min(BN, Lk - j * BN);
      if (!(valid == BN ? step(j, valid, std::false_type{}) : step(j, valid, std::true_type{}))) {
        ok = false;
        break;
      }
    }
    if (ok && parts > 1 && mbar_wait_warp(&bars[bOFinal + x], 0, abort, &g_attn_status, lim)) {
      // one part of a split unit: leave the unnormalised O row, m and l for the merge
      tc_fence_after();
      float4* dst = a.ws + ws_slot(a, unit, part, x) * 33 * BM + r;
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {
        uint32_t o[32];
        tmem_ld32_wait(tO + 32 * k, o);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          dst[(8 * k + c) * BM] = make_float4(__uint_as_float(o[4 * c]), __uint_as_float(o[4 * c + 1]),
                                              __uint_as_float(o[4 * c + 2]), __uint_as_float(o[4 * c + 3]));
      }
      dst[32 * BM] = make_float4(m, l, 0.0f, 0.0f);
      __threadfence();
    } else if (ok && mbar_wait_warp(&bars[bOFinal + x], 0, abort, &g_attn_status, lim)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      if (STATS && qi < a.Lq) {
        constexpr float kLn2 = 0.69314718055994531f;
        const float lg = log2f(l);
        float4 st;
        st.x = kLn2 * (m + lg);               // log-sum-exp of the scaled logits (natural log)
        st.y = kLn2 * (lg - lb * inv);        // entropy of the attention row (nats)
        st.z = ex2(mtrue - m) * inv;          // largest attention weight
        st.w = ls * inv;                      // attention mass on the sink tokens
        *reinterpret_cast<float4*>(a.stats + ((static_cast<int64_t>(b) * a.Lq + qi) * a.H + h) * 4) = st;
      }
      if (a.tma_out) {
        // Stage the normalised tile in the (no longer read) Q_x buffer, in the
        // layout of Q (two 64-column SWIZZLE_128B atoms), then one thread stores
        // it to every destination with TMA: 256-byte rows, asynchronous, so the
        // traffic to peers drains while the SM runs its next CTA.
        const uint32_t stage = sbase + kOffQ + x * kQTile;
#pragma unroll 1
        for (int k = 0; k < 4; ++k) {
          uint32_t o[32];
          tmem_ld32_wait(tO + 32 * k, o);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int ch = 4 * k + c;  // 16-byte chunk = 8 columns
            st_shared_v4(stage + (ch >> 3) * kQAtom + r * 128 + (((ch & 7) ^ (r & 7)) << 4),
                         make_uint4(pack_bf16x2(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                                    pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                                    pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                                    pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv)));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[bEpi + x]);
        if ((warp & 3) == 0 && lane == 0 && mbar_wait(&bars[bEpi + x], 0, abort, &g_attn_status, lim)) {
          const int xq = (a.out_head0 + h) * D, yq = q0 + x * BM;
          // destinations in an order rotated by the block index: with peers, the CTAs
          // of a wave then push into every GPU's NVLink ingress at once, not all into one
          for (int i = 0; i < a.n_out; ++i) {
            const int d = (i + static_cast<int>(blockIdx.x)) % a.n_out;
            tma_store_3d(&a.tm_out[d], stage, xq, yq, b);
            tma_store_3d(&a.tm_out[d], stage + kQAtom, xq + 64, yq, b);
          }
          bulk_commit();
          bulk_wait_read_all();  // the staging buffer must outlive the reads
        }
        __syncwarp();
      } else {
      const int64_t off = b * a.o_batch_stride + static_cast<int64_t>(qi) * a.o_tok_stride +
                          static_cast<int64_t>(a.out_head0 + h) * D;
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {
        uint32_t o[32];
        tmem_ld32_wait(tO + 32 * k, o);
        if (qi < a.Lq) {
          uint4 v[4];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            v[c] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                              pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                              pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                              pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
          // the row goes to every destination: with peer buffers (mapped over
          // NVLink) this epilogue is the all-gather of the head-sharded output
#pragma unroll 1
          for (int i = 0; i < a.n_out; ++i) {
            const int d = (i + static_cast<int>(blockIdx.x)) % a.n_out;  // rotated, as the TMA epilogue
#pragma unroll
            for (int c = 0; c < 4; ++c) st_global_v4(a.out[d] + off + 32 * k + 8 * c, v[c]);
          }
        }
      }
      }
      // No fence: the peer stores drain while the SM runs its next CTA; the
      // consumer orders them by the kernel's completion (stream synchronize on
      // the writing rank, then a cross-rank barrier).
    }
  } else if (warp < 8) {
    // a Q tile without queries: nothing to do
  } else if (warp < kProdWarp) {
    // ------------------------------------------------------------ converters
    const int t = tid - kConvWarp0 * 32;
    const int r = t & (BN - 1);
    const int is_v = t >> 6;
    const uint16_t* scales = is_v ? a.vs : a.ks;
    const uint32_t codes_base = sbase + (is_v ? kOffVC : kOffKC);
    const uint32_t kv_base = sbase + (is_v ? kOffV : kOffK);
    // this row's scales of tile j + 1 are loaded while tile j is converted
    auto load_sw = [&](int jj, ScaleWords<L>& sw) {
      const int jt = jj * BN + r;
      const int64_t tok = lo + jt;
      if (jj < nkv && jt < Lk && tok >= a.sink_tokens)
        load_scale_words<L>(scales + ((static_cast<int64_t>(b) * a.cache_tokens + tok) * a.H + h) * L::G, sw);
    };
    ScaleWords<L> sw_next;
    load_sw(0, sw_next);
    for (int j = 0; j < nkv; ++j) {
      const int ls = j % NS_LD, ks = j % NS_KV;
      const int jt = j * BN + r;
      const int64_t tok = lo + jt;
      const bool live = jt < Lk;
      const bool coded = live && tok >= a.sink_tokens;
      const ScaleWords<L> sw = sw_next;
      load_sw(j + 1, sw_next);
      if (!mbar_wait_warp(&bars[bLdFull + is_v * NS_LD + ls], (j / NS_LD) & 1, abort, &g_attn_status, lim)) break;
      if (j >= NS_KV &&
          !mbar_wait_warp(&bars[bKvEmpty + is_v * NS_KV + ks], ((j / NS_KV) - 1) & 1, abort, &g_attn_status, lim))
        break;
      const uint32_t dst = kv_base + ks * kKVTile;
      if (!live) {
#pragma unroll
        for (int c = 0; c < 16; ++c) st_shared_v4(dst + tile_off(r, c), make_uint4(0, 0, 0, 0));
      } else if (coded) {
        uint32_t sp[L::G];
        scale_pairs<L>(sw, sp);
        if (KB == 8 && !is_v) {
          // int8 K row: 128 B of codes, SWIZZLE_128B staging
          float sf[L::G];
#pragma unroll
          for (int g = 0; g < L::G; ++g) sf[g] = __uint_as_float(sp[g] << 16);
          deq_row_i8<L>(codes_base + ls * kCodeTileK + r * 128, sf, dst, r, std::make_integer_sequence<int, 8>{});
        } else {
          const uint32_t src = codes_base + ls * (is_v ? kCodeTileV : kCodeTileK) + r * 64;
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 v = ld_shared_v4(src + ((c ^ ((r >> 1) & 3)) << 4));
            w[4 * c] = v.x;
            w[4 * c + 1] = v.y;
            w[4 * c + 2] = v.z;
            w[4 * c + 3] = v.w;
          }
          deq_row<L>(w, sp, dst, r, std::make_integer_sequence<int, 16>{});
        }
      }
      // sink rows were written into the tile by the TMA
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars[bLdEmpty + is_v * NS_LD + ls]);
        mbar_arrive(&bars[bKvFull + is_v * NS_KV + ks]);
      }
    }
  } else if (warp == kProdWarp || warp == kProdWarpV) {
    // ------------------------------------------------------------ TMA producers
    // warp 12: K codes and K sink rows; warp 15: V
    const int pv = warp != kProdWarp;
    if (lane == 0 && !pv) {
      // the Q tiles first (after the barrier set-up above is visible): two
      // 64-column SWIZZLE_128B atoms per tile, the S MMA's A layout
      for (int x = 0; x < nq; ++x) {
        mbar_arrive_expect_tx(&bars[bQReady + x], static_cast<uint32_t>(kQTile));
        tma_load_3d(sbase + kOffQ + x * kQTile, &a.tm_q, h * D, q0 + x * BM, b, &bars[bQReady + x]);
        tma_load_3d(sbase + kOffQ + x * kQTile + kQAtom, &a.tm_q, h * D + 64, q0 + x * BM, b, &bars[bQReady + x]);
      }
    }
    if (lane == 0) {
      const CUtensorMap* tc = pv ? &a.tm_vc : &a.tm_kc;
      const CUtensorMap* tsk = pv ? &a.tm_vs : &a.tm_ks;
      const uint32_t code_tile = pv ? static_cast<uint32_t>(kCodeTileV) : static_cast<uint32_t>(kCodeTileK);
      const uint32_t code_base = sbase + (pv ? kOffVC : kOffKC);
      const uint32_t kv_base = sbase + (pv ? kOffV : kOffK);
      const int code_x = h * (pv ? 64 : (KB == 4 ? 64 : 128));
      int issued = 0;  // tiles whose loads were issued
      for (int j = 0; j < nkv; ++j) {
        const int ls = j % NS_LD, ks = j % NS_KV;
        if (!pv && j == a.stall_tile) break;  // abort test: tile j never arrives
        if (j >= NS_LD &&
            !mbar_wait(&bars[bLdEmpty + pv * NS_LD + ls], ((j / NS_LD) - 1) & 1, abort, &g_attn_status, lim))
          break;
        const int64_t t0 = lo + static_cast<int64_t>(j) * BN;
        const int64_t t1 = lo + min(static_cast<int64_t>(j + 1) * BN, static_cast<int64_t>(Lk));
        const bool has_sink = t0 < a.sink_tokens;
        const bool has_codes = t1 > a.sink_tokens;
        if (has_sink && j >= NS_KV &&
            !mbar_wait(&bars[bKvEmpty + pv * NS_KV + ks], ((j / NS_KV) - 1) & 1, abort, &g_attn_status, lim))
          break;
        const uint32_t bytes = (has_codes ? code_tile : 0u) + (has_sink ? static_cast<uint32_t>(kKVTile) : 0u);
        uint64_t* full = &bars[bLdFull + pv * NS_LD + ls];
        mbar_arrive_expect_tx(full, bytes);
        if (has_codes) {
          const int row = static_cast<int>(static_cast<int64_t>(b) * a.cache_tokens + t0);
          tma_load_2d(code_base + ls * code_tile, tc, code_x, row, full);
        }
        if (has_sink) {
          const int row = static_cast<int>(static_cast<int64_t>(b) * a.sink_tokens + t0);
          const uint32_t d = kv_base + ks * kKVTile;
          tma_load_2d(d, tsk, h * D, row, full);
          tma_load_2d(d + kAtom, tsk, h * D + 64, row, full);
        }
        issued = j + 1;
      }
      // Leave no copy into this CTA's shared memory in flight, also when another
      // thread gave up before consuming it: wait for the last NS_LD tiles issued
      // (each on its own stage, so each parity names one phase) and for the Q
      // tiles. Without an abort they have landed long ago.
      for (int j = max(0, issued - NS_LD); j < issued; ++j)
        mbar_drain(&bars[bLdFull + pv * NS_LD + j % NS_LD], (j / NS_LD) & 1, &g_attn_status, lim);
      if (!pv)
        for (int x = 0; x < nq; ++x) mbar_drain(&bars[bQReady + x], 0, &g_attn_status, lim);
    }
    __syncwarp();
  } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
    // ------------------------------------------------------------ MMA issuers
    const int x = warp - kMmaWarp;
    if (lane == 0 && x < nq) {
      constexpr uint32_t idS = idesc_bf16(BM, BN, 0);
      constexpr uint32_t idPV = idesc_bf16(BM, D, 1);
      const uint32_t tS0 = tmem + kColS + 128 * x, tO = tmem + kColO + 128 * x;
      const uint32_t qaddr = sbase + kOffQ + x * kQTile;
      // S_x(j) into buffer j & 1; Q and K K-major SWIZZLE_128B in shared memory
      auto issue_s = [&](int j) {
        const uint32_t kaddr = sbase + kOffK + (j % NS_KV) * kKVTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_bf16_ss(tS0 + 64 * (j & 1), smem_desc_sw128(qaddr + (kk >> 2) * kQAtom + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw128(kaddr + (kk >> 2) * kAtom + (kk & 3) * 32, 16, 1024), idS, kk > 0);
        mma_commit(&bars[bSFull + 2 * x + (j & 1)]);
      };
      // O_x += P_x(j) V(j): P in TMEM over S_x(j), V MN-major
      auto issue_pv = [&](int j) {
        const uint32_t vaddr = sbase + kOffV + (j % NS_KV) * kKVTile;
        const uint32_t p = tS0 + 64 * (j & 1);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_bf16_ts(tO, p + 8 * kk, smem_desc_sw128(vaddr + kk * 2048, kAtom, 1024), idPV,
                      (j > 0 || kk > 0) ? 1u : 0u);
      };
      auto wait_kv = [&](int j) {
        return mbar_wait(&bars[bKvFull + j % NS_KV], (j / NS_KV) & 1, abort, &g_attn_status, lim);
      };
      bool ok = mbar_wait(&bars[bQReady + x], 0, abort, &g_attn_status, lim) && wait_kv(0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        if (nkv > 1 && (ok = wait_kv(1))) {
          tc_fence_after();
          issue_s(1);
        }
      }
      for (int j = 0; j < nkv && ok; ++j) {
        // V(j) and K(j+2) were converted tiles ago (their stages came free at
        // S(j-2)): confirm them before waiting for P_x(j), off the chain
        // P_x(j) -> PV_x(j) -> S_x(j+2)
        if (!(ok = mbar_wait(&bars[bKvFull + NS_KV + j % NS_KV], (j / NS_KV) & 1, abort, &g_attn_status, lim)))
          break;
        if (j + 2 < nkv && !(ok = wait_kv(j + 2))) break;
        if (!(ok = mbar_wait(&bars[bPFull + 2 * x + (j & 1)], (j >> 1) & 1, abort, &g_attn_status, lim))) break;
        tc_fence_after();
        issue_pv(j);
        if (j + 2 < nkv) {
          // S_x(j+2) into the buffer PV_x(j) is reading: behind it in issue order
          issue_s(j + 2);
        } else if (j + 2 == nkv) {
          mma_commit(&bars[bOReady + x]);  // PV_x(nkv-2): a rescale at the last tile waits for it
        }
      }
      if (ok) mma_commit(&bars[bOFinal + x]);
      // all MMAs issued by this thread have completed before TMEM is released
      mma_commit(&bars[bMmaDone + x]);
      mbar_drain(&bars[bMmaDone + x], 0, &g_attn_status, lim);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (parts > 1) {
    // The part that finishes last merges the unit: every part's partial row is in
    // the workspace (written and fenced before the barrier above), so after the
    // atomic count this CTA reads them all, combines them in base-2 exponent
    // space, normalises and stores the output tile as the whole units do.
    volatile int* last = reinterpret_cast<volatile int*>(smem + kOffMisc + 16);
    if (tid == 0) {
      int is_last = 0;
      if (!*abort) {
        const unsigned old = atomicAdd(&a.ctr[unit], 1u);
        is_last = old == static_cast<unsigned>(parts - 1);
        if (is_last) a.ctr[unit] = 0u;  // ready for the next launch
      }
      *last = is_last;
    }
    __syncthreads();
    if (*last) {
      __threadfence();
      if (warp < 4 * nq) {
        const int x = warp >> 2;
        const int r = tid - x * BM;
        const float4* src = a.ws + ws_slot(a, unit, 0, x) * 33 * BM + r;
        // float4s from one part's slot to the next
        const int64_t pstride = (unit < a.split_full ? 2 : 1) * static_cast<int64_t>(33) * BM;
        float wp[kMaxParts];
        float mx = -INFINITY, lsum = 0.0f;
#pragma unroll
        for (int p = 0; p < kMaxParts; ++p)
          if (p < parts) mx = fmaxf(mx, __ldcg(src + p * pstride + 32 * BM).x);
#pragma unroll
        for (int p = 0; p < kMaxParts; ++p) {
          wp[p] = 0.0f;
          if (p < parts) {
            const float4 ml = __ldcg(src + p * pstride + 32 * BM);
            wp[p] = ex2(ml.x - mx);
            lsum = fmaf(ml.y, wp[p], lsum);
          }
        }
        const float inv = 1.0f / lsum;
        const uint32_t stage = sbase + kOffQ + x * kQTile;
#pragma unroll 1
        for (int ch = 0; ch < 16; ++ch) {  // 8 output channels per 16-byte chunk
          float acc[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
          for (int p = 0; p < kMaxParts; ++p) {
            if (p < parts) {
              const float4 v0 = __ldcg(src + p * pstride + (2 * ch) * BM);
              const float4 v1 = __ldcg(src + p * pstride + (2 * ch + 1) * BM);
              acc[0] = fmaf(v0.x, wp[p], acc[0]);
              acc[1] = fmaf(v0.y, wp[p], acc[1]);
              acc[2] = fmaf(v0.z, wp[p], acc[2]);
              acc[3] = fmaf(v0.w, wp[p], acc[3]);
              acc[4] = fmaf(v1.x, wp[p], acc[4]);
              acc[5] = fmaf(v1.y, wp[p], acc[5]);
              acc[6] = fmaf(v1.z, wp[p], acc[6]);
              acc[7] = fmaf(v1.w, wp[p], acc[7]);
            }
          }
          st_shared_v4(stage + (ch >> 3) * kQAtom + r * 128 + (((ch & 7) ^ (r & 7)) << 4),
                       make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                                  pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv)));
        }
        fence_proxy_async_smem();
      }
      __syncthreads();
      if (tid < nq * BM && (tid & (BM - 1)) == 0) {
        const int x = tid / BM;
        const uint32_t stage = sbase + kOffQ + x * kQTile;
        const int xq = (a.out_head0 + h) * D, yq = q0 + x * BM;
        // destinations in an order rotated by the block index: with peers, the CTAs
        // of a wave then push into every GPU's NVLink ingress at once, not all into one
        for (int i = 0; i < a.n_out; ++i) {
          const int d = (i + static_cast<int>(blockIdx.x)) % a.n_out;
          tma_store_3d(&a.tm_out[d], stage, xq, yq, b);
          tma_store_3d(&a.tm_out[d], stage + kQAtom, xq + 64, yq, b);
        }
        bulk_commit();
        bulk_wait_read_all();
      }
    }
  }
}

// ---------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// 2-D map over `rows` rows of `row_elems` elements (row stride `row_bytes`), box
// box_x x box_y, given swizzle; out-of-range boxes are zero-filled.
static int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t row_elems,
                    uint64_t row_bytes, uint64_t rows, uint32_t box_x, uint32_t box_y, CUtensorMapSwizzle sw,
                    const char* what) {
  EncodeFn fn = encode_fn();
  KVQ_REQUIRE(fn != nullptr, KVQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {row_elems, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KVQ_REQUIRE(r == CUDA_SUCCESS, KVQ_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what, (int)r);
  return KVQ_OK;
}

// 3-D map over an attention output [batch][n_q][heads * D] bf16 (token stride
// tok elements): box 64 columns x 128 tokens x 1 stream, SWIZZLE_128B; tokens
// past n_q are clipped by the map, not written into the next stream.
static int make_out_map(CUtensorMap* m, void* base, uint64_t row_elems, uint64_t tok, uint64_t n_q, uint64_t batch) {
  EncodeFn fn = encode_fn();
  KVQ_REQUIRE(fn != nullptr, KVQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {row_elems, n_q, batch};
  cuuint64_t strides[2] = {tok * 2, tok * 2 * n_q};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(BM), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KVQ_REQUIRE(r == CUDA_SUCCESS, KVQ_ERR_CUDA, "cuTensorMapEncodeTiled(output) failed with %d", (int)r);
  return KVQ_OK;
}

// ---------------------------------------------------------------- wave balance
// How the units of a launch are cut for the last wave (Args: split_full,
// split_single), and the workspace the parts need.
struct SplitPlan {
  int split_full = 0, split_single = 1, units = 0;
  int64_t ws_bytes = 0, ctr_offset = 0;
};

// Makespan, in units of a two-tile CTA's time, of list-scheduling `n_whole`
// two-tile CTAs, then `2 k2` halves, then `P n_single` parts of the one-tile
// CTAs on `sms` SMs, in that order (the order of the block indices). Costs:
// two-tile 1, one-tile 0.82 (its per-tile pace is set by the KV pipeline, not
// by its one Q tile), a part its share plus 0.04 for the partial store and merge.
static double makespan(int n_whole, int k2, int n_single, int P, int sms) {
  std::vector<double> t(static_cast<size_t>(sms), 0.0);
  std::priority_queue<double, std::vector<double>, std::greater<double>> h(t.begin(), t.end());
  auto run = [&](int n, double c) {
    for (int i = 0; i < n; ++i) {
      const double f = h.top();
      h.pop();
      h.push(f + c);
    }
  };
  run(n_whole, 1.0);
  run(2 * k2, 0.5 + 0.04);
  run(P * n_single, P == 1 ? 0.82 : 0.82 / P + 0.04);
  double m = 0.0;
  while (!h.empty()) {
    m = std::max(m, h.top());
    h.pop();
  }
  return m;
}

static SplitPlan plan_split(int64_t n_q, int n_hb, int64_t n_kv, int sms) {
  SplitPlan p;
  const int n_pairs = static_cast<int>((n_q + 2 * BM - 1) / (2 * BM));
  const int n_full = n_q - static_cast<int64_t>(n_pairs - 1) * 2 * BM > BM ? n_pairs : n_pairs - 1;
  const int n_ft = n_full * n_hb, n_s = (n_pairs - n_full) * n_hb;
  const int nkv = static_cast<int>((n_kv + BN - 1) / BN);
  if (nkv < 2 || n_ft + n_s > 64 * sms) return p;  // nothing to split, or the tail is a small share
  struct Key {
    int n_ft, n_s, nkv, sms;
  };
  static std::mutex mu;
  static std::vector<std::pair<Key, SplitPlan>> cache;
  {
    std::lock_guard<std::mutex> g(mu);
    for (auto& e : cache)
      if (e.first.n_ft == n_ft && e.first.n_s == n_s && e.first.nkv == nkv && e.first.sms == sms) return e.second;
  }
  const double base = makespan(n_ft, 0, n_s, 1, sms);
  double best = base;
  int best_k = 0, best_p = 1;
  for (int P = 1; P <= kMaxParts && P <= nkv; P *= 2) {
    if (P > 1 && n_s == 0) break;
    for (int k = 0; k <= std::min(n_ft, 2 * sms); k += 4) {
      const double m = makespan(n_ft - k, k, n_s, P, sms);
      if (m < best - 1e-9) {
        best = m;
        best_k = k;
        best_p = P;
      }
    }
  }
  if (best < base * 0.99) {  // worth the partial stores
    p.split_full = best_k;
    p.split_single = best_p;
    p.units = best_k + (best_p > 1 ? n_s : 0);
    const int64_t slots = static_cast<int64_t>(4) * best_k + (best_p > 1 ? static_cast<int64_t>(n_s) * best_p : 0);
    const int64_t f4 = slots * 33 * BM;
    p.ctr_offset = (f4 * 16 + 255) / 256 * 256;
    p.ws_bytes = p.ctr_offset + static_cast<int64_t>(p.units) * 4;
  }
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() >= 64) cache.erase(cache.begin());
  cache.push_back({Key{n_ft, n_s, nkv, sms}, p});
  return p;
}

static int num_sms() {
  static int sms[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    sms[dev] = n;
  }
  return sms[dev];
}

template <class L, int KB, bool STATS>
int launch(const Args& a, int n_ctas, int batch, cudaStream_t st) {
  constexpr int kSmemBytes = Geo<KB>::kSmemBytes;
  static bool configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<L, KB, STATS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(attention): %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    configured[dev] = true;
  }
  (void)batch;
  cudaError_t e = launch_pdl(attention_kernel<L, KB, STATS>, static_cast<unsigned>(n_ctas), kThreads,
                             kSmemBytes, st, a);
  if (e != cudaSuccess) {
    set_error("kvq_attention: launch failed: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  return check_launch("kvq_attention");
}

template <class L>
int launch_layout(const Args& a, int n_ctas, int batch, cudaStream_t st, int k_bits, bool stats) {
  if (k_bits == 4)
    return stats ? launch<L, 4, true>(a, n_ctas, batch, st) : launch<L, 4, false>(a, n_ctas, batch, st);
  return stats ? launch<L, 8, true>(a, n_ctas, batch, st) : launch<L, 8, false>(a, n_ctas, batch, st);
}

}  // namespace attn
}  // namespace kvq

using namespace kvq;

static int attention_impl(const void* q, int64_t q_token_stride, const void* k_codes, const void* k_scales,
                          const void* k_sink, const void* v_codes, const void* v_scales, const void* v_sink,
                          int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi, void* const* outs,
                          int n_outs, int out_head0, int out_heads, int64_t out_token_stride, int batch, int64_t n_q,
                          int n_heads, int head_dim, const int32_t* chan_band, int n_groups, int k_bits, int v_bits,
                          float softmax_scale, void* stream, bool tma_out, float* stats,
                          long long wait_cycles = sm100::kWaitCycles, int stall_tile = -1,
                          void* workspace = nullptr, int64_t workspace_bytes = 0) {
  KVQ_REQUIRE(head_dim == 128, KVQ_ERR_UNSUPPORTED, "attention supports head_dim 128, got %d", head_dim);
  KVQ_REQUIRE((k_bits == 4 || k_bits == 8) && v_bits == 4, KVQ_ERR_UNSUPPORTED,
              "attention reads int4 or int8 K and int4 V (got %d/%d bits)",
              k_bits, v_bits);
  KVQ_REQUIRE(batch >= 1 && n_heads >= 1 && n_q >= 0 && cache_tokens >= 1, KVQ_ERR_ARG, "bad shape");
  KVQ_REQUIRE(n_heads <= 65535 && batch <= 65535, KVQ_ERR_ARG, "too many heads or streams");
  KVQ_REQUIRE(0 <= lo && lo < hi && hi <= cache_tokens, KVQ_ERR_ARG,
              "window [%lld, %lld) is empty or outside the cache of %lld tokens", (long long)lo, (long long)hi,
              (long long)cache_tokens);
  KVQ_REQUIRE(n_q <= (int64_t)1 << 30, KVQ_ERR_ARG, "too many queries");
  KVQ_REQUIRE((n_q + 2 * attn::BM - 1) / (2 * attn::BM) * n_heads * batch <= 0x7FFFFFFF, KVQ_ERR_ARG,
              "too many queries x heads x streams for one launch");
  KVQ_REQUIRE((int64_t)batch * cache_tokens < ((int64_t)1 << 31) - 256, KVQ_ERR_ARG,
              "batch * cache_tokens must stay below 2^31");
  KVQ_REQUIRE(sink_tokens >= 0 && sink_tokens <= cache_tokens, KVQ_ERR_ARG, "bad sink_tokens");
  KVQ_REQUIRE(sink_tokens == 0 || (k_sink && v_sink), KVQ_ERR_ARG, "sink_tokens > 0 needs both sink buffers");
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  KVQ_REQUIRE(layout != kLayoutGeneric, KVQ_ERR_UNSUPPORTED,
              "attention supports the bands, bands2, bands4, blind32 and blind64 group maps");
  if (n_q == 0) return KVQ_OK;
  KVQ_REQUIRE(outs && n_outs >= 1 && n_outs <= attn::kMaxOut, KVQ_ERR_ARG, "1 to %d outputs, got %d",
              attn::kMaxOut, n_outs);
  KVQ_REQUIRE(out_head0 >= 0 && out_head0 + n_heads <= out_heads, KVQ_ERR_ARG,
              "heads [%d, %d) do not fit an output of %d heads", out_head0, out_head0 + n_heads, out_heads);
  KVQ_REQUIRE(q && k_codes && k_scales && v_codes && v_scales, KVQ_ERR_ARG, "NULL data pointer");
  for (int d = 0; d < n_outs; ++d) KVQ_REQUIRE(outs[d], KVQ_ERR_ARG, "NULL output pointer %d", d);
  KVQ_REQUIRE(q_token_stride >= (int64_t)n_heads * head_dim && out_token_stride >= (int64_t)out_heads * head_dim,
              KVQ_ERR_ARG, "token strides must be >= heads*head_dim");
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KVQ_REQUIRE(al16(q) && q_token_stride % 8 == 0 && out_token_stride % 8 == 0, KVQ_ERR_ALIGN,
              "q and out must be 16-byte aligned with token strides that are multiples of 8");
  for (int d = 0; d < n_outs; ++d) KVQ_REQUIRE(al16(outs[d]), KVQ_ERR_ALIGN, "output %d is not 16-byte aligned", d);
  KVQ_REQUIRE(al16(k_codes) && al16(v_codes) && (!k_sink || al16(k_sink)) && (!v_sink || al16(v_sink)),
              KVQ_ERR_ALIGN, "codes and sink buffers must be 16-byte aligned");
  const int sa = (n_groups * 2) % 8 == 0 ? 8 : (n_groups * 2) % 4 == 0 ? 4 : 2;
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(k_scales) % sa) == 0 && (reinterpret_cast<uintptr_t>(v_scales) % sa) == 0,
              KVQ_ERR_ALIGN, "scales must be %d-byte aligned for %d groups", sa, n_groups);
  int rc = require_sm100();
  if (rc) return rc;

  attn::Args a;
  memset(&a, 0, sizeof(a));
  const uint64_t rows = static_cast<uint64_t>(batch) * cache_tokens;
  const uint64_t kcw = k_bits == 4 ? 64 : 128;  // K code bytes per (token, head)
  rc = attn::make_map(&a.tm_kc, k_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)n_heads * kcw,
                      (uint64_t)n_heads * kcw, rows, static_cast<uint32_t>(kcw), attn::BN,
                      k_bits == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, "k codes");
  if (rc) return rc;
  rc = attn::make_map(&a.tm_vc, v_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)n_heads * 64,
                      (uint64_t)n_heads * 64, rows, 64, attn::BN, CU_TENSOR_MAP_SWIZZLE_64B, "v codes");
  if (rc) return rc;
  if (sink_tokens > 0) {
    const uint64_t srows = static_cast<uint64_t>(batch) * sink_tokens;
    rc = attn::make_map(&a.tm_ks, k_sink, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)n_heads * 128,
                        (uint64_t)n_heads * 256, srows, 64, attn::BN, CU_TENSOR_MAP_SWIZZLE_128B, "k sink");
    if (rc) return rc;
    rc = attn::make_map(&a.tm_vs, v_sink, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)n_heads * 128,
                        (uint64_t)n_heads * 256, srows, 64, attn::BN, CU_TENSOR_MAP_SWIZZLE_128B, "v sink");
    if (rc) return rc;
  }
  rc = attn::make_out_map(&a.tm_q, const_cast<void*>(q), static_cast<uint64_t>(n_heads) * head_dim,
                          static_cast<uint64_t>(q_token_stride), static_cast<uint64_t>(n_q),
                          static_cast<uint64_t>(batch));
  if (rc) return rc;
  a.q = static_cast<const uint16_t*>(q);
  a.q_tok_stride = q_token_stride;
  a.q_batch_stride = q_token_stride * n_q;
  a.ks = static_cast<const uint16_t*>(k_scales);
  a.vs = static_cast<const uint16_t*>(v_scales);
  a.cache_tokens = cache_tokens;
  a.sink_tokens = sink_tokens;
  a.lo = lo;
  a.Lk = static_cast<int>(hi - lo);
  a.Lq = static_cast<int>(n_q);
  a.H = n_heads;
  for (int d = 0; d < n_outs; ++d) a.out[d] = static_cast<uint16_t*>(outs[d]);
  a.tma_out = tma_out ? 1 : 0;
  KVQ_REQUIRE(stats == nullptr || (reinterpret_cast<uintptr_t>(stats) & 15) == 0, KVQ_ERR_ALIGN,
              "stats must be 16-byte aligned");
  a.stats = stats;
  if (tma_out) {
    for (int d = 0; d < n_outs; ++d) {
      rc = attn::make_out_map(&a.tm_out[d], outs[d], static_cast<uint64_t>(out_heads) * head_dim,
                              static_cast<uint64_t>(out_token_stride), static_cast<uint64_t>(n_q),
                              static_cast<uint64_t>(batch));
      if (rc) return rc;
    }
  }
  a.n_out = n_outs;
  a.out_head0 = out_head0;
  a.o_tok_stride = out_token_stride;
  a.o_batch_stride = out_token_stride * n_q;
  const float sc = softmax_scale > 0.0f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  a.scale_log2 = sc * 1.4426950408889634f;
  a.wait_cycles = wait_cycles;
  a.stall_tile = stall_tile;
  a.n_hb = n_heads * batch;
  a.split_full = 0;
  a.split_single = 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n_pairs = (n_q + 2 * attn::BM - 1) / (2 * attn::BM);
  int ctas = static_cast<int>(n_pairs * a.n_hb);
  if (workspace && stats == nullptr && stall_tile < 0) {
    const attn::SplitPlan sp = attn::plan_split(n_q, a.n_hb, hi - lo, attn::num_sms());
    if (sp.units > 0 && workspace_bytes >= sp.ws_bytes) {
      KVQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, KVQ_ERR_ALIGN,
                  "the workspace must be 256-byte aligned");
      a.split_full = sp.split_full;
      a.split_single = sp.split_single;
      a.ws = static_cast<float4*>(workspace);
      a.ctr = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + sp.ctr_offset);
      const int64_t n_full = n_q - (n_pairs - 1) * 2 * attn::BM > attn::BM ? n_pairs : n_pairs - 1;
      ctas = static_cast<int>(n_full * a.n_hb + sp.split_full + (n_pairs - n_full) * a.n_hb * sp.split_single);
      cudaError_t e = cudaMemsetAsync(a.ctr, 0, static_cast<size_t>(sp.units) * 4, st);
      if (e != cudaSuccess) {
        set_error("kvq_attention: clearing the workspace counters failed: %s", cudaGetErrorString(e));
        return KVQ_ERR_CUDA;
      }
    }
  }
  switch (layout) {
    case kLayoutBands: return attn::launch_layout<LayoutBands>(a, ctas, batch, st, k_bits, stats != nullptr);
    case kLayoutBands2: return attn::launch_layout<LayoutBands2>(a, ctas, batch, st, k_bits, stats != nullptr);
    case kLayoutBands4: return attn::launch_layout<LayoutBands4>(a, ctas, batch, st, k_bits, stats != nullptr);
    case kLayoutBlind32: return attn::launch_layout<LayoutBlind32>(a, ctas, batch, st, k_bits, stats != nullptr);
    case kLayoutBlind64: return attn::launch_layout<LayoutBlind64>(a, ctas, batch, st, k_bits, stats != nullptr);
    default: break;
  }
  set_error("internal: unhandled layout %d", layout);
  return KVQ_ERR_UNSUPPORTED;
}

// The output is stored through the TMA epilogue (full 256-byte rows, two tensor
// stores per Q tile); it is measurably faster than per-thread 16-byte stores.
extern "C" int kvq_attention(const void* q, int64_t q_token_stride, const void* k_codes, const void* k_scales,
                             const void* k_sink, const void* v_codes, const void* v_scales, const void* v_sink,
                             int64_t cache_tokens, int64_t sink_tokens, int64_t lo, int64_t hi, void* out,
                             int64_t out_token_stride, int batch, int64_t n_q, int n_heads, int head_dim,
                             const int32_t* chan_band, int n_groups, int k_bits, int v_bits, float softmax_scale,
                             void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  void* outs[1] = {out};
  if (n_q > 0 && !out) {
    set_error("NULL data pointer");
    return KVQ_ERR_ARG;
  }
  return attention_impl(q, q_token_stride, k_codes, k_scales, k_sink, v_codes, v_scales, v_sink, cache_tokens,
                        sink_tokens, lo, hi, outs, 1, 0, n_heads, out_token_stride, batch, n_q, n_heads, head_dim,
                        chan_band, n_groups, k_bits, v_bits, softmax_scale, stream, true, nullptr, sm100::kWaitCycles,
                        -1, workspace, workspace_bytes);
}

extern "C" int kvq_attention_workspace_bytes(int batch, int64_t n_q, int n_heads, int64_t n_kv_tokens,
                                             int64_t* bytes) {
  clear_error();
  KVQ_REQUIRE(bytes && batch >= 1 && n_heads >= 1 && n_q >= 0 && n_kv_tokens >= 0, KVQ_ERR_ARG, "bad shape");
  *bytes = 0;
  if (n_q == 0 || n_kv_tokens == 0) return KVQ_OK;
  int rc = require_sm100();
  if (rc) return rc;
  *bytes = attn::plan_split(n_q, n_heads * batch, n_kv_tokens, attn::num_sms()).ws_bytes;
  return KVQ_OK;
}

// ------------------------------------------------------- no-allocation variant
// Some callers cannot hand the launch a workspace: a frame loop in which a
// cudaMalloc or cudaFree would synchronize the device and stall the frame, or a
// host framework that owns the device memory through its own pool and gives a
// plugin no way to ask for more. For them the wave-balance workspace lives in the
// library itself: a fixed array in device memory, one instance per device, which
// no call allocates. Calls on one device share it, so calls that may overlap on
// the GPU (unordered streams) race; order them on one stream.
static constexpr int64_t kNoAllocScratchBytes = KVQ_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

// Device address of g_attn_scratch on the current device. The first call on a
// device looks it up (cudaGetSymbolAddress, which loads the module if it is not
// loaded yet); later calls read the cached address.
static int noalloc_scratch(void** ptr) {
  static std::mutex mu;
  static void* addr[64];
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  KVQ_REQUIRE(e == cudaSuccess, KVQ_ERR_CUDA, "kvq_attention_noalloc: cudaGetDevice failed: %s",
              cudaGetErrorString(e));
  KVQ_REQUIRE(dev >= 0 && dev < 64, KVQ_ERR_DEVICE, "kvq_attention_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    KVQ_REQUIRE(e == cudaSuccess && p != nullptr, KVQ_ERR_CUDA,
                "kvq_attention_noalloc: looking up the scratch on device %d failed: %s", dev,
                cudaGetErrorString(e));
    addr[dev] = p;
  }
  *ptr = addr[dev];
  return KVQ_OK;
}

extern "C" int kvq_attention_noalloc(const void* q, int64_t q_token_stride, const void* k_codes,
                                     const void* k_scales, const void* k_sink, const void* v_codes,
                                     const void* v_scales, const void* v_sink, int64_t cache_tokens,
                                     int64_t sink_tokens, int64_t lo, int64_t hi, void* out,
                                     int64_t out_token_stride, int batch, int64_t n_q, int n_heads, int head_dim,
                                     const int32_t* chan_band, int n_groups, int k_bits, int v_bits,
                                     float softmax_scale, void* stream) {
  clear_error();
  int rc = require_sm100();
  if (rc) return rc;
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  void* outs[1] = {out};
  if (n_q > 0 && !out) {
    set_error("NULL data pointer");
    return KVQ_ERR_ARG;
  }
  // the shape checks attention_impl makes first, so that the plan below sees a sane shape
  const bool planned = n_q > 0 && batch >= 1 && n_heads >= 1 && batch <= 65535 && n_heads <= 65535 &&
                       n_q <= ((int64_t)1 << 30) && 0 <= lo && lo < hi &&
                       (n_q + 2 * attn::BM - 1) / (2 * attn::BM) * n_heads * batch <= 0x7FFFFFFF;
  if (planned) {
    const int64_t need = attn::plan_split(n_q, n_heads * batch, hi - lo, attn::num_sms()).ws_bytes;
    KVQ_REQUIRE(need <= kNoAllocScratchBytes, KVQ_ERR_UNSUPPORTED,
                "kvq_attention_noalloc: this shape needs %lld bytes of scratch, more than the %lld the library "
                "holds; call kvq_attention with a workspace of kvq_attention_workspace_bytes() bytes",
                (long long)need, (long long)kNoAllocScratchBytes);
  }
  return attention_impl(q, q_token_stride, k_codes, k_scales, k_sink, v_codes, v_scales, v_sink, cache_tokens,
                        sink_tokens, lo, hi, outs, 1, 0, n_heads, out_token_stride, batch, n_q, n_heads, head_dim,
                        chan_band, n_groups, k_bits, v_bits, softmax_scale, stream, true, nullptr, sm100::kWaitCycles,
                        -1, scratch, kNoAllocScratchBytes);
}

extern "C" int kvq_attention_stats(const void* q, int64_t q_token_stride, const void* k_codes,
                                   const void* k_scales, const void* k_sink, const void* v_codes,
                                   const void* v_scales, const void* v_sink, int64_t cache_tokens,
                                   int64_t sink_tokens, int64_t lo, int64_t hi, void* out, int64_t out_token_stride,
                                   float* stats, int batch, int64_t n_q, int n_heads, int head_dim,
                                   const int32_t* chan_band, int n_groups, int k_bits, int v_bits,
                                   float softmax_scale, void* stream) {
  clear_error();
  void* outs[1] = {out};
  if (n_q > 0 && (!out || !stats)) {
    set_error("NULL output or stats pointer");
    return KVQ_ERR_ARG;
  }
  return attention_impl(q, q_token_stride, k_codes, k_scales, k_sink, v_codes, v_scales, v_sink, cache_tokens,
                        sink_tokens, lo, hi, outs, 1, 0, n_heads, out_token_stride, batch, n_q, n_heads, head_dim,
                        chan_band, n_groups, k_bits, v_bits, softmax_scale, stream, false, stats);
}

extern "C" int kvq_attention_gather(const void* q, int64_t q_token_stride, const void* k_codes,
                                    const void* k_scales, const void* k_sink, const void* v_codes,
                                    const void* v_scales, const void* v_sink, int64_t cache_tokens,
                                    int64_t sink_tokens, int64_t lo, int64_t hi, void* const* outs, int n_outs,
                                    int out_head0, int out_heads, int64_t out_token_stride, int batch, int64_t n_q,
                                    int n_heads, int head_dim, const int32_t* chan_band, int n_groups, int k_bits,
                                    int v_bits, float softmax_scale, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
  clear_error();
  return attention_impl(q, q_token_stride, k_codes, k_scales, k_sink, v_codes, v_scales, v_sink, cache_tokens,
                        sink_tokens, lo, hi, outs, n_outs, out_head0, out_heads, out_token_stride, batch, n_q,
                        n_heads, head_dim, chan_band, n_groups, k_bits, v_bits, softmax_scale, stream, true, nullptr,
                        sm100::kWaitCycles, -1, workspace, workspace_bytes);
}

namespace kvq {
constexpr int kMaxRanks = 64;
struct BarrierArgs {
  unsigned* counters[kMaxRanks];  // every rank's counter (this GPU's own and its peers', mapped)
  int n, self;
  unsigned target;
  long long limit;
};

// One thread: every write of the kernels before this one on the stream has
// completed (kernel boundary); release-add 1 to every rank's counter, then wait
// (acquire) until this rank's counter reaches the target, i.e. until every rank
// has passed the same point of its stream. Gives up after `limit` cycles and
// raises the device status word instead of hanging.
__global__ void gather_barrier_kernel(const __grid_constant__ BarrierArgs a) {
  sm100::fence_proxy_async_global();
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int d = 0; d < a.n; ++d) sm100::red_release_sys_add(a.counters[d], 1u);
  const unsigned* mine = a.counters[a.self];
  const long long t0 = clock64();
  while (static_cast<int>(sm100::ld_acquire_sys(mine) - a.target) < 0) {
    if (clock64() - t0 > a.limit) {
      atomicExch(&g_attn_status, sm100::kDevTimeout);
      return;
    }
    __nanosleep(128);
  }
  sm100::fence_proxy_async_global();
}
}  // namespace kvq

extern "C" int kvq_gather_barrier(unsigned int* const* counters, int n_ranks, int self, unsigned int target,
                                  int64_t wait_cycles, void* stream) {
  clear_error();
  KVQ_REQUIRE(counters && n_ranks >= 1 && n_ranks <= kvq::kMaxRanks && self >= 0 && self < n_ranks, KVQ_ERR_ARG,
              "1 to %d counters and 0 <= self < n_ranks", kvq::kMaxRanks);
  KVQ_REQUIRE(wait_cycles >= 1000 && wait_cycles <= sm100::kWaitCycles, KVQ_ERR_ARG,
              "wait_cycles must lie in [1000, %lld]", (long long)sm100::kWaitCycles);
  kvq::BarrierArgs a;
  memset(&a, 0, sizeof(a));
  for (int d = 0; d < n_ranks; ++d) {
    KVQ_REQUIRE(counters[d] && (reinterpret_cast<uintptr_t>(counters[d]) & 3) == 0, KVQ_ERR_ARG,
                "counter %d is NULL or not 4-byte aligned", d);
    a.counters[d] = counters[d];
  }
  a.n = n_ranks;
  a.self = self;
  a.target = target;
  a.limit = wait_cycles;
  int rc = require_sm100();
  if (rc) return rc;
  kvq::gather_barrier_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("kvq_gather_barrier");
}

extern "C" int kvq_test_attention_timeout(const void* q, int64_t q_token_stride, const void* k_codes,
                                          const void* k_scales, const void* k_sink, const void* v_codes,
                                          const void* v_scales, const void* v_sink, int64_t cache_tokens,
                                          int64_t sink_tokens, int64_t lo, int64_t hi, void* out,
                                          int64_t out_token_stride, int batch, int64_t n_q, int n_heads, int head_dim,
                                          const int32_t* chan_band, int n_groups, int k_bits, int v_bits,
                                          float softmax_scale, int stall_tile, int64_t wait_cycles, void* stream) {
  clear_error();
  KVQ_REQUIRE(stall_tile >= 0, KVQ_ERR_ARG, "stall_tile must be >= 0");
  KVQ_REQUIRE(wait_cycles >= 1000 && wait_cycles <= sm100::kWaitCycles, KVQ_ERR_ARG,
              "wait_cycles must lie in [1000, %lld]", (long long)sm100::kWaitCycles);
  void* outs[1] = {out};
  KVQ_REQUIRE(n_q > 0 && out, KVQ_ERR_ARG, "NULL output or no queries");
  return attention_impl(q, q_token_stride, k_codes, k_scales, k_sink, v_codes, v_scales, v_sink, cache_tokens,
                        sink_tokens, lo, hi, outs, 1, 0, n_heads, out_token_stride, batch, n_q, n_heads, head_dim,
                        chan_band, n_groups, k_bits, v_bits, softmax_scale, stream, true, nullptr, wait_cycles,
                        stall_tile);
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
