// Quantize-on-append / rebuild and dequantize kernels (sm_100a) + their C ABI.
//
// Reference semantics: QuantKVTensor._quantize / _dequantize (quant_kv.py:142-176),
// torch path, bit-exact. The reference's Triton kernels (quant_kv_kernels.py:33-84)
// round ties away from zero and are NOT the parity target.
//
// Quantize, specialised layouts (head_dim 128): persistent CTAs of 128 threads
// (three per SM for int4 codes, two for int8) walk 128-row tiles of (token, head) rows with a grid stride:
//   1. each thread keeps the next tile's input in flight (cp.async, 16 bytes per
//      copy, 2 stages), chunk c of row r stored at slot c ^ (r & 7) so that the
//      per-row reads of step 2 are bank-conflict free;
//   2. thread r owns row r: 64 bf16x2 words in registers, per-group absmax on
//      packed bf16x2 (NaN-propagating), the group scale amax / qmax by two FMAs
//      (equal to the IEEE divide for every bf16 amax, kvqo_check_scale_div), one
//      reciprocal per group (approximation + Newton step, within one ulp), then
//      per element the
//      division-free code
//        y0 = x*r, rem = fma(-y0, s, x), y = fma(rem, r, y0), code = rne(y)
//      which equals rne(x / s) for every finite bf16 pair (x, amax) with
//      amax >= 2^-100 (kvqo_check_fast_codes); other groups use the exact divide;
//      rne and the +8 / +128 offset come from one add of a magic constant;
//   3. codes and scales are staged in shared memory and written out with
//      coalesced stores; rows inside the sink are copied to the bf16 sink buffer
//      from the staged input.
// Any other group map runs quantize_rows_generic (one warp per row, shared-memory
// atomics for the per-group max), with the same results.
#include <utility>

#include "kvq_common.cuh"

namespace kvq {

constexpr int kQT = 128;  // threads per CTA = rows per tile (dequantize)
constexpr int kQR = 128;  // threads per CTA = rows per tile (quantize)
constexpr int kQD = 128;  // head_dim of the specialised kernels

struct QuantArgs {
  const uint16_t* x;
  int64_t x_token_stride;  // elements
  uint8_t* codes;
  uint16_t* scales;
  uint16_t* sink;
  int64_t n_rows;     // n_tokens * H
  int64_t sink_rows;  // rows of x that are also copied to sink
  int H;
  int rows_contig;  // x_token_stride == H * D
  // fused rotary embedding (kvq_rope_quantize): pair i of a row rotates by
  // freqs[pos[t][axis(i)]][i] = (cos, sin), fp64, axis 0/1/2 for pairs [0,22)/[22,43)/[43,64)
  const double2* freqs;
  const int* pos;  // [n_tokens][3]
  int max_pos;
};

// Up to kMaxTensors tensors of identical shape quantized by one launch (the
// layers x {K, V} of a rebuild); tile t of the launch is tile t % tiles_per of
// tensor t / tiles_per.
constexpr int kMaxTensors = 96;
struct QuantBatch {
  QuantArgs t[kMaxTensors];
  int n;
  int64_t tiles_per;
  __device__ __forceinline__ const QuantArgs& tensor(int64_t i) const { return t[i]; }
};
// One tensor: the small parameter block of a plain launch (no indexed lookups).
struct QuantOne {
  QuantArgs a;
  int64_t tiles_per;
  __device__ __forceinline__ const QuantArgs& tensor(int64_t) const { return a; }
};

__device__ __forceinline__ const uint16_t* x_row_ptr(const QuantArgs& a, int64_t row, int D) {
  if (a.rows_contig) return a.x + row * D;
  int64_t t = row / a.H;
  int h = static_cast<int>(row - t * a.H);
  return a.x + t * a.x_token_stride + static_cast<int64_t>(h) * D;
}

// Absolute values of a bf16x2 word, max'ed into m with NaN propagation.
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t m, uint32_t w) {
  uint32_t a = w & 0x7FFF7FFFu;
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(a));
  return r;
}

// Division-free code of x: returns the bit pattern of rne(x/s) + magic, whose low
// byte is the offset code (see file comment). `fast` groups only.
__device__ __forceinline__ uint32_t code_fast(float x, float s, float r, float magic) {
  float y0 = __fmul_rn(x, r);
  float rem = __fmaf_rn(-y0, s, x);
  float y = __fmaf_rn(rem, r, y0);
  return __float_as_uint(__fadd_rn(y, magic));
}

// Reference formula with the IEEE divide; clamps so non-finite inputs give codes
// in range (they are outside the parity contract).
__device__ __forceinline__ uint32_t code_exact(float x, float s, float qmax, float magic) {
  float y = __fdiv_rn(x, s);
  y = fminf(fmaxf(y, -qmax), qmax);
  return __float_as_uint(__fadd_rn(y, magic));
}

template <int BITS>
struct QuantConsts {
  static constexpr int kQmax = (1 << (BITS - 1)) - 1;
  // 1.5 * 2^23 + offset: adding it rounds to the nearest even integer and puts
  // code + offset in the low bits of the result.
  static constexpr float kMagic = 12582912.0f + (BITS == 4 ? 8.0f : 128.0f);
  static constexpr int kCodeBytes = BITS == 4 ? kQD / 2 : kQD;  // per row
};

// Group scale s = amax / qmax without a divide: q0 = amax * r, rem = amax - q0 * qmax
// (FMA), s = q0 + rem * r (FMA), r = RN(1/qmax). Equal to the IEEE quotient for
// every positive finite bf16 amax (exhaustively checked by the oracle's
// kvqo_check_scale_div); non-finite amax take the IEEE divide.
template <int QMAX>
__device__ __forceinline__ float group_scale(float amax) {
  if (!(amax <= 3.0e38f)) return __fdiv_rn(amax, static_cast<float>(QMAX));
  const float r = QMAX == 7 ? 0.142857149243354797f : 0.00787401571869850159f;
  const float q0 = __fmul_rn(amax, r);
  const float rem = __fmaf_rn(-q0, static_cast<float>(QMAX), amax);
  return __fmaf_rn(rem, r, q0);
}

// __byte_perm selectors that replace byte p of the first operand with byte 0 of
// the second and keep the other three
__device__ constexpr uint32_t kInsertByte[4] = {0x3214u, 0x3240u, 0x3410u, 0x4210u};

template <int LO, int HI, int BITS, int G_INDEX>
__device__ __forceinline__ void quant_group(const uint32_t (&w)[64], uint32_t (&ow)[BITS == 4 ? 16 : 32],
                                            uint16_t& scale_out, uint32_t& slow_mask) {
  using C = QuantConsts<BITS>;
  static_assert(LO % 2 == 0 && HI % 2 == 0 && LO < HI, "groups must start and end on even channels");
  uint32_t m = 0;
#pragma unroll
  for (int k = LO / 2; k < HI / 2; ++k) m = absmax_bf16x2(m, w[k]);
  float amax;
  {
    uint32_t lo = m << 16, hi = m & 0xFFFF0000u;
    float a = __uint_as_float(lo), b = __uint_as_float(hi);
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(amax) : "f"(a), "f"(b));  // NaN if either is NaN
  }
  float s = group_scale<C::kQmax>(amax);
  s = (s > 0.0f) ? s : 1.0f;  // quant_kv.py:152 (also maps NaN to 1, like torch.where)
  scale_out = f32_to_bf16_bits(s);
  // groups with a tiny or non-finite amax are recomputed with the IEEE divide by
  // quant_fix_slow after staging; the fast chain below still runs for them (any
  // value it produces is overwritten)
  if (!((amax >= 0x1p-100f) && (amax <= 3.0e38f))) slow_mask |= 1u << G_INDEX;
  // reciprocal within one ulp of 1/s: hardware approximation + one Newton step
  // (the code formula holds for any such r, kvqo_check_fast_codes_rcp)
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
  r = __fmaf_rn(r, __fmaf_rn(-s, r, 1.0f), r);
  // the per-element chain on packed f32x2: two channels per instruction
  const float2 r2 = make_float2(r, r), ns2 = make_float2(-s, -s);
  const float2 mg2 = make_float2(C::kMagic, C::kMagic);
#pragma unroll
  for (int k = LO / 2; k < HI / 2; ++k) {
    const float2 x = make_float2(bf16lo_to_f32(w[k]), bf16hi_to_f32(w[k]));
    const float2 y0 = __fmul2_rn(x, r2);
    const float2 rem = __ffma2_rn(y0, ns2, x);
    const float2 t = __fadd2_rn(__ffma2_rn(rem, r2, y0), mg2);
    const uint32_t c0 = __float_as_uint(t.x), c1 = __float_as_uint(t.y);
    if constexpr (BITS == 4) {
      // low byte of c0 + 16 * c1 is the packed pair (code bytes are < 16)
      const uint32_t pair = c0 + (c1 << 4);
      ow[k >> 2] = __byte_perm(ow[k >> 2], pair, kInsertByte[k & 3]);
    } else {
      const uint32_t half = __byte_perm(c0, c1, 0x0040);
      ow[k >> 1] = __byte_perm(ow[k >> 1], half, (k & 1) ? 0x5410u : 0x3254u);
    }
  }
}

template <class L, int BITS, int... Gs>
__device__ __forceinline__ void quant_row(const uint32_t (&w)[64], uint32_t (&ow)[BITS == 4 ? 16 : 32],
                                          uint16_t (&sc)[L::G], uint32_t& slow_mask,
                                          std::integer_sequence<int, Gs...>) {
  (quant_group<L::E[Gs], L::E[Gs + 1], BITS, Gs>(w, ow, sc[Gs], slow_mask), ...);
}

template <class L, int... Is>
__device__ __forceinline__ void fill_edges(int (&e)[L::G + 1], std::integer_sequence<int, Is...>) {
  ((e[Is] = std::integral_constant<int, L::E[Is]>::value), ...);
}

// Rare path: recomputes the codes of the groups flagged in slow_mask (amax below
// 2^-100 or not finite) with the reference formula, IEEE divide and clamp, from
// the row in the swizzled input stage, and patches the staged codes.
template <int BITS>
__device__ __noinline__ void quant_fix_slow(const uint4* tin_row, int r, uint32_t slow_mask, const int* edges,
                                            const uint16_t* scales_row, uint4* codes_row) {
  using C = QuantConsts<BITS>;
  const float q = static_cast<float>(C::kQmax);
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(tin_row);
  uint8_t* cb = reinterpret_cast<uint8_t*>(codes_row);
  for (int g = 0; slow_mask; ++g, slow_mask >>= 1) {
    if (!(slow_mask & 1u)) continue;
    // the unrounded fp32 scale of the group, as the main path computed it
    float amax = 0.0f;
    bool nan = false;
    for (int c = edges[g]; c < edges[g + 1]; ++c) {
      const int chunk = c >> 3, e = c & 7;
      const float x = bf16_bits_to_f32(xr[((chunk ^ (r & 7)) << 3) + e]);
      nan |= (x != x);
      amax = fmaxf(amax, fabsf(x));
    }
    if (nan) amax = __uint_as_float(0x7FC00000u);
    float s = __fdiv_rn(amax, q);
    s = (s > 0.0f) ? s : 1.0f;
    for (int c = edges[g]; c < edges[g + 1]; ++c) {
      const int chunk = c >> 3, e = c & 7;
      const float x = bf16_bits_to_f32(xr[((chunk ^ (r & 7)) << 3) + e]);
      const uint32_t code = code_exact(x, s, q, C::kMagic) & 0xFFu;
      if constexpr (BITS == 4) {
        const int byte = c >> 1, chunk16 = byte >> 4;
        const int slot = chunk16 ^ ((r >> 1) & 3);
        uint8_t& b = cb[(slot << 4) + (byte & 15)];
        b = (c & 1) ? static_cast<uint8_t>((b & 0x0F) | (code << 4)) : static_cast<uint8_t>((b & 0xF0) | code);
      } else {
        const int chunk16 = c >> 4;
        const int slot = chunk16 ^ (r & 7);
        cb[(slot << 4) + (c & 15)] = static_cast<uint8_t>(code);
      }
    }
    (void)scales_row;
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int BITS>
struct PipeCfg {
  static constexpr int kStages = 2;  // one tile in flight per CTA, three CTAs per SM (int4)
  static constexpr int kMaxPerSm = 3;
};

template <class L, int BITS>
constexpr int pipe_smem_bytes() {
  return PipeCfg<BITS>::kStages * kQR * 256 + kQR * QuantConsts<BITS>::kCodeBytes + ((kQR * L::G * 2 + 15) / 16) * 16;
}

// Rotary embedding of one channel pair (two bf16 in one word) as the upstream
// complex128 product (x0 + i x1)(cos + i sin) = (x0 cos - x1 sin) + i (x0 sin +
// x1 cos), rounded to fp32 and then to bf16 (the upstream result is float32 and
// the cache stores bf16). Products and sums are separate IEEE fp64 operations.
__device__ __forceinline__ uint32_t rope_pair(uint32_t w, double2 cs) {
  const double x0 = static_cast<double>(__uint_as_float(w << 16));
  const double x1 = static_cast<double>(__uint_as_float(w & 0xFFFF0000u));
  const double y0 = __dsub_rn(__dmul_rn(x0, cs.x), __dmul_rn(x1, cs.y));
  const double y1 = __dadd_rn(__dmul_rn(x0, cs.y), __dmul_rn(x1, cs.x));
  return pack_bf16x2(__double2float_rn(y0), __double2float_rn(y1));
}

// Rotary embedding of one staged row in place (16 chunks of 4 pairs, XOR-
// swizzled), two chunks per step: the pairs of a step are independent
// chains (two conversions to fp64, two products, a sum, a conversion back), so
// more of them per step hide more of each chain's latency. The (cos, sin) loads
// go through the read-only path and the stage through explicit shared-memory
// accesses, so that the next step's loads are issued before this step's stores.
constexpr int kRopeChunks = 2;
__device__ __forceinline__ void rope_row(const QuantArgs& a, int64_t token, uint32_t trow, int r) {
  constexpr int NP = 4 * kRopeChunks;  // pairs per step
  const int* pp = a.pos + token * 3;
  const int p0 = min(max(__ldg(pp), 0), a.max_pos - 1), p1 = min(max(__ldg(pp + 1), 0), a.max_pos - 1),
            p2 = min(max(__ldg(pp + 2), 0), a.max_pos - 1);  // out-of-range positions clamp
  const double2* f0 = a.freqs + static_cast<int64_t>(p0) * 64;
  const double2* f1 = a.freqs + static_cast<int64_t>(p1) * 64;
  const double2* f2 = a.freqs + static_cast<int64_t>(p2) * 64;
  auto fetch = [&](int i) { return __ldg((i < 22 ? f0 : (i < 43 ? f1 : f2)) + i); };
  double2 cs[2][NP];
#pragma unroll
  for (int k = 0; k < NP; ++k) cs[0][k] = fetch(k);
#pragma unroll
  for (int st = 0; st < 64 / NP; ++st) {
    if (st + 1 < 64 / NP) {
#pragma unroll
      for (int k = 0; k < NP; ++k) cs[(st + 1) & 1][k] = fetch(NP * (st + 1) + k);
    }
    uint32_t w[NP];
#pragma unroll
    for (int h = 0; h < kRopeChunks; ++h) {
      const uint32_t addr = trow + (((kRopeChunks * st + h) ^ (r & 7)) << 4);
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w[4 * h]), "=r"(w[4 * h + 1]), "=r"(w[4 * h + 2]), "=r"(w[4 * h + 3])
                   : "r"(addr));
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) w[k] = rope_pair(w[k], cs[st & 1][k]);
#pragma unroll
    for (int h = 0; h < kRopeChunks; ++h) {
      const uint32_t addr = trow + (((kRopeChunks * st + h) ^ (r & 7)) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * h]), "r"(w[4 * h + 1]),
                   "r"(w[4 * h + 2]), "r"(w[4 * h + 3])
                   : "memory");
    }
  }
}

// One staged tile (kQR rows, XOR-swizzled in tin): thread tid < nrows quantizes
// row tid into the codes / scales staging buffers; after a barrier of the CTA,
// threads [0, kQR) store the tile's codes, scales and sink rows.
template <class L, int BITS>
__device__ __forceinline__ void quant_tile(const QuantArgs& a, int64_t row0, int nrows, const uint4* tin,
                                           uint4* sm_codes, uint16_t* sm_sc, int tid) {
  using C = QuantConsts<BITS>;
  constexpr int G = L::G;
  constexpr int CW = C::kCodeBytes;
  constexpr int CCH = CW / 16;
  if (tid < nrows) {
    uint32_t w[64];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = tin[tid * 16 + (c ^ (tid & 7))];
      w[4 * c + 0] = v.x;
      w[4 * c + 1] = v.y;
      w[4 * c + 2] = v.z;
      w[4 * c + 3] = v.w;
    }
    uint32_t ow[BITS == 4 ? 16 : 32];
#pragma unroll
    for (int q = 0; q < (BITS == 4 ? 16 : 32); ++q) ow[q] = 0;
    uint16_t sc[G];
    uint32_t slow_mask = 0;
    quant_row<L, BITS>(w, ow, sc, slow_mask, std::make_integer_sequence<int, G>{});
#pragma unroll
    for (int c = 0; c < CCH; ++c) {
      const int slot = (BITS == 4) ? (c ^ ((tid >> 1) & 3)) : (c ^ (tid & 7));
      sm_codes[tid * CCH + slot] = make_uint4(ow[4 * c], ow[4 * c + 1], ow[4 * c + 2], ow[4 * c + 3]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) sm_sc[tid * G + g] = sc[g];
    if (slow_mask) {
      int edges[G + 1];
      fill_edges<L>(edges, std::make_integer_sequence<int, G + 1>{});
      quant_fix_slow<BITS>(tin + tid * 16, tid, slow_mask, edges, sm_sc + tid * G, sm_codes + tid * CCH);
    }
  }
  __syncthreads();
  {
    uint4* dst = reinterpret_cast<uint4*>(a.codes + row0 * CW);
    for (int i = tid; i < nrows * CCH; i += kQR) {
      const int r = i / CCH, c = i % CCH;
      const int slot = (BITS == 4) ? (c ^ ((r >> 1) & 3)) : (c ^ (r & 7));
      st_global_v4(dst + i, sm_codes[r * CCH + slot]);
    }
  }
  {
    uint16_t* dst = a.scales + row0 * G;
    const int n = nrows * G;
    if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0 && (n % 8) == 0) {
      const uint4* s4 = reinterpret_cast<const uint4*>(sm_sc);
      for (int i = tid; i < n / 8; i += kQR) st_global_v4(reinterpret_cast<uint4*>(dst) + i, s4[i]);
    } else if ((reinterpret_cast<uintptr_t>(dst) & 3) == 0 && (n % 2) == 0) {
      const uint32_t* s2 = reinterpret_cast<const uint32_t*>(sm_sc);
      for (int i = tid; i < n / 2; i += kQR) reinterpret_cast<uint32_t*>(dst)[i] = s2[i];
    } else {
      for (int i = tid; i < n; i += kQR) dst[i] = sm_sc[i];
    }
  }
  if (a.sink != nullptr && row0 < a.sink_rows) {
    const int ns = static_cast<int>(min(static_cast<int64_t>(nrows), a.sink_rows - row0));
    uint4* dst = reinterpret_cast<uint4*>(a.sink + row0 * kQD);
    for (int i = tid; i < ns * 16; i += kQR) {
      const int r = i >> 4, c = i & 15;
      st_global_v4(dst + i, tin[r * 16 + (c ^ (r & 7))]);
    }
  }
}

// Persistent CTAs walk the kQR-row tiles with a grid stride; each thread keeps
// the next kStages-1 tiles' input in flight (cp.async, 16 bytes per copy, into
// the XOR-swizzled layout) while it quantizes its row of the current tile.
template <class L, int BITS, class P, bool ROPE>
__global__ void __launch_bounds__(kQR, 3) quantize_rows_pipe(const __grid_constant__ P bt, int64_t n_tiles) {
  constexpr int S = PipeCfg<BITS>::kStages;
  constexpr int CW = QuantConsts<BITS>::kCodeBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint4* sm_in = reinterpret_cast<uint4*>(smem_raw);                                   // S x kQR x 16 chunks
  uint4* sm_codes = reinterpret_cast<uint4*>(smem_raw + S * kQR * 256);                // kQR x CW / 16
  uint16_t* sm_sc = reinterpret_cast<uint16_t*>(smem_raw + S * kQR * 256 + kQR * CW);  // kQR x G
  const int tid = threadIdx.x;
  const uint32_t in_base = static_cast<uint32_t>(__cvta_generic_to_shared(sm_in));
  pdl_wait();
  pdl_launch_dependents();

  // A launch tile is (tensor ti, tile loc of it). The grid-stride walk advances
  // (ti, loc) by additions; a division only places the first tiles.
  const int64_t tpt = bt.tiles_per;
  auto advance = [&](int64_t& ti, int64_t& loc) {
    loc += gridDim.x;
    while (loc >= tpt) {
      loc -= tpt;
      ++ti;
    }
  };
  // Thread t copies the 16-byte chunks t + kQR k of the tile: chunk t % 16 of rows
  // t / 16 + 8 k. Its shared-memory destinations are 2048 bytes apart (the swizzle
  // depends on the row mod 8 only), and so are its sources when the tile's rows are
  // one contiguous range; strided rows step (token, head) by 8 heads per copy. The
  // addresses come from one base per tile: per-copy 64-bit address arithmetic here
  // cost more issue slots than the quantization itself.
  auto issue = [&](int64_t ti, int64_t loc, int stage) {
    const QuantArgs& a = bt.tensor(ti);
    const int64_t row0 = loc * kQR;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kQR), a.n_rows - row0));
    const int r0 = tid >> 4, c = tid & 15;
    const uint32_t dst = in_base + (((stage * kQR + r0) * 16 + (c ^ (r0 & 7))) << 4);
    if (a.rows_contig && nrows == kQR) {
      const char* src = reinterpret_cast<const char*>(a.x + row0 * kQD) + tid * 16;
#pragma unroll
      for (int k = 0; k < 16; ++k) cp_async16(dst + k * 2048, src + k * 2048);
    } else {
      int64_t t = (row0 + r0) / a.H;
      int h = static_cast<int>(row0 + r0 - t * a.H);
#pragma unroll 4
      for (int k = 0; k < 16; ++k) {
        if (r0 + 8 * k < nrows)
          cp_async16(dst + k * 2048, a.x + t * a.x_token_stride + static_cast<int64_t>(h) * kQD + c * 8);
        h += 8;
        while (h >= a.H) {
          h -= a.H;
          ++t;
        }
      }
    }
  };

  const int64_t first = blockIdx.x;
#pragma unroll
  for (int s = 0; s < S - 1; ++s) {
    const int64_t t = first + static_cast<int64_t>(s) * gridDim.x;
    if (t < n_tiles) issue(t / tpt, t % tpt, s);
    cp_async_commit();
  }
  int64_t ci = first / tpt, cl = first % tpt;  // the tile processed next
  const int64_t fn = first + static_cast<int64_t>(S - 1) * gridDim.x;
  int64_t ni = fn / tpt, nl = fn % tpt;        // the tile prefetched next
  for (int64_t k = 0;; ++k) {
    const int64_t tile = first + k * gridDim.x;
    if (tile >= n_tiles) break;
    {
      const int64_t tn = tile + static_cast<int64_t>(S - 1) * gridDim.x;
      if (tn < n_tiles) issue(ni, nl, static_cast<int>((k + S - 1) % S));
      cp_async_commit();
      advance(ni, nl);
    }
    cp_async_wait<S - 1>();
    __syncthreads();
    const int stage = static_cast<int>(k % S);
    const uint4* tin = sm_in + stage * kQR * 16;
    const QuantArgs& a = bt.tensor(ci);
    const int64_t row0 = cl * kQR;
    advance(ci, cl);
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kQR), a.n_rows - row0));
    if constexpr (ROPE) {
      // the rotated row replaces the staged input: the loads in quant_tile, the
      // exact-divide fix-up and the sink copy all read the stage
      if (tid < nrows) rope_row(a, (row0 + tid) / a.H, in_base + ((stage * kQR + tid) * 16 << 4), tid);
    }
    quant_tile<L, BITS>(a, row0, nrows, tin, sm_codes, sm_sc, tid);
    __syncthreads();  // the stage and the staging buffers are reused by later tiles
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------- generic quantize
constexpr int kGW = 8;  // warps per CTA

__global__ void __launch_bounds__(kGW * 32) quantize_rows_generic(QuantArgs a, GroupMap map, int D, int G,
                                                                  int bits) {
  __shared__ uint32_t gmax[kGW][kMaxGroups];
  __shared__ uint8_t gid[kMaxHeadDim];
  for (int c = threadIdx.x; c < D; c += blockDim.x) gid[c] = map.gid[c];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qmax = (1 << (bits - 1)) - 1;
  const float qf = static_cast<float>(qmax);
  const float magic = 12582912.0f + (bits == 4 ? 8.0f : 128.0f);
  const int cw = bits == 4 ? D / 2 : D;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kGW + warp; row < a.n_rows;
       row += static_cast<int64_t>(gridDim.x) * kGW) {
    for (int g = lane; g < G; g += 32) gmax[warp][g] = 0u;
    __syncwarp();
    const uint32_t* src = reinterpret_cast<const uint32_t*>(x_row_ptr(a, row, D));
    for (int p = lane; p < D / 2; p += 32) {
      uint32_t wv = src[p];
      atomicMax(&gmax[warp][gid[2 * p]], (wv << 16) & 0x7FFF0000u);
      atomicMax(&gmax[warp][gid[2 * p + 1]], wv & 0x7FFF0000u);
    }
    __syncwarp();
    for (int p = lane; p < D / 2; p += 32) {
      uint32_t wv = src[p];
      float x0 = bf16lo_to_f32(wv), x1 = bf16hi_to_f32(wv);
      float s0 = __fdiv_rn(__uint_as_float(gmax[warp][gid[2 * p]]), qf);
      float s1 = __fdiv_rn(__uint_as_float(gmax[warp][gid[2 * p + 1]]), qf);
      s0 = (s0 > 0.0f) ? s0 : 1.0f;
      s1 = (s1 > 0.0f) ? s1 : 1.0f;
      uint32_t c0 = code_exact(x0, s0, qf, magic), c1 = code_exact(x1, s1, qf, magic);
      if (bits == 4) {
        a.codes[row * cw + p] = static_cast<uint8_t>((c0 & 0xFu) | ((c1 & 0xFu) << 4));
      } else {
        reinterpret_cast<uint16_t*>(a.codes + row * cw)[p] =
            static_cast<uint16_t>((c0 & 0xFFu) | ((c1 & 0xFFu) << 8));
      }
      if (a.sink != nullptr && row < a.sink_rows) reinterpret_cast<uint32_t*>(a.sink + row * D)[p] = wv;
    }
    for (int g = lane; g < G; g += 32) {
      float s = __fdiv_rn(__uint_as_float(gmax[warp][g]), qf);
      s = (s > 0.0f) ? s : 1.0f;
      a.scales[row * G + g] = f32_to_bf16_bits(s);
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------- dequantize
struct DequantArgs {
  const uint8_t* codes;
  const uint16_t* scales;
  const uint16_t* sink;
  int64_t sink_rows;
  uint16_t* out;
  int64_t out_token_stride;
  int64_t n_rows;
  int H, D, G, bits;
  int rows_contig;
};

// One thread per 8 channels of a row: reads 4 (int4) or 8 (int8) code bytes and
// the row's scales, writes 16 bytes of bf16. bf16((q) * float(scale)) is exact in
// fp32 before the final round to nearest even, as in quant_kv.py:174-175.
__global__ void __launch_bounds__(256) dequantize_rows(DequantArgs a, GroupMap map) {
  __shared__ uint8_t gid[kMaxHeadDim];
  for (int c = threadIdx.x; c < a.D; c += blockDim.x) gid[c] = map.gid[c];
  __syncthreads();
  const int cpr = a.D / 8;
  const int64_t total = a.n_rows * cpr;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = idx / cpr;
    const int c8 = static_cast<int>(idx - row * cpr);
    uint16_t* dst;
    if (a.rows_contig) {
      dst = a.out + row * a.D + c8 * 8;
    } else {
      int64_t t = row / a.H;
      int h = static_cast<int>(row - t * a.H);
      dst = a.out + t * a.out_token_stride + static_cast<int64_t>(h) * a.D + c8 * 8;
    }
    if (a.sink != nullptr && row < a.sink_rows) {
      st_global_v4(dst, *reinterpret_cast<const uint4*>(a.sink + row * a.D + c8 * 8));
      continue;
    }
    int q[8];
    if (a.bits == 4) {
      uint32_t wv = *reinterpret_cast<const uint32_t*>(a.codes + row * (a.D / 2) + c8 * 4);
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = static_cast<int>((wv >> (4 * k)) & 0xFu) - 8;
    } else {
      uint2 wv = *reinterpret_cast<const uint2*>(a.codes + row * a.D + c8 * 8);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        q[k] = static_cast<int>((wv.x >> (8 * k)) & 0xFFu) - 128;
        q[4 + k] = static_cast<int>((wv.y >> (8 * k)) & 0xFFu) - 128;
      }
    }
    const uint16_t* srow = a.scales + row * a.G;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      v[k] = __fmul_rn(static_cast<float>(q[k]), bf16_bits_to_f32(srow[gid[c8 * 8 + k]]));
    st_global_v4(dst, make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                 pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7])));
  }
}

// Dequantize, specialised layouts (head_dim 128, int4): persistent CTAs of 128
// threads walk 128-row tiles. The next tiles' codes are in flight (cp.async into a
// 64B-swizzled stage) while each thread turns its row into 128 bf16: pair (2i,
// 2i+1) = byte i becomes bf16x2 (128 + lo, 128 + hi) by a byte permute and a
// mask/or, minus 136 (exact), times the group's (s, s) -- the exact product
// rounded to bf16, i.e. bf16(float(q) * float(scale)) (quant_kv.py:174-175). Rows
// inside the sink are copied from the bf16 sink. The tile is staged XOR-swizzled
// in shared memory and written out with coalesced 16-byte stores.
constexpr int kDStages = 3;

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <class L>
__host__ __device__ constexpr int chan_group(int ch) {
  int g = 0;
  while (g + 1 < L::G && ch >= L::E[g + 1]) ++g;
  return g;
}

template <class L, int C>
__device__ __forceinline__ uint4 deq_word(uint32_t w, const uint32_t (&sp)[L::G]) {
  const uint32_t ws = w >> 4;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = (__byte_perm(w, ws, static_cast<uint32_t>(((4 + i) << 8) | i)) & 0x000F000Fu) | 0x43004300u;
  constexpr uint32_t k136 = 0x43084308u;  // bf16x2 (136, 136)
  return make_uint4(bf16x2_mul(bf16x2_sub(o[0], k136), sp[chan_group<L>(8 * C + 0)]),
                    bf16x2_mul(bf16x2_sub(o[1], k136), sp[chan_group<L>(8 * C + 2)]),
                    bf16x2_mul(bf16x2_sub(o[2], k136), sp[chan_group<L>(8 * C + 4)]),
                    bf16x2_mul(bf16x2_sub(o[3], k136), sp[chan_group<L>(8 * C + 6)]));
}

template <class L, int... Cs>
__device__ __forceinline__ void deq_row_to(uint4* out_row, int r, const uint32_t (&w)[16], const uint32_t (&sp)[L::G],
                                           std::integer_sequence<int, Cs...>) {
  ((out_row[Cs ^ (r & 7)] = deq_word<L, Cs>(w[Cs], sp)), ...);
}

template <class L>
__global__ void __launch_bounds__(kQT, 3) dequantize_rows_pipe(DequantArgs a, int64_t n_tiles) {
  constexpr int G = L::G;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint4* sm_out = reinterpret_cast<uint4*>(smem_raw);                  // kQT x 16 chunks
  const uint32_t code_base = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw + kQT * 256));
  const uint4* sm_code = reinterpret_cast<const uint4*>(smem_raw + kQT * 256);  // kDStages x kQT x 4 chunks
  const int tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();

  auto issue = [&](int64_t tile, int stage) {
    const int64_t row0 = tile * kQT;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kQT), a.n_rows - row0));
#pragma unroll
    for (int i = tid; i < kQT * 4; i += kQT) {
      const int r = i >> 2, c = i & 3;
      if (r < nrows)
        cp_async16(code_base + (((stage * kQT + r) * 4 + (c ^ ((r >> 1) & 3))) << 4), a.codes + (row0 + r) * 64 + c * 16);
    }
  };

  const int64_t first = blockIdx.x;
#pragma unroll
  for (int s = 0; s < kDStages - 1; ++s) {
    const int64_t t = first + static_cast<int64_t>(s) * gridDim.x;
    if (t < n_tiles) issue(t, s);
    cp_async_commit();
  }
  for (int64_t k = 0;; ++k) {
    const int64_t tile = first + k * gridDim.x;
    if (tile >= n_tiles) break;
    const int64_t row0 = tile * kQT;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kQT), a.n_rows - row0));
    const int64_t row = row0 + tid;
    const bool mine = tid < nrows;
    const bool from_sink = mine && a.sink != nullptr && row < a.sink_rows;
    // this row's scales (or sink row) are requested before waiting for the codes
    uint32_t sp[G];
    uint4 sink_row[16];
    if (from_sink) {
#pragma unroll
      for (int c = 0; c < 16; ++c) sink_row[c] = ld_global_nc_v4(a.sink + row * kQD + c * 8);
    } else if (mine) {
      const uint16_t* srow = a.scales + row * G;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint32_t v = __ldg(srow + g);
        sp[g] = v | (v << 16);
      }
    }
    {
      const int64_t tn = tile + static_cast<int64_t>(kDStages - 1) * gridDim.x;
      if (tn < n_tiles) issue(tn, static_cast<int>((k + kDStages - 1) % kDStages));
      cp_async_commit();
    }
    cp_async_wait<kDStages - 1>();
    __syncthreads();
    const int stage = static_cast<int>(k % kDStages);
    uint4* orow = sm_out + tid * 16;
    if (from_sink) {
#pragma unroll
      for (int c = 0; c < 16; ++c) orow[c ^ (tid & 7)] = sink_row[c];
    } else if (mine) {
      uint32_t w[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = sm_code[(stage * kQT + tid) * 4 + (c ^ ((tid >> 1) & 3))];
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      deq_row_to<L>(orow, tid, w, sp, std::make_integer_sequence<int, 16>{});
    }
    __syncthreads();
    if (a.rows_contig && nrows == kQT) {
      // full tile, one contiguous range: thread t stores chunks t + kQT k (row
      // t / 16 + 8 k, chunk t % 16), constant strides on both sides
      uint4* dst = reinterpret_cast<uint4*>(a.out + row0 * kQD) + tid;
      const uint4* src = sm_out + (tid >> 4) * 16 + ((tid & 15) ^ ((tid >> 4) & 7));
#pragma unroll
      for (int k = 0; k < 16; ++k) st_global_v4(dst + k * kQT, src[k * kQT]);
    } else if (a.rows_contig) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + row0 * kQD);
      for (int i = tid; i < nrows * 16; i += kQT) {
        const int r = i >> 4, c = i & 15;
        st_global_v4(dst + i, sm_out[r * 16 + (c ^ (r & 7))]);
      }
    } else {
      for (int i = tid; i < nrows * 16; i += kQT) {
        const int r = i >> 4, c = i & 15;
        const int64_t rr = row0 + r;
        const int64_t t = rr / a.H;
        const int hh = static_cast<int>(rr - t * a.H);
        st_global_v4(a.out + t * a.out_token_stride + static_cast<int64_t>(hh) * kQD + c * 8,
                     sm_out[r * 16 + (c ^ (r & 7))]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
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

template <class L, int BITS, class P, bool ROPE = false>
static int launch_fast(const P& b, int64_t tiles, cudaStream_t st) {
  constexpr int smem = pipe_smem_bytes<L, BITS>();
  constexpr int cap_sm = PipeCfg<BITS>::kMaxPerSm;
  constexpr int per_sm = (227 * 1024) / smem < cap_sm ? (227 * 1024) / smem : cap_sm;
  static_assert(per_sm >= 2, "at least two CTAs per SM must fit");
  // opt in to > 48 KB of dynamic shared memory once per device
  static bool configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(quantize_rows_pipe<L, BITS, P, ROPE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(quantize): %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    configured[dev] = true;
  }
  const int64_t cap = static_cast<int64_t>(per_sm) * num_sms();
  const unsigned grid = static_cast<unsigned>(tiles < cap ? tiles : cap);
  cudaError_t e = launch_pdl(quantize_rows_pipe<L, BITS, P, ROPE>, grid, kQR, smem, st, b, tiles);
  if (e != cudaSuccess) {
    set_error("kvq_quantize: launch failed: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  return check_launch("kvq_quantize");
}

template <int BITS, class P, bool ROPE = false>
static int dispatch_fast(int layout, const P& a, int64_t tiles, cudaStream_t st) {
  switch (layout) {
    case kLayoutBands: return launch_fast<LayoutBands, BITS, P, ROPE>(a, tiles, st);
    case kLayoutBands2: return launch_fast<LayoutBands2, BITS, P, ROPE>(a, tiles, st);
    case kLayoutBands4: return launch_fast<LayoutBands4, BITS, P, ROPE>(a, tiles, st);
    case kLayoutBlind32: return launch_fast<LayoutBlind32, BITS, P, ROPE>(a, tiles, st);
    case kLayoutBlind64: return launch_fast<LayoutBlind64, BITS, P, ROPE>(a, tiles, st);
    default: break;
  }
  set_error("internal: no specialised kernel for layout %d", layout);
  return KVQ_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------- requantize
// The requantizing move of the reference's eviction, kv[:, a:b] = kv[:, c:d].clone()
// (quant_kv.py:13; the clone dequantizes, quant_kv.py:189-199, and the write
// quantizes, quant_kv.py:201-215), in one pass over packed rows: each row is
// dequantized into shared memory exactly as dequantize_rows_pipe does (or taken
// from the source's bf16 rows below its sink), then quantized by quant_tile, which
// also copies the first dst.sink_rows rows into the destination sink. Codes and
// scales equal dequantize-then-quantize bit for bit; no bf16 window goes through
// HBM (176 bytes per row instead of 688).
struct RequantArgs {
  DequantArgs src;  // codes, scales; sink / sink_rows = the source's bf16 rows below its sink
  QuantArgs dst;    // codes, scales; sink / sink_rows = the destination's sink rows
};

constexpr int kRStages = 2;  // code stages of the requantize kernel (one tile in flight)

template <class L>
__global__ void __launch_bounds__(kQR, 4) requantize_rows_pipe(const __grid_constant__ RequantArgs ra,
                                                               int64_t n_tiles) {
  constexpr int G = L::G;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint4* tin = reinterpret_cast<uint4*>(smem_raw);  // kQR x 16 chunks of bf16, XOR-swizzled
  const uint32_t code_base = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw + kQR * 256));
  uint4* sm_code = reinterpret_cast<uint4*>(smem_raw + kQR * 256);  // kRStages x kQR x 4 chunks
  uint16_t* sm_sc = reinterpret_cast<uint16_t*>(smem_raw + kQR * 256 + kRStages * kQR * 64);
  const DequantArgs& a = ra.src;
  const int tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();

  auto issue = [&](int64_t tile, int stage) {
    const int64_t row0 = tile * kQR;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kQR), a.n_rows - row0));
#pragma unroll
    for (int i = tid; i < kQR * 4; i += kQR) {
      const int r = i >> 2, c = i & 3;
      if (r < nrows)
        cp_async16(code_base + (((stage * kQR + r) * 4 + (c ^ ((r >> 1) & 3))) << 4), a.codes + (row0 + r) * 64 + c * 16);
    }
  };

  const int64_t first = blockIdx.x;
  if (first < n_tiles) issue(first, 0);
  cp_async_commit();
  for (int64_t k = 0;; ++k) {
    const int64_t tile = first + k * gridDim.x;
    if (tile >= n_tiles) break;
    const int64_t row0 = tile * kQR;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kQR), a.n_rows - row0));
    const int64_t row = row0 + tid;
    const bool mine = tid < nrows;
    const bool exact = mine && a.sink != nullptr && row < a.sink_rows;
    // this row's scales are requested before waiting for the codes
    uint32_t sp[G];
    if (mine && !exact) {
      const uint16_t* srow = a.scales + row * G;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint32_t v = __ldg(srow + g);
        sp[g] = v | (v << 16);
      }
    }
    {
      const int64_t tn = tile + gridDim.x;
      if (tn < n_tiles) issue(tn, static_cast<int>((k + 1) % kRStages));
      cp_async_commit();
    }
    cp_async_wait<1>();
    __syncthreads();  // the tile's codes have landed; the previous tile's stage reads are done
    const int stage = static_cast<int>(k % kRStages);
    uint4* orow = tin + tid * 16;
    if (exact) {
#pragma unroll
      for (int c = 0; c < 16; ++c) orow[c ^ (tid & 7)] = ld_global_nc_v4(a.sink + row * kQD + c * 8);
    } else if (mine) {
      uint32_t w[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = sm_code[(stage * kQR + tid) * 4 + (c ^ ((tid >> 1) & 3))];
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      deq_row_to<L>(orow, tid, w, sp, std::make_integer_sequence<int, 16>{});
    }
    // The tile's code stage doubles as the codes staging buffer: each thread has
    // read its own row's codes above and quant_tile writes that row's new codes
    // over them (same 64 bytes, same swizzle) before its barrier.
    quant_tile<L, 4>(ra.dst, row0, nrows, tin, sm_code + stage * kQR * 4, sm_sc, tid);
    __syncthreads();  // tin and the staging buffers are rewritten by the next tile
  }
  cp_async_wait<0>();
}

template <class L>
constexpr int requant_smem_bytes() {
  return kQR * 256 + kRStages * kQR * 64 + ((kQR * L::G * 2 + 15) / 16) * 16;
}

template <class L>
static int launch_requant(const RequantArgs& ra, cudaStream_t st) {
  constexpr int smem = requant_smem_bytes<L>();
  static_assert(4 * (smem + 1024) <= 228 * 1024, "four CTAs per SM must fit");
  static bool configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(requantize_rows_pipe<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(requantize): %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    configured[dev] = true;
  }
  const int64_t tiles = (ra.src.n_rows + kQR - 1) / kQR;
  const int64_t cap = 4LL * num_sms();
  cudaError_t e = launch_pdl(requantize_rows_pipe<L>, static_cast<unsigned>(tiles < cap ? tiles : cap), kQR, smem,
                             st, ra, tiles);
  if (e != cudaSuccess) {
    set_error("kvq_requantize: launch failed: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  return check_launch("kvq_requantize");
}

template <class L>
static int launch_dequant(const DequantArgs& a, cudaStream_t st) {
  constexpr int smem = kQT * 256 + kDStages * kQT * 64;
  static bool configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(dequantize_rows_pipe<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(dequantize): %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    configured[dev] = true;
  }
  const int64_t tiles = (a.n_rows + kQT - 1) / kQT;
  const int64_t cap = 3LL * num_sms();
  cudaError_t e = launch_pdl(dequantize_rows_pipe<L>, static_cast<unsigned>(tiles < cap ? tiles : cap), kQT, smem,
                             st, a, tiles);
  if (e != cudaSuccess) {
    set_error("kvq_dequantize: launch failed: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  return check_launch("kvq_dequantize");
}

}  // namespace kvq

using namespace kvq;

// Checks of one tensor's pointers for kvq_quantize / kvq_rebuild_layers.
static int check_quant_tensor(const void* x, int64_t x_token_stride, const void* codes, const void* scales,
                              const void* sink, int n_heads, int head_dim, int index) {
  KVQ_REQUIRE(x && codes && scales, KVQ_ERR_ARG, "NULL data pointer (tensor %d)", index);
  KVQ_REQUIRE(x_token_stride >= static_cast<int64_t>(n_heads) * head_dim, KVQ_ERR_ARG,
              "x_token_stride %lld < n_heads*head_dim", (long long)x_token_stride);
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (x_token_stride % 8) == 0, KVQ_ERR_ALIGN,
              "x must be 16-byte aligned with a token stride that is a multiple of 8 elements (tensor %d)", index);
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(codes) & 15) == 0, KVQ_ERR_ALIGN,
              "codes must be 16-byte aligned (tensor %d)", index);
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(scales) & 1) == 0, KVQ_ERR_ALIGN,
              "scales must be 2-byte aligned (tensor %d)", index);
  KVQ_REQUIRE(sink == nullptr || (reinterpret_cast<uintptr_t>(sink) & 15) == 0, KVQ_ERR_ALIGN,
              "sink must be 16-byte aligned (tensor %d)", index);
  return KVQ_OK;
}

static QuantArgs quant_args(const void* x, int64_t x_token_stride, void* codes, void* scales, void* sink,
                            int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim) {
  QuantArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.x_token_stride = x_token_stride;
  a.codes = static_cast<uint8_t*>(codes);
  a.scales = static_cast<uint16_t*>(scales);
  a.sink = static_cast<uint16_t*>(sink);
  a.n_rows = n_tokens * n_heads;
  a.sink_rows = (sink ? (sink_tokens < n_tokens ? sink_tokens : n_tokens) : 0) * n_heads;
  a.H = n_heads;
  a.rows_contig = x_token_stride == static_cast<int64_t>(n_heads) * head_dim;
  a.freqs = nullptr;
  a.pos = nullptr;
  a.max_pos = 0;
  return a;
}

// n tensors of one shape: one launch of the specialised kernel, or one launch of
// the generic kernel per tensor.
static int quantize_tensors(int layout, const GroupMap& map, const QuantArgs* args, int n, int head_dim,
                            int n_groups, int bits, cudaStream_t st) {
  if (layout != kLayoutGeneric) {
    const int64_t tpt = (args[0].n_rows + kQR - 1) / kQR;
    if (n == 1) {
      QuantOne o;
      o.a = args[0];
      o.tiles_per = tpt;
      return bits == 4 ? dispatch_fast<4>(layout, o, tpt, st) : dispatch_fast<8>(layout, o, tpt, st);
    }
    static thread_local QuantBatch b;  // 6 KB: kept off the stack
    b.n = n;
    b.tiles_per = tpt;
    for (int i = 0; i < n; ++i) b.t[i] = args[i];
    return bits == 4 ? dispatch_fast<4>(layout, b, tpt * n, st) : dispatch_fast<8>(layout, b, tpt * n, st);
  }
  for (int i = 0; i < n; ++i) {
    const int64_t blocks = (args[i].n_rows + kGW - 1) / kGW;
    const int grid = static_cast<int>(blocks < num_sms() * 8 ? blocks : num_sms() * 8);
    quantize_rows_generic<<<grid, kGW * 32, 0, st>>>(args[i], map, head_dim, n_groups, bits);
    int rc = check_launch("kvq_quantize(generic)");
    if (rc) return rc;
  }
  return KVQ_OK;
}

extern "C" int kvq_quantize(const void* x, int64_t x_token_stride, void* codes, void* scales, void* sink,
                            int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim,
                            const int32_t* chan_band, int n_groups, int bits, void* stream) {
  clear_error();
  KVQ_REQUIRE(bits == 4 || bits == 8, KVQ_ERR_ARG, "bits must be 4 or 8, got %d", bits);
  KVQ_REQUIRE(n_tokens >= 0 && n_heads > 0, KVQ_ERR_ARG, "bad shape: n_tokens %lld, n_heads %d",
              (long long)n_tokens, n_heads);
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  if (n_tokens == 0) return KVQ_OK;
  KVQ_REQUIRE(sink_tokens >= 0, KVQ_ERR_ARG, "negative sink_tokens");
  int rc = check_quant_tensor(x, x_token_stride, codes, scales, sink, n_heads, head_dim, 0);
  if (rc) return rc;
  rc = require_sm100();
  if (rc) return rc;
  const QuantArgs a = quant_args(x, x_token_stride, codes, scales, sink, sink_tokens, n_tokens, n_heads, head_dim);
  return quantize_tensors(layout, map, &a, 1, head_dim, n_groups, bits, static_cast<cudaStream_t>(stream));
}

extern "C" int kvq_rope_quantize(const void* x, int64_t x_token_stride, void* codes, void* scales, void* sink,
                                 int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim,
                                 const int32_t* chan_band, int n_groups, int bits, const double* freqs, int max_pos,
                                 const int32_t* positions, void* stream) {
  clear_error();
  KVQ_REQUIRE(bits == 4 || bits == 8, KVQ_ERR_ARG, "bits must be 4 or 8, got %d", bits);
  KVQ_REQUIRE(n_tokens >= 0 && n_heads > 0, KVQ_ERR_ARG, "bad shape: n_tokens %lld, n_heads %d",
              (long long)n_tokens, n_heads);
  KVQ_REQUIRE(head_dim == 128, KVQ_ERR_UNSUPPORTED, "the fused rotary embedding is for head_dim 128, got %d",
              head_dim);
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  KVQ_REQUIRE(layout != kLayoutGeneric, KVQ_ERR_UNSUPPORTED,
              "the fused rotary embedding supports the bands, bands2, bands4, blind32 and blind64 group maps");
  if (n_tokens == 0) return KVQ_OK;
  KVQ_REQUIRE(sink_tokens >= 0, KVQ_ERR_ARG, "negative sink_tokens");
  KVQ_REQUIRE(freqs && positions && max_pos > 0, KVQ_ERR_ARG, "NULL freqs or positions, or max_pos < 1");
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(freqs) & 15) == 0 && (reinterpret_cast<uintptr_t>(positions) & 3) == 0,
              KVQ_ERR_ALIGN, "freqs must be 16-byte and positions 4-byte aligned");
  int rc = check_quant_tensor(x, x_token_stride, codes, scales, sink, n_heads, head_dim, 0);
  if (rc) return rc;
  rc = require_sm100();
  if (rc) return rc;
  QuantOne o;
  o.a = quant_args(x, x_token_stride, codes, scales, sink, sink_tokens, n_tokens, n_heads, head_dim);
  o.a.freqs = reinterpret_cast<const double2*>(freqs);
  o.a.pos = positions;
  o.a.max_pos = max_pos;
  o.tiles_per = (o.a.n_rows + kQR - 1) / kQR;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return bits == 4 ? dispatch_fast<4, QuantOne, true>(layout, o, o.tiles_per, st)
                   : dispatch_fast<8, QuantOne, true>(layout, o, o.tiles_per, st);
}

extern "C" int kvq_rebuild_layers(int n_tensors, const void* const* x, int64_t x_token_stride, void* const* codes,
                                  void* const* scales, void* const* sink, int64_t sink_tokens, int64_t n_tokens,
                                  int n_heads, int head_dim, const int32_t* chan_band, int n_groups, int bits,
                                  void* stream) {
  clear_error();
  KVQ_REQUIRE(n_tensors >= 1 && n_tensors <= kMaxTensors, KVQ_ERR_ARG, "1 to %d tensors, got %d", kMaxTensors,
              n_tensors);
  KVQ_REQUIRE(x && codes && scales, KVQ_ERR_ARG, "NULL pointer array");
  KVQ_REQUIRE(bits == 4 || bits == 8, KVQ_ERR_ARG, "bits must be 4 or 8, got %d", bits);
  KVQ_REQUIRE(n_tokens >= 0 && n_heads > 0, KVQ_ERR_ARG, "bad shape: n_tokens %lld, n_heads %d",
              (long long)n_tokens, n_heads);
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  if (n_tokens == 0) return KVQ_OK;
  KVQ_REQUIRE(sink_tokens >= 0, KVQ_ERR_ARG, "negative sink_tokens");
  QuantArgs args[kMaxTensors];
  for (int i = 0; i < n_tensors; ++i) {
    void* si = sink ? sink[i] : nullptr;
    int rc = check_quant_tensor(x[i], x_token_stride, codes[i], scales[i], si, n_heads, head_dim, i);
    if (rc) return rc;
    args[i] = quant_args(x[i], x_token_stride, codes[i], scales[i], si, sink_tokens, n_tokens, n_heads, head_dim);
  }
  int rc = require_sm100();
  if (rc) return rc;
  return quantize_tensors(layout, map, args, n_tensors, head_dim, n_groups, bits, static_cast<cudaStream_t>(stream));
}

extern "C" int kvq_dequantize(const void* codes, const void* scales, const void* sink, int64_t sink_tokens,
                              void* out, int64_t out_token_stride, int64_t n_tokens, int n_heads, int head_dim,
                              const int32_t* chan_band, int n_groups, int bits, void* stream) {
  clear_error();
  KVQ_REQUIRE(bits == 4 || bits == 8, KVQ_ERR_ARG, "bits must be 4 or 8, got %d", bits);
  KVQ_REQUIRE(n_tokens >= 0 && n_heads > 0, KVQ_ERR_ARG, "bad shape");
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  if (n_tokens == 0) return KVQ_OK;
  KVQ_REQUIRE(codes && scales && out, KVQ_ERR_ARG, "NULL data pointer");
  KVQ_REQUIRE(out_token_stride >= static_cast<int64_t>(n_heads) * head_dim, KVQ_ERR_ARG,
              "out_token_stride too small");
  KVQ_REQUIRE(sink_tokens >= 0, KVQ_ERR_ARG, "negative sink_tokens");
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0 && (out_token_stride % 8) == 0, KVQ_ERR_ALIGN,
              "out must be 16-byte aligned with a token stride that is a multiple of 8 elements");
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(codes) & 7) == 0, KVQ_ERR_ALIGN, "codes must be 8-byte aligned");
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(scales) & 1) == 0, KVQ_ERR_ALIGN, "scales must be 2-byte aligned");
  KVQ_REQUIRE(sink == nullptr || (reinterpret_cast<uintptr_t>(sink) & 15) == 0, KVQ_ERR_ALIGN,
              "sink must be 16-byte aligned");
  int rc = require_sm100();
  if (rc) return rc;
  DequantArgs a;
  a.codes = static_cast<const uint8_t*>(codes);
  a.scales = static_cast<const uint16_t*>(scales);
  a.sink = static_cast<const uint16_t*>(sink);
  a.sink_rows = (sink ? (sink_tokens < n_tokens ? sink_tokens : n_tokens) : 0) * n_heads;
  a.out = static_cast<uint16_t*>(out);
  a.out_token_stride = out_token_stride;
  a.n_rows = n_tokens * n_heads;
  a.H = n_heads;
  a.D = head_dim;
  a.G = n_groups;
  a.bits = bits;
  a.rows_contig = out_token_stride == static_cast<int64_t>(n_heads) * head_dim;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bits == 4 && layout != kLayoutGeneric && (reinterpret_cast<uintptr_t>(codes) & 15) == 0) {
    switch (layout) {
      case kLayoutBands: return launch_dequant<LayoutBands>(a, st);
      case kLayoutBands2: return launch_dequant<LayoutBands2>(a, st);
      case kLayoutBands4: return launch_dequant<LayoutBands4>(a, st);
      case kLayoutBlind32: return launch_dequant<LayoutBlind32>(a, st);
      case kLayoutBlind64: return launch_dequant<LayoutBlind64>(a, st);
      default: break;
    }
  }
  const int64_t work = a.n_rows * (head_dim / 8);
  const int64_t blocks = (work + 255) / 256;
  const int grid = static_cast<int>(blocks < num_sms() * 16 ? blocks : num_sms() * 16);
  dequantize_rows<<<grid, 256, 0, st>>>(a, map);
  return check_launch("kvq_dequantize");
}

extern "C" int kvq_requantize(const void* src_codes, const void* src_scales, const void* src_exact,
                              int64_t exact_tokens, void* dst_codes, void* dst_scales, void* dst_sink,
                              int64_t sink_tokens, int64_t n_tokens, int n_heads, int head_dim,
                              const int32_t* chan_band, int n_groups, int bits, void* stream) {
  clear_error();
  KVQ_REQUIRE(n_tokens >= 0 && n_heads > 0, KVQ_ERR_ARG, "bad shape: n_tokens %lld, n_heads %d",
              (long long)n_tokens, n_heads);
  KVQ_REQUIRE(bits == 4 || bits == 8, KVQ_ERR_ARG, "bits must be 4 or 8, got %d", bits);
  KVQ_REQUIRE(bits == 4 && head_dim == kQD, KVQ_ERR_UNSUPPORTED,
              "the fused requantize is for int4 codes of head_dim %d (got %d bits, head_dim %d)", kQD, bits,
              head_dim);
  GroupMap map;
  int layout = resolve_layout(chan_band, head_dim, n_groups, &map);
  if (layout < 0) return layout;
  KVQ_REQUIRE(layout != kLayoutGeneric, KVQ_ERR_UNSUPPORTED,
              "the fused requantize supports the bands, bands2, bands4, blind32 and blind64 group maps");
  KVQ_REQUIRE(exact_tokens >= 0 && sink_tokens >= 0, KVQ_ERR_ARG, "negative exact_tokens or sink_tokens");
  KVQ_REQUIRE(exact_tokens == 0 || src_exact, KVQ_ERR_ARG, "exact_tokens > 0 needs src_exact");
  KVQ_REQUIRE(sink_tokens == 0 || dst_sink, KVQ_ERR_ARG, "sink_tokens > 0 needs dst_sink");
  if (n_tokens == 0) return KVQ_OK;
  KVQ_REQUIRE(src_codes && src_scales && dst_codes && dst_scales, KVQ_ERR_ARG, "NULL data pointer");
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KVQ_REQUIRE(al16(src_codes) && al16(dst_codes), KVQ_ERR_ALIGN, "codes must be 16-byte aligned");
  KVQ_REQUIRE((reinterpret_cast<uintptr_t>(src_scales) & 1) == 0 && (reinterpret_cast<uintptr_t>(dst_scales) & 1) == 0,
              KVQ_ERR_ALIGN, "scales must be 2-byte aligned");
  KVQ_REQUIRE((exact_tokens == 0 || al16(src_exact)) && (sink_tokens == 0 || al16(dst_sink)), KVQ_ERR_ALIGN,
              "src_exact and dst_sink must be 16-byte aligned");
  int rc = require_sm100();
  if (rc) return rc;
  RequantArgs ra;
  memset(&ra, 0, sizeof(ra));
  ra.src.codes = static_cast<const uint8_t*>(src_codes);
  ra.src.scales = static_cast<const uint16_t*>(src_scales);
  ra.src.sink = exact_tokens > 0 ? static_cast<const uint16_t*>(src_exact) : nullptr;
  ra.src.sink_rows = (exact_tokens < n_tokens ? exact_tokens : n_tokens) * n_heads;
  ra.src.n_rows = n_tokens * n_heads;
  ra.src.H = n_heads;
  ra.src.D = head_dim;
  ra.src.G = n_groups;
  ra.src.bits = bits;
  ra.src.rows_contig = 1;
  ra.dst = quant_args(nullptr, static_cast<int64_t>(n_heads) * head_dim, dst_codes, dst_scales,
                      sink_tokens > 0 ? dst_sink : nullptr, sink_tokens, n_tokens, n_heads, head_dim);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (layout) {
    case kLayoutBands: return launch_requant<LayoutBands>(ra, st);
    case kLayoutBands2: return launch_requant<LayoutBands2>(ra, st);
    case kLayoutBands4: return launch_requant<LayoutBands4>(ra, st);
    case kLayoutBlind32: return launch_requant<LayoutBlind32>(ra, st);
    case kLayoutBlind64: return launch_requant<LayoutBlind64>(ra, st);
    default: break;
  }
  set_error("internal: unhandled layout %d", layout);
  return KVQ_ERR_UNSUPPORTED;
}
