// Fused attention over the packed INT4 KV cache (decode and short multi-query).
//
// Semantics follow kernels/llama3/attention_quant.py:24-152 of the reference:
//   out[b, h, i] = softmax_j(q[b,h,i] . K[b, h/R, j] * sm_scale) . V[b, h/R, j]
// with K/V = (code - 8) * scale dequantized inside the kernel, R = Hq/Hkv,
// and (is_causal) keys j <= sk - sq + i visible (bottom-right alignment).
//
// Two device paths:
//  * fast (kv4_attn_fast): one CTA = 4 warps streams 128-token tiles of
//    packed K/V + scales from HBM into shared memory (packed rows by 4-D TMA
//    boxes with the hardware swizzle of the row width, scales by 1-D bulk
//    copies; no multicast), two stages: "full" mbarriers signal a landed
//    tile, and the last warp done with a stage refills it.  All q heads
//    of a GQA group (and all query rows, up to 8 columns per CTA) share ONE
//    read of the group's KV.  Scores and P.V run on the tensor cores
//    (mma.m16n8k16 bf16 -> fp32) with the packed nibbles turned into bf16
//    "128 + code" operands in registers; per-group scales are applied
//    exactly in fp32 (K: after each group's partial dot product; V: folded
//    into P).  Split-K: each work unit (batch, KV head, column chunk) is cut
//    into equal token ranges, one CTA each, sized to one wave of resident
//    CTAs; the last CTA to finish a unit (per-unit counter) merges the
//    (o, lse) partials with a log-sum-exp -- one launch per call.  Variants:
//    the new token's quantize-on-append fused in (kv4_append_attention) and
//    a paged cache read through a block table (kv4_attention_paged).
//  * generic (kv4_attn_generic): a warp-per-token FFMA kernel for any shape,
//    dtype, stride, group size and long query blocks.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <climits>
#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace kv4 {

// device error word written by bounded waits (read and cleared by kv4_device_error)
static __device__ int g_device_error = 0;

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegInf = -INFINITY;

// Output modes of both paths
enum OutMode : int { OUT_FINAL = 0, OUT_PARTIAL = 1 };

struct AttnCommon {
  const void *q;
  int64_t qs[4];
  int q_dtype;
  void *out;  // OUT_FINAL: [B,Hq,sq,d] in out_dtype ; OUT_PARTIAL: part_o f32
  int64_t os[4];
  int out_dtype;
  float *lse;  // OUT_PARTIAL: part_lse f32 [B,Hq,sq]
  int64_t ls[3];
  int mode;
  int B, Hq, Hkv, R, sq, sk, d, G;
  int causal;
  int64_t k_offset, sk_total;  // global key positions of this cache slice
  float scale_log2;            // sm_scale * log2(e)
};

// visible-key limit (exclusive, local index) of query row qi
__device__ __forceinline__ int64_t key_limit(const AttnCommon &C, int qi) {
  if (!C.causal) return C.sk;
  int64_t lim = C.sk_total - C.sq + qi + 1 - C.k_offset;
  return lim < C.sk ? lim : C.sk;
}

// write one finished (m, l, o) row: o_unnorm/l to out (FINAL) or (o, lse) to partials
__device__ __forceinline__ void emit_value(const AttnCommon &C, int b, int h, int qi, int dd,
                                           float val) {
  const int64_t off = b * C.os[0] + h * C.os[1] + qi * C.os[2] + dd * C.os[3];
  if (C.mode == OUT_FINAL) store_from_f32(C.out, C.out_dtype, off, val);
  else static_cast<float *>(C.out)[off] = val;
}
__device__ __forceinline__ void emit_lse(const AttnCommon &C, int b, int h, int qi,
                                         float lse_log2) {
  if (C.mode != OUT_PARTIAL) return;
  C.lse[b * C.ls[0] + h * C.ls[1] + qi * C.ls[2]] = lse_log2 * kLn2;
}

// ===========================================================================
// generic path
// ===========================================================================
struct GenParams {
  AttnCommon c;
  const uint8_t *kp, *vp;
  const void *ks, *vs;
  int64_t kps[4], vps[4], kss[4], vss[4];
  int s_dtype;
};

__device__ __forceinline__ float deq(const uint8_t *p, const int64_t *ps, const void *s,
                                     const int64_t *ss, int sdt, int64_t base_p,
                                     int64_t base_s, int dd, int G) {
  const uint8_t byte = p[base_p + (dd >> 1) * ps[3]];
  const int code = (dd & 1) ? (byte >> 4) : (byte & 15);
  return static_cast<float>(code - 8) * load_as_f32(s, sdt, base_s + (dd / G) * ss[3]);
}

template <int NDI>
__global__ void __launch_bounds__(128) kv4_attn_generic(const GenParams P) {
  const AttnCommon &C = P.c;
  const int bh = blockIdx.x;
  const int b = bh / C.Hq, h = bh % C.Hq;
  const int qi = blockIdx.y;
  const int kvh = h / C.R;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = 4;

  float qv[NDI], acc[NDI];
#pragma unroll
  for (int i = 0; i < NDI; ++i) {
    const int dd = lane + 32 * i;
    qv[i] = dd < C.d ? load_as_f32(C.q, C.q_dtype,
                                   b * C.qs[0] + h * C.qs[1] + qi * C.qs[2] + dd * C.qs[3])
                     : 0.0f;
    acc[i] = 0.0f;
  }
  float m = kNegInf, l = 0.0f;
  const int64_t lim = key_limit(C, qi);
  for (int64_t t = warp; t < lim; t += NW) {
    const int64_t bpk = b * P.kps[0] + kvh * P.kps[1] + t * P.kps[2];
    const int64_t bsk = b * P.kss[0] + kvh * P.kss[1] + t * P.kss[2];
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < NDI; ++i) {
      const int dd = lane + 32 * i;
      if (dd < C.d) part += qv[i] * deq(P.kp, P.kps, P.ks, P.kss, P.s_dtype, bpk, bsk, dd, C.G);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const float s = part * C.scale_log2;
    const float mn = fmaxf(m, s);
    const float alpha = exp2f(m - mn);  // m == -inf -> 0
    const float p = exp2f(s - mn);
    l = l * alpha + p;
    const int64_t bpv = b * P.vps[0] + kvh * P.vps[1] + t * P.vps[2];
    const int64_t bsv = b * P.vss[0] + kvh * P.vss[1] + t * P.vss[2];
#pragma unroll
    for (int i = 0; i < NDI; ++i) {
      const int dd = lane + 32 * i;
      const float vv =
          dd < C.d ? deq(P.vp, P.vps, P.vs, P.vss, P.s_dtype, bpv, bsv, dd, C.G) : 0.0f;
      acc[i] = acc[i] * alpha + p * vv;
    }
    m = mn;
  }
  // merge the 4 warps
  __shared__ float sm_m[NW], sm_l[NW];
  __shared__ float sm_o[NW][NDI * 32];
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < NDI; ++i) sm_o[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  float M = kNegInf;
#pragma unroll
  for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w]);
  float L = 0.0f, f[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    f[w] = (M == kNegInf) ? 0.0f : exp2f(sm_m[w] - M);
    L += sm_l[w] * f[w];
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
  for (int dd = threadIdx.x; dd < C.d; dd += blockDim.x) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) o += sm_o[w][dd] * f[w];
    emit_value(C, b, h, qi, dd, o * inv);
  }
  if (threadIdx.x == 0) emit_lse(C, b, h, qi, L > 0.0f ? M + log2f(L) : kNegInf);
}

// ===========================================================================
// fast path
// ===========================================================================
constexpr int TOK = 128;   // tokens per pipeline stage (4 warps x 32 rows)
constexpr int NWARP = 4;
constexpr int WROWS = 32;  // token rows per warp per stage (two m16 sub-tiles)
constexpr int NCOL = 8;    // (head, query row) columns per CTA = MMA N
constexpr int MERGE_GROUP = 8;  // split-K parts merged per first-level group

struct FastParams {
  AttnCommon c;
  int ncols;      // R * sq
  int hc;         // column chunks per (b, kvh)
  int tpu;        // tiles per unit
  int L;          // tiles per CTA (stream-K chunk)
  int64_t total_tiles;
  int maxp;       // partial slots per unit
  float *ws_o;    // [units*maxp][NCOL][d]
  float *ws_lse;  // [units*maxp][NCOL]   (log2 domain)
  int *counters;  // [units] finished-segment counts (zero between calls); the
                  // [units][ngroups] first-level counters sit right before
  int units;
  int cs;         // > 1: launched as clusters of cs CTAs (consecutive parts of a unit)
  int drop_last;  // test knob: the last tile of each CTA is never loaded
  int early;      // launched with programmatic stream serialization (see the kernel)
  uint32_t wait_limit;  // polls of a bounded mbarrier wait (each <= 1 ms)
  const char *ks, *vs;         // scale tensors
  int64_t ks_sb, ks_sh, vs_sb, vs_sh;  // their batch / head strides in bytes
  // Fused quantize-on-append (app_row >= 0): the new token's K/V rows
  // (kn/vn [B, Hkv, 1, d], unit dim stride) are quantized into cache row
  // app_row.  Every CTA that streams that row quantizes it itself and patches
  // its staged copy; the hc == 0 CTA of the (b, kvh) also writes it to HBM.
  int app_row;
  int app_tie;
  int kn_dtype;
  const void *kn, *vn;
  int64_t kn_sb, kn_sh, vn_sb, vn_sh;  // elements
  uint8_t *kpw, *vpw;                  // packed caches (bytes)
  int64_t kp_sb, kp_sh, kp_st, vp_sb, vp_sh, vp_st;
  // Paged layout (page > 0): packed/scale tensors are page pools
  // [npages, Hkv, page, ...] (ks_sb / vs_sb are then page strides); token t
  // of sequence b lives in page bt[b * bt_stride + t / page], row t % page;
  // sequence b holds seq_lens[b] tokens (c.sk is the grid's upper bound).
  int page;
  int npages;
  const int32_t *bt;
  int64_t bt_stride;
  const int32_t *seq_lens;
  int bt_slots;  // shared-memory slots for the CTA's block-table slice
};

// Quantize one d-wide row with a warp: lane l owns dims [DPL*l, DPL*l + DPL)
// (v, loaded by load_row_lane) and returns their packed nibbles (low nibble =
// even dim) and its group's fp32 scale.  Same arithmetic as quantize_kernel
// for each tie mode.
template <int D>
__device__ __forceinline__ void load_row_lane(const void *x, int dt, int64_t off, int lane,
                                              float (&v)[D / 32]) {
#pragma unroll
  for (int e = 0; e < D / 32; ++e) v[e] = load_as_f32(x, dt, off + (D / 32) * lane + e);
}
template <int D, int G>
__device__ __forceinline__ void quant_row_regs(const float (&v)[D / 32], int tie, uint32_t &w,
                                               float &scale) {
  constexpr int DPL = D / 32, LPG = G / DPL;
  float mx = 0.0f;
#pragma unroll
  for (int e = 0; e < DPL; ++e) mx = fmaxf(mx, fabsf(v[e]));
#pragma unroll
  for (int o = 1; o < LPG; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  w = 0;
  if (tie == KV4_TIE_HALF_EVEN) {
    scale = group_scale<KV4_TIE_HALF_EVEN>(mx);
#pragma unroll
    for (int e = 0; e < DPL; ++e) w |= code_of<KV4_TIE_HALF_EVEN>(v[e], scale) << (4 * e);
  } else if (tie == KV4_TIE_HALF_AWAY_IEEE) {
    scale = group_scale<KV4_TIE_HALF_AWAY_IEEE>(mx);
#pragma unroll
    for (int e = 0; e < DPL; ++e) w |= code_of<KV4_TIE_HALF_AWAY_IEEE>(v[e], scale) << (4 * e);
  } else {
    scale = group_scale<KV4_TIE_HALF_AWAY>(mx);
#pragma unroll
    for (int e = 0; e < DPL; ++e) w |= code_of<KV4_TIE_HALF_AWAY>(v[e], scale) << (4 * e);
  }
}

// store the DPL/2 low bytes of w (1, 2 or 4; the address is aligned to that)
template <int NB>
__device__ __forceinline__ void st_bytes_global(uint8_t *p, uint32_t w) {
  if constexpr (NB == 1) *p = static_cast<uint8_t>(w);
  else if constexpr (NB == 2) *reinterpret_cast<uint16_t *>(p) = static_cast<uint16_t>(w);
  else *reinterpret_cast<uint32_t *>(p) = w;
}
template <int NB>
__device__ __forceinline__ void st_bytes_shared(uint32_t a, uint32_t w) {
  if constexpr (NB == 1) asm volatile("st.shared.u8 [%0], %1;" ::"r"(a), "r"(w) : "memory");
  else if constexpr (NB == 2) asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "r"(w) : "memory");
  else asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(w) : "memory");
}
// one scale (bf16 / f16 / f32 in shared memory) as fp32
template <typename ST>
__device__ __forceinline__ float lds_scale(uint32_t a) {
  if constexpr (sizeof(ST) == 2) {
    const uint32_t w = lds16(a);
    if constexpr (std::is_same<ST, __nv_bfloat16>::value) return __uint_as_float(w << 16);
    else return __half2float(__ushort_as_half(static_cast<unsigned short>(w)));
  } else {
    return __uint_as_float(lds32(a));
  }
}
template <int NB>
__device__ __forceinline__ uint32_t ld_bytes_shared(uint32_t a) {
  uint32_t w;
  if constexpr (NB == 1) asm volatile("ld.shared.u8 %0, [%1];" : "=r"(w) : "r"(a) : "memory");
  else if constexpr (NB == 2) asm volatile("ld.shared.u16 %0, [%1];" : "=r"(w) : "r"(a) : "memory");
  else asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w) : "r"(a) : "memory");
  return w;
}
template <typename ST>
__device__ __forceinline__ void st_scale_shared(uint32_t a, ST v) {
  if constexpr (sizeof(ST) == 2) {
    const uint32_t b = *reinterpret_cast<const uint16_t *>(&v);
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "r"(b) : "memory");
  } else {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(static_cast<float>(v)) : "memory");
  }
}

// Shared-memory layout of one stage (per tensor): packed codes token-major
// [token][P bytes] as TMA writes them with the P-byte swizzle (16-byte chunk c
// of row r lands at chunk c ^ ((r >> SH) & SWZ)); scales token-major
// [token][group].  Every row a lane reads has the same XOR key, so the
// swizzle folds into lane-constant chunk offsets.
template <int D, int G, typename ST>
struct FastCfg {
  static constexpr int P = D / 2;             // packed bytes per token
  static constexpr int NCH = D / 32;          // 16-byte chunks per token row
  static constexpr int NG = D / G;            // scale groups per token
  static constexpr int CPG = G / 32;          // chunks per group
  static constexpr int SROW = NG * (int)sizeof(ST);  // scale bytes per token
  static constexpr int SWZ = (P == 32) ? 1 : (P == 64) ? 3 : 7;  // XOR key mask
  static constexpr int SH = (P == 32) ? 2 : (P == 64) ? 1 : 0;    // row -> key shift
  static constexpr int KP = TOK * P;          // packed bytes per stage per tensor
  static constexpr int KS = TOK * SROW;       // scale bytes per stage per tensor
  static constexpr int STAGE = ((2 * KP + 2 * KS) + 1023) / 1024 * 1024;
  // 3 x 18 KB at d=128 with 3 CTAs/SM (measured faster than 2 stages at 4
  // CTAs/SM: 64K context 37.4 -> 33.6 us); d=256 keeps 2 stages so 2 CTAs fit
#ifndef KV4_RELEASE_ATOM
#define KV4_RELEASE_ATOM "atom.acq_rel.cta.shared::cta.add.u32"
#endif
#ifndef KV4_STAGES
#define KV4_STAGES 3
#endif
#ifndef KV4_MINB
#define KV4_MINB 3
#endif
  static constexpr int STAGES = (D == 256) ? 2 : KV4_STAGES;
  static constexpr int MERGE = (NWARP + 1) * NCOL * D * 4;  // per-warp o + the CTA's o
  static_assert(MERGE <= STAGES * STAGE, "merge buffer aliases the stages");
  static constexpr int APP = 2 * P + 2 * SROW;  // staged new row (fused append)
  static constexpr int BIAS = NWARP * NG * 4 * 16;  // per warp: [group][tg] C quads
  static constexpr int SMEM = STAGES * STAGE + 3 * NWARP * NCOL * 4 + 2 * NCOL * 4 +
                              16 * STAGES + (APP + 15) / 16 * 16 + BIAS + 1024;
  static constexpr uint32_t TX = 2 * KP + 2 * KS;
};

// Nibble extraction into bf16x2 "128 + code" values (exact; bf16 0x4300|n ==
// 128 + n).  Each picks the same nibble of bytes k and k+2 of x into the low
// and high 16-bit halves: one shift (except for the nibble already in place)
// and one LOP3 ((x >> s) & 0x000F000F | magic), 7 integer ops per 8 codes.
__device__ __forceinline__ uint32_t lop_nib(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(0x000F000Fu), "r"(0x43004300u));
  return r;  // (x & m) | magic
}
__device__ __forceinline__ uint32_t nib_lo0(uint32_t x) { return lop_nib(x); }
__device__ __forceinline__ uint32_t nib_hi0(uint32_t x) { return lop_nib(x >> 4); }
__device__ __forceinline__ uint32_t nib_lo1(uint32_t x) { return lop_nib(x >> 8); }
__device__ __forceinline__ uint32_t nib_hi1(uint32_t x) { return lop_nib(x >> 12); }

// Nibble extraction into f16x2 values with the f16 magic 1024 (exponent 10:
// the 10 mantissa bits hold two nibble fields): the low nibble of bytes k and
// k+2 becomes 1024 + code, the high nibble 1024 + 16 * code, both exact, one
// LOP3 each, no shift.  The other two bytes need one shift by 8 for both
// fields: 5 integer ops per 8 codes.
__device__ __forceinline__ uint32_t h_lo(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(0x000F000Fu), "r"(0x64006400u));
  return r;  // 1024 + code
}
__device__ __forceinline__ uint32_t h_hi(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(0x00F000F0u), "r"(0x64006400u));
  return r;  // 1024 + 16 * code
}

// One token row of scales in shared memory, kept as raw words and converted
// to fp32 where used (one vector load per row instead of one load per group).
template <int NG, typename ST>
struct SRow {
  static constexpr int BYTES = NG * static_cast<int>(sizeof(ST));
  static constexpr int WORDS = (BYTES + 3) / 4;
  uint32_t w[WORDS];
  __device__ __forceinline__ void load(uint32_t a) {
    if constexpr (BYTES == 2) {
      w[0] = lds16(a);
    } else if constexpr (BYTES == 4) {
      w[0] = lds32(a);
    } else if constexpr (BYTES == 8) {
      const uint2 t = lds64(a);
      w[0] = t.x; w[1] = t.y;
    } else {
#pragma unroll
      for (int k = 0; k < BYTES / 16; ++k) {
        const uint4 t = lds128(a + 16 * k);
        w[4 * k] = t.x; w[4 * k + 1] = t.y; w[4 * k + 2] = t.z; w[4 * k + 3] = t.w;
      }
    }
  }
  __device__ __forceinline__ float get(int gi) const {
    if constexpr (sizeof(ST) == 4) {
      return __uint_as_float(w[gi]);
    } else if constexpr (std::is_same<ST, __nv_bfloat16>::value) {
      return (gi & 1) ? bf16hi_to_f32(w[gi >> 1]) : bf16lo_to_f32(w[gi >> 1]);
    } else {
      return (gi & 1) ? f16hi_to_f32(w[gi >> 1]) : f16lo_to_f32(w[gi >> 1]);
    }
  }
  // (this row's scale of group gi, row b's) as bf16x2, low half = this row
  __device__ __forceinline__ uint32_t pair_bf16(const SRow &b, int gi) const {
    if constexpr (std::is_same<ST, __nv_bfloat16>::value) {
      return prmt(w[gi >> 1], b.w[gi >> 1], (gi & 1) ? 0x7632u : 0x5410u);
    } else {
      return pack_bf16x2(get(gi), b.get(gi));
    }
  }
};

template <int NG, typename ST>
__device__ __forceinline__ void scales_row(uint32_t addr, float (&s)[NG]) {
  if constexpr (sizeof(ST) == 2) {
    if constexpr (NG == 1) {
      uint32_t w = lds16(addr);
      s[0] = to_f32(*reinterpret_cast<const ST *>(&w));
    } else if constexpr (NG == 2) {
      uint32_t w = lds32(addr);
      const ST *h = reinterpret_cast<const ST *>(&w);
      s[0] = to_f32(h[0]); s[1] = to_f32(h[1]);
    } else if constexpr (NG == 4) {
      uint2 w = lds64(addr);
      const ST *h = reinterpret_cast<const ST *>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) s[i] = to_f32(h[i]);
    } else {
#pragma unroll
      for (int k = 0; k < NG / 8; ++k) {
        uint4 w = lds128(addr + 16 * k);
        const ST *h = reinterpret_cast<const ST *>(&w);
#pragma unroll
        for (int i = 0; i < 8; ++i) s[8 * k + i] = to_f32(h[i]);
      }
    }
  } else {
    if constexpr (NG == 1) {
      s[0] = __uint_as_float(lds32(addr));
    } else if constexpr (NG == 2) {
      uint2 w = lds64(addr);
      s[0] = __uint_as_float(w.x); s[1] = __uint_as_float(w.y);
    } else {
#pragma unroll
      for (int k = 0; k < NG / 4; ++k) {
        uint4 w = lds128(addr + 16 * k);
        s[4 * k + 0] = __uint_as_float(w.x); s[4 * k + 1] = __uint_as_float(w.y);
        s[4 * k + 2] = __uint_as_float(w.z); s[4 * k + 3] = __uint_as_float(w.w);
      }
    }
  }
}

// MODE: 0 = bf16 q; 1 = fp16/fp32 q as a hi/lo pair (SPLIT); 2 = bf16 q with
// at most 4 columns per KV head, paired into the 8 MMA columns (PAIR)
template <int D, int G, typename ST, int MODE, bool PAGED>
__global__ void __launch_bounds__(128, (D == 256 ? 2 : KV4_MINB))
    kv4_attn_fast(const FastParams P, const __grid_constant__ CUtensorMap tm_kp,
                  const __grid_constant__ CUtensorMap tm_vp) {
  constexpr bool SPLIT = MODE == 1;
  constexpr bool PAIR = MODE == 2;
  using Cfg = FastCfg<D, G, ST>;
  constexpr int NCH = Cfg::NCH, NG = Cfg::NG, CPG = Cfg::CPG;
  const AttnCommon &C = P.c;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // the warp-merge buffer aliases the stage buffers: each CTA flushes once,
  // after its last tile, when no TMA load is in flight any more
  float *merge_o = reinterpret_cast<float *>(smem);
  float *merge_m = reinterpret_cast<float *>(smem + Cfg::STAGES * Cfg::STAGE);
  float *merge_l = merge_m + NWARP * NCOL;
  float *merge_f = merge_l + NWARP * NCOL;
  float *merge_lse = merge_f + NWARP * NCOL;
  uint64_t *bars = reinterpret_cast<uint64_t *>(merge_lse + 2 * NCOL);  // full[S] (+ spare)
  // fused append: quantized new row [K codes P][V codes P][K scales][V scales]
  uint8_t *app_buf = reinterpret_cast<uint8_t *>(bars + 2 * Cfg::STAGES);
  __shared__ int sh_abort;
  __shared__ int sh_last;
  __shared__ uint32_t sh_done[Cfg::STAGES];  // warps finished with each stage

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tg = lane & 3;

  // Split-K: CTA = (unit, part); part p of kparts streams tiles
  // [p*tpu/kparts, (p+1)*tpu/kparts) of its unit's sequence.
  const int kparts = P.maxp;
  const int u = static_cast<int>(blockIdx.x) / kparts;
  const int part = static_cast<int>(blockIdx.x) - u * kparts;
  const int t_begin = static_cast<int>(static_cast<int64_t>(part) * P.tpu / kparts);
  const int t_end = static_cast<int>(static_cast<int64_t>(part + 1) * P.tpu / kparts);
  const int u_bk = u / P.hc, u_hc = u - u_bk * P.hc;
  const int u_b = u_bk / C.Hkv, u_kvh = u_bk - u_b * C.Hkv;
  // keys of this unit: c.sk, or (paged) the sequence's own length; a CTA
  // whose range lies past it streams nothing but still takes part in the merge
  constexpr bool paged = PAGED;
  int sk_u = C.sk;
  if (paged) {
    const int sl = P.seq_lens[u_b];
    sk_u = sl < 0 ? 0 : (sl < C.sk ? sl : C.sk);
  }
  const int ntiles = max(0, min(t_end, (sk_u + TOK - 1) / TOK) - t_begin);
  // (a CTA of a cluster never leaves early: its cluster waits for it at the merge)
  if (ntiles <= 0 && !paged && P.cs <= 1) return;

  // q of this lane's B-operand column (n = g), requested before anything
  // else so that it is not queued behind the CTA's tile loads in HBM
  const int q_n = u_hc * NCOL + (PAIR ? (g & 3) : g);
  const bool q_ok = q_n < P.ncols;
  const int64_t q_base = q_ok ? u_b * C.qs[0] + (u_kvh * C.R + q_n % C.R) * C.qs[1] +
                                    (q_n / C.R) * C.qs[2]
                              : 0;
  const bool q_vec =
      q_ok && C.q_dtype == KV4_BF16 && C.qs[3] == 1 &&
      (reinterpret_cast<uintptr_t>(static_cast<const __nv_bfloat16 *>(C.q) + q_base + 8 * tg) &
       15) == 0;
  uint4 q_raw[NCH];
  auto load_q = [&]() {
    if (q_vec) {
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        q_raw[c] = __ldg(reinterpret_cast<const uint4 *>(
            static_cast<const __nv_bfloat16 *>(C.q) + q_base + 32 * c + 8 * tg));
    }
  };
  // Early start (P.early, launched with programmatic stream serialization):
  // until griddepcontrol.wait returns, the kernel reads only cache tiles that
  // the preceding kernel cannot be writing (host contract: it writes at most
  // row app_row - 1 of these views; the tile holding that row waits) and
  // writes nothing outside shared memory.  q, the new row, the workspace and
  // the output are touched after the wait.
  const bool early = P.early != 0 && !paged;
  if (!early) load_q();

  const uint32_t smem_base = smem_u32(smem);
  const uint32_t bar_base = smem_u32(bars);

  // per warp, per scale group and lane quad tg: the C quad (b0, b1, b0, b1)
  // that starts the group's score accumulators, b = -136 * sum(q) over the
  // group for columns 2tg, 2tg+1 (loaded as one 16-byte vector per use)
  const uint32_t bias_s = smem_u32(app_buf + (Cfg::APP + 15) / 16 * 16);
  // paged: the CTA's slice of the block table (-1 past the sequence's blocks)
  int *sh_bt = reinterpret_cast<int *>(app_buf + (Cfg::APP + 15) / 16 * 16 + Cfg::BIAS);
  const int ppt = paged ? TOK / P.page : 0;  // pages per tile
  if (paged) {
    const int nblk = (sk_u + P.page - 1) / P.page;
    for (int e = tid; e < ntiles * ppt; e += blockDim.x) {
      const int blk = t_begin * ppt + e;
      sh_bt[e] = blk < nblk ? P.bt[u_b * P.bt_stride + blk] : -1;
    }
  }

  if (tid < Cfg::STAGES) sh_done[tid] = 0;
  if (tid == 0) {
    sh_abort = 0;
    prefetch_tmap(&tm_kp);
    prefetch_tmap(&tm_vp);
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(bar_base + 8 * s, 1);                            // full: producer + tx
    }
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int i) {  // local tile i -> stage i % STAGES (thread 0 only)
    const int b = u_b, kvh = u_kvh;
    const int t0 = (t_begin + i) * TOK;
    const int s = i % Cfg::STAGES;
    const uint32_t bar = bar_base + 8 * s;
    const uint32_t dst = smem_base + s * Cfg::STAGE;
    if (paged) {
      // one TMA box per page and tensor, one bulk copy per page of scales;
      // pages past the sequence are not loaded, ids outside the pool are
      // reported through the device error word and skipped
      int nv = 0;
      for (int k = 0; k < ppt; ++k) {
        const int pg = sh_bt[i * ppt + k];
        nv += (pg >= 0 && pg < P.npages) ? 1 : 0;
      }
      const uint32_t pbytes = static_cast<uint32_t>(P.page) * (2 * Cfg::P + 2 * Cfg::SROW);
      mbar_arrive_expect_tx(bar, nv * pbytes);
      for (int k = 0; k < ppt; ++k) {
        const int pg = sh_bt[i * ppt + k];
        if (pg < 0 || pg >= P.npages) {
          if (pg >= P.npages || (pg < 0 && t0 + k * P.page < sk_u))
            atomicOr(&g_device_error, DEV_ERR_BAD_PAGE);
          continue;
        }
        const uint32_t op = static_cast<uint32_t>(k * P.page * Cfg::P);
        const uint32_t os = static_cast<uint32_t>(k * P.page * Cfg::SROW);
        tma_load_4d(dst + op, &tm_kp, bar, 0, 0, kvh, pg);
        tma_load_4d(dst + Cfg::KP + op, &tm_vp, bar, 0, 0, kvh, pg);
        bulk_load(dst + 2 * Cfg::KP + os, P.ks + pg * P.ks_sb + kvh * P.ks_sh,
                  P.page * Cfg::SROW, bar);
        bulk_load(dst + 2 * Cfg::KP + Cfg::KS + os, P.vs + pg * P.vs_sb + kvh * P.vs_sh,
                  P.page * Cfg::SROW, bar);
      }
      return;
    }
    if (P.drop_last && i == ntiles - 1) return;  // test knob: this tile never lands
    // packed codes: 2 tiled TMA loads (zero-filled past sk); scales: one bulk
    // copy per tensor of the tile's contiguous rows, rounded up to 16 bytes
    const int rem = min(TOK, C.sk - t0);
    const uint32_t sbytes = static_cast<uint32_t>(rem * Cfg::SROW + 15) & ~15u;
    mbar_arrive_expect_tx(bar, 2 * Cfg::KP + 2 * sbytes);
    tma_load_4d(dst, &tm_kp, bar, 0, t0, kvh, b);
    tma_load_4d(dst + Cfg::KP, &tm_vp, bar, 0, t0, kvh, b);
    const int64_t soff = static_cast<int64_t>(t0) * Cfg::SROW;
    bulk_load(dst + 2 * Cfg::KP, P.ks + b * P.ks_sb + kvh * P.ks_sh + soff, sbytes, bar);
    bulk_load(dst + 2 * Cfg::KP + Cfg::KS, P.vs + b * P.vs_sb + kvh * P.vs_sh + soff, sbytes, bar);
  };

  const int pre = min(ntiles, Cfg::STAGES);
  if (early) {
    // tiles of this CTA's first stages that cannot hold row app_row - 1 load
    // before the wait; the rest (at most one tile) after it
    const int hot = P.app_row > 0 ? (P.app_row - 1) / TOK - t_begin : -1;
    if (tid == 0)
      for (int i = 0; i < pre; ++i)
        if (i != hot) issue(i);
    griddep_wait();
    griddep_launch_dependents();
    load_q();
    if (tid == 0 && hot >= 0 && hot < pre) issue(hot);
  } else if (tid == 0) {
    for (int i = 0; i < pre; ++i) issue(i);
  }

  // ---- fused append: the owner warp of the new row loads it now (the loads
  // complete while the tiles stream) and quantizes it when it reaches the
  // row's tile: into the staged copy and, for hc == 0, into the cache in HBM.
  constexpr int DPL = D / 32, NBL = DPL / 2;  // dims / packed bytes per lane
  int app_key = -1;                           // (local tile) * NWARP + owner warp
  float app_k[DPL], app_v[DPL];
  {
    const int app_tile = P.app_row >= 0 ? P.app_row / TOK : -1;
    if (app_tile >= t_begin && app_tile < t_end) {
      const int app_warp = (P.app_row - app_tile * TOK) / WROWS;
      app_key = (app_tile - t_begin) * NWARP + app_warp;
      if (warp == app_warp) {
        load_row_lane<D>(P.kn, P.kn_dtype, u_b * P.kn_sb + u_kvh * P.kn_sh, lane, app_k);
        load_row_lane<D>(P.vn, P.kn_dtype, u_b * P.vn_sb + u_kvh * P.vn_sh, lane, app_v);
      }
    }
  }

  // ---- per-unit state --------------------------------------------------
  uint32_t qf[NCH][2][2];               // q B-fragments (hi), [chunk][kstep][reg]
  uint32_t qfl[(SPLIT || PAIR) ? NCH : 1][2][2];  // SPLIT: lo parts; PAIR: slab-1 fragments
  float o_acc[NCH][2][4];               // O^T fragments [chunk][j][c]
  float sp_acc[NG][4];                  // sum of P' per group (for the +128 bias of V codes)
  float m_run[2], l_run[2];
  float col_inv[2];  // score factor of columns 2tg, 2tg+1 (log2 domain)
  int vexp = 0;      // MODE 0/2: per-warp power-of-two factor of the f16 P'' (adjust_vexp)
  int col_lim[2];
  int lim_min = 0;  // smallest key limit over the CTA's columns (warp-uniform)

  auto load_unit = [&]() {
    const int hcid = u_hc, b = u_b, kvh = u_kvh;
    {
      // B operand column n = g (q fetched at kernel start when vectorizable)
      const bool ok = q_ok;
      const int64_t qbase = q_base;
      (void)hcid; (void)b; (void)kvh;
      float gsum[NG];
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) gsum[gi] = 0.0f;
      float vv[NCH][8];
      float qmax = 0.0f;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float *v = vv[c];
        const int64_t qoff = qbase + (32 * c + 8 * tg) * C.qs[3];
        if (q_vec) {
          const uint32_t ws4[4] = {q_raw[c].x, q_raw[c].y, q_raw[c].z, q_raw[c].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[2 * e] = bf16lo_to_f32(ws4[e]);
            v[2 * e + 1] = bf16hi_to_f32(ws4[e]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            v[e] = ok ? load_as_f32(C.q, C.q_dtype, qbase + (32 * c + 8 * tg + e) * C.qs[3]) : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) qmax = fmaxf(qmax, fabsf(v[e]));
      }
      if constexpr (SPLIT) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float hi[8], lo[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            hi[e] = __bfloat162float(__float2bfloat16_rn(vv[c][e]));
            lo[e] = __bfloat162float(__float2bfloat16_rn(vv[c][e] - hi[e]));
            gsum[c / CPG] += -136.0f * (hi[e] + lo[e]);
          }
          // k-step 0: (b0,b1) <- dims (0,4) ; (b2,b3) <- dims (1,5)
          // k-step 1: (b0,b1) <- dims (2,6) ; (b2,b3) <- dims (3,7)
          qf[c][0][0] = pack_bf16x2(hi[0], hi[4]);
          qf[c][0][1] = pack_bf16x2(hi[1], hi[5]);
          qf[c][1][0] = pack_bf16x2(hi[2], hi[6]);
          qf[c][1][1] = pack_bf16x2(hi[3], hi[7]);
          qfl[c][0][0] = pack_bf16x2(lo[0], lo[4]);
          qfl[c][0][1] = pack_bf16x2(lo[1], lo[5]);
          qfl[c][1][0] = pack_bf16x2(lo[2], lo[6]);
          qfl[c][1][1] = pack_bf16x2(lo[3], lo[7]);
        }
        col_inv[0] = col_inv[1] = C.scale_log2;
      } else {
        // f16 operands: column g is pre-scaled by sigma = scale_log2 * 2^e,
        // e chosen so that max |q * sigma| lies in [2^13, 2^14) (exact
        // power-of-2 range shift, undone by 2^-e on the scores).  Slots that
        // meet the "1024 + 16 * code" operands take q * sigma / 16.
        qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
        qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 2));
        const float ml = qmax * C.scale_log2;
        int e = 0;
        if (ml > 0.0f) {
          e = 13 - (static_cast<int>((__float_as_uint(ml) >> 23) & 0xFFu) - 127);
          e = max(-100, min(100, e));
        }
        const float sig = C.scale_log2 * __int_as_float((e + 127) << 23);
        const float inv = __int_as_float((127 - e) << 23);
        col_inv[0] = __shfl_sync(0xffffffffu, inv, (2 * tg) * 4);
        col_inv[1] = __shfl_sync(0xffffffffu, inv, (2 * tg + 1) * 4);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float w[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) w[k] = vv[c][k] * sig;
          qf[c][0][0] = pack_f16x2(w[0], w[4]);
          qf[c][0][1] = pack_f16x2(w[1] * 0.0625f, w[5] * 0.0625f);
          qf[c][1][0] = pack_f16x2(w[2], w[6]);
          qf[c][1][1] = pack_f16x2(w[3] * 0.0625f, w[7] * 0.0625f);
          // code bias of the rounded operands: a slot of weight w' meets
          // 1024 + code (x1 slots) or 1024 + 16 * code (x16 slots), whose
          // (code - 8) value needs -1032 w' resp. -1152 w'
          const float b1 = f16lo_to_f32(qf[c][0][0]) + f16hi_to_f32(qf[c][0][0]) +
                           f16lo_to_f32(qf[c][1][0]) + f16hi_to_f32(qf[c][1][0]);
          const float b16 = f16lo_to_f32(qf[c][0][1]) + f16hi_to_f32(qf[c][0][1]) +
                            f16lo_to_f32(qf[c][1][1]) + f16hi_to_f32(qf[c][1][1]);
          gsum[c / CPG] += -1032.0f * b1 - 1152.0f * b16;
        }
        if constexpr (PAIR) {  // slab 0 runs against lanes g < 4, slab 1 against g >= 4
#pragma unroll
          for (int c = 0; c < NCH; ++c)
#pragma unroll
            for (int k = 0; k < 2; ++k)
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                qfl[c][k][j] = g >= 4 ? qf[c][k][j] : 0u;
                qf[c][k][j] = g < 4 ? qf[c][k][j] : 0u;
              }
        }
      }
      // reduce the per-group sums over the 4 lanes of the quad (tg)
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        gsum[gi] += __shfl_xor_sync(0xffffffffu, gsum[gi], 1);
        gsum[gi] += __shfl_xor_sync(0xffffffffu, gsum[gi], 2);
      }
      // lane (g, tg) now holds column g's sums; fetch columns 2tg, 2tg+1
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        const float s0 = __shfl_sync(0xffffffffu, gsum[gi], (2 * tg) * 4);
        const float s1 = __shfl_sync(0xffffffffu, gsum[gi], (2 * tg + 1) * 4);
        if (g == 0) {
          const float b0 = s0, b1 = s1;
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %1, %2};" ::"r"(
                           bias_s + ((warp * NG + gi) * 4 + tg) * 16),
                       "f"(b0), "f"(b1)
                       : "memory");
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = hcid * NCOL + (PAIR ? ((2 * tg + j) & 3) : 2 * tg + j);
      const int qi = n < P.ncols ? n / C.R : 0;
      int64_t lim = sk_u;
      if (C.causal) {
        const int64_t total = paged ? sk_u : C.sk_total;
        lim = total - C.sq + qi + 1 - C.k_offset;
        lim = lim < sk_u ? lim : sk_u;
      }
      col_lim[j] = n < P.ncols ? static_cast<int>(lim) : 0;
      m_run[j] = kNegInf;
      l_run[j] = 0.0f;
    }
    {
      // padding columns (n >= ncols) never mask real ones: treat them as unlimited
      const int n0 = hcid * NCOL + (PAIR ? ((2 * tg) & 3) : 2 * tg);
      const int a = (n0 < P.ncols) ? col_lim[0] : INT_MAX;
      const int b2 = (n0 + 1 < P.ncols) ? col_lim[1] : INT_MAX;
      lim_min = __reduce_min_sync(0xffffffffu, min(a, b2));
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o_acc[c][j][e] = 0.0f;
#pragma unroll
    for (int gi = 0; gi < NG; ++gi)
#pragma unroll
      for (int e = 0; e < 4; ++e) sp_acc[gi][e] = 0.0f;
  };

  // Log-sum-exp merge of nsl partial slots (slot0, slot0 + stride, ...) of
  // this CTA's unit: into partial slot dst (dst >= 0) or into the output.
  // Up to 8 slots' loads are in flight per round.
  auto merge_slots = [&](int64_t slot0, int64_t stride, int nsl, int64_t dst, int first = 0,
                         int step = 1) {
    constexpr int D4 = D / 4;
    for (int idx = first * static_cast<int>(blockDim.x) + tid; idx < NCOL * D4;
         idx += step * static_cast<int>(blockDim.x)) {
      const int col = idx / D4, d4 = idx - col * D4;
      const int n = u_hc * NCOL + col;
      if (n >= P.ncols) continue;
      const float4 *src = reinterpret_cast<const float4 *>(P.ws_o + (slot0 * NCOL + col) * D) + d4;
      const float *lsrc = P.ws_lse + slot0 * NCOL + col;
      float M = kNegInf, W = 0.0f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p0 = 0; p0 < nsl; p0 += 8) {
        float4 v[8];
        float lp[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int64_t pp = static_cast<int64_t>(min(p0 + e, nsl - 1)) * stride;
          v[e] = __ldcg(src + pp * NCOL * D4);
          lp[e] = (p0 + e < nsl) ? __ldcg(lsrc + pp * NCOL) : kNegInf;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float mn = fmaxf(M, lp[e]);
          if (mn == kNegInf) continue;
          const float a = exp2f(M - mn), w = exp2f(lp[e] - mn);
          W = W * a + w;
          acc.x = acc.x * a + w * v[e].x; acc.y = acc.y * a + w * v[e].y;
          acc.z = acc.z * a + w * v[e].z; acc.w = acc.w * a + w * v[e].w;
          M = mn;
        }
      }
      const float inv = W > 0.0f ? 1.0f / W : 0.0f;
      const float lse = W > 0.0f ? M + log2f(W) : kNegInf;
      if (dst >= 0) {
        reinterpret_cast<float4 *>(P.ws_o + (dst * NCOL + col) * D)[d4] =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        if (d4 == 0) P.ws_lse[dst * NCOL + col] = lse;
      } else {
        const int qi = n / C.R, h = u_kvh * C.R + n % C.R;
        const int dd = 4 * d4;
        emit_value(C, u_b, h, qi, dd, acc.x * inv);
        emit_value(C, u_b, h, qi, dd + 1, acc.y * inv);
        emit_value(C, u_b, h, qi, dd + 2, acc.z * inv);
        emit_value(C, u_b, h, qi, dd + 3, acc.w * inv);
        if (dd == 0) emit_lse(C, u_b, h, qi, lse);
      }
    }
  };

  // Finish the CTA's unit segment: merge the 4 warps through smem, then
  // either write the output (unit wholly inside this CTA) or a partial slot;
  // the last CTA to finish a split unit (per-unit counter) merges all of the
  // unit's slots in one pass (online log-sum-exp) and re-arms the counter.
  auto flush = [&]() {
    const int hcid = u_hc, b = u_b, kvh = u_kvh;
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // l over the 8 token-row lanes (PAIR: and both slabs)
      if constexpr (PAIR) l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 2);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 4);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 8);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 16);
    }
    __syncthreads();  // merge_o aliases the stages other warps may still be reading
    if (g == 0) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        merge_m[warp * NCOL + 2 * tg + j] = m_run[j];
        merge_l[warp * NCOL + 2 * tg + j] = l_run[j];
      }
    }
    // O^T fragment -> smem [warp][col][dim] (dims d0, d0+1 as one float2);
    // remove the +128 code bias
    float *mo = merge_o + warp * NCOL * D;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int gi = c / CPG;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int d0 = 32 * c + 4 * g + 2 * j;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {  // column 2tg + cc
          if constexpr (!SPLIT) {
            // f16 V operands: even dims hold 1024 + code, odd dims 1024 + 16 code;
            // undo the warp's 2^vexp factor
            const float sp = sp_acc[gi][cc];
            const float ivf = __int_as_float((127 - vexp) << 23);
            *reinterpret_cast<float2 *>(&mo[(2 * tg + cc) * D + d0]) =
                make_float2((o_acc[c][j][cc] - 1032.0f * sp) * ivf,
                            (o_acc[c][j][2 + cc] * 0.0625f - 72.0f * sp) * ivf);
          } else {
            const float corr = 136.0f * sp_acc[gi][cc];
            *reinterpret_cast<float2 *>(&mo[(2 * tg + cc) * D + d0]) =
                make_float2(o_acc[c][j][cc] - corr, o_acc[c][j][2 + cc] - corr);
          }
        }
      }
    }
    __syncthreads();
    const bool whole = kparts == 1;
    const int slot = u * kparts + part;
    if (tid < NCOL) {  // per-column warp weights (already divided by the total l)
      float M = kNegInf;
#pragma unroll
      for (int w = 0; w < NWARP; ++w) M = fmaxf(M, merge_m[w * NCOL + tid]);
      float f[NWARP], Lsum = 0.0f;
#pragma unroll
      for (int w = 0; w < NWARP; ++w) {
        f[w] = (M == kNegInf) ? 0.0f : exp2f(merge_m[w * NCOL + tid] - M);
        Lsum += merge_l[w * NCOL + tid] * f[w];
      }
      const float inv = Lsum > 0.0f ? 1.0f / Lsum : 0.0f;
#pragma unroll
      for (int w = 0; w < NWARP; ++w) merge_f[w * NCOL + tid] = f[w] * inv;
      merge_lse[tid] = Lsum > 0.0f ? M + log2f(Lsum) : kNegInf;
    }
    __syncthreads();
    constexpr int D4 = D / 4;
    const int cs = P.cs;  // > 1: the unit's parts are clusters of cs CTAs
    // the CTA's own partial (o normalised, lse) for the cluster merge
    float *cta_o = merge_o + NWARP * NCOL * D;
    for (int idx = tid; idx < NCOL * D4; idx += blockDim.x) {
      const int col = idx / D4, d4 = idx - col * D4;
      const int n = hcid * NCOL + col;
      if (n >= P.ncols) continue;
      float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < NWARP; ++w) {
        float4 x = *reinterpret_cast<const float4 *>(&merge_o[(w * NCOL + col) * D + 4 * d4]);
        if constexpr (PAIR) {  // column col + 4 holds the same q column's slab-1 rows
          const float4 y =
              *reinterpret_cast<const float4 *>(&merge_o[(w * NCOL + col + 4) * D + 4 * d4]);
          x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
        }
        const float f = merge_f[w * NCOL + col];
        val.x += f * x.x; val.y += f * x.y; val.z += f * x.z; val.w += f * x.w;
      }
      if (whole) {
        const int qi = n / C.R, h = kvh * C.R + n % C.R;
        emit_value(C, b, h, qi, 4 * d4, val.x);
        emit_value(C, b, h, qi, 4 * d4 + 1, val.y);
        emit_value(C, b, h, qi, 4 * d4 + 2, val.z);
        emit_value(C, b, h, qi, 4 * d4 + 3, val.w);
        if (d4 == 0) emit_lse(C, b, h, qi, merge_lse[col]);
      } else if (cs > 1) {
        *reinterpret_cast<float4 *>(&cta_o[col * D + 4 * d4]) = val;
      } else {
        reinterpret_cast<float4 *>(P.ws_o + (static_cast<int64_t>(slot) * NCOL + col) * D)[d4] = val;
        if (d4 == 0) P.ws_lse[static_cast<int64_t>(slot) * NCOL + col] = merge_lse[col];
      }
    }
    if (!whole && cs > 1) {
      // Cluster merge: the cs CTAs of a cluster are consecutive parts of the
      // unit; each reads the cs partials from the CTAs' shared memory
      // (distributed shared memory) for its slice of the outputs.  With one
      // cluster per unit that is the output; otherwise the slices form the
      // cluster's group slot in global memory, and the last cluster of the
      // unit to finish (per-unit counter) merges the group slots.
      const int rank = static_cast<int>(cluster_ctarank());
      const int ngrp = kparts / cs, grp = part / cs;
      const int64_t gslot0 = static_cast<int64_t>(P.units) * kparts + static_cast<int64_t>(u) * ngrp;
      cluster_sync();
      for (int idx = rank * static_cast<int>(blockDim.x) + tid; idx < NCOL * D4;
           idx += cs * static_cast<int>(blockDim.x)) {
        const int col = idx / D4, d4 = idx - col * D4;
        const int n = hcid * NCOL + col;
        if (n >= P.ncols) continue;
        const uint32_t ao = smem_u32(&cta_o[col * D + 4 * d4]);
        const uint32_t al = smem_u32(&merge_lse[col]);
        float4 v[8];
        float lp[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q < cs) {
            v[q] = ld_dsmem_f4(dsmem_addr(ao, q));
            lp[q] = ld_dsmem_f32(dsmem_addr(al, q));
          }
        }
        float M = kNegInf;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < cs) M = fmaxf(M, lp[q]);
        float W = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (M != kNegInf) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (q < cs) {
              const float w = exp2f(lp[q] - M);
              W += w;
              acc.x += w * v[q].x; acc.y += w * v[q].y; acc.z += w * v[q].z; acc.w += w * v[q].w;
            }
          }
        }
        const float inv = W > 0.0f ? 1.0f / W : 0.0f;
        const float lse = W > 0.0f ? M + log2f(W) : kNegInf;
        if (ngrp == 1) {
          const int qi = n / C.R, h = kvh * C.R + n % C.R;
          emit_value(C, b, h, qi, 4 * d4, acc.x * inv);
          emit_value(C, b, h, qi, 4 * d4 + 1, acc.y * inv);
          emit_value(C, b, h, qi, 4 * d4 + 2, acc.z * inv);
          emit_value(C, b, h, qi, 4 * d4 + 3, acc.w * inv);
          if (d4 == 0) emit_lse(C, b, h, qi, lse);
        } else {
          const int64_t gs = gslot0 + grp;
          reinterpret_cast<float4 *>(P.ws_o + (gs * NCOL + col) * D)[d4] =
              make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
          if (d4 == 0) P.ws_lse[gs * NCOL + col] = lse;
        }
      }
      if (ngrp > 1) __threadfence();  // group-slot stores before the cluster's release below
      cluster_sync();  // every read of another CTA's shared memory is done
      if (ngrp > 1) {
        if (rank == 0 && tid == 0) {
          const int prev = atom_add_acq_rel_gpu(&P.counters[u], 1);
          sh_last = (prev == ngrp - 1);
          if (sh_last) P.counters[u] = 0;  // re-arm for the next call
        }
        cluster_sync();
        const int last = ld_dsmem_s32(dsmem_addr(smem_u32(&sh_last), 0));
        cluster_sync();  // rank 0's flag is read before any CTA exits
        if (last) merge_slots(gslot0, 1, ngrp, -1, rank, cs);
      }
    }
    if (!whole && cs <= 1) {
      // Two-level merge.  Parts are grouped by MERGE_GROUP; the last CTA of a
      // group to finish merges the group's partials (one round of loads in
      // flight) into a group slot, and the last group merger of the unit
      // merges the group slots into the output.  With a single group the
      // group merger writes the output directly.  Bar.sync orders every
      // thread's stores before thread 0's acq_rel atomic (release is
      // cumulative); the last arriver acquires them all.
      const int ngrp = (kparts + MERGE_GROUP - 1) / MERGE_GROUP;
      const int grp = part / MERGE_GROUP;
      const int gfirst = grp * MERGE_GROUP;
      const int gsize = min(MERGE_GROUP, kparts - gfirst);
      int *cnt_grp = P.counters - static_cast<int64_t>(P.units) * ngrp;  // [units][ngrp]
      __syncthreads();
      if (tid == 0) {
        int *cp = ngrp > 1 ? &cnt_grp[static_cast<int64_t>(u) * ngrp + grp] : &P.counters[u];
        const int prev = atom_add_acq_rel_gpu(cp, 1);
        sh_last = (prev == gsize - 1);
        if (sh_last) *cp = 0;  // re-arm for the next call
      }
      __syncthreads();
      if (sh_last) {
        const int64_t gslot = static_cast<int64_t>(P.units) * kparts +
                              static_cast<int64_t>(u) * ngrp + grp;
        merge_slots(static_cast<int64_t>(u) * kparts + gfirst, 1, gsize, ngrp == 1 ? -1 : gslot);
        if (ngrp > 1) {
          __syncthreads();
          if (tid == 0) {
            const int prev = atom_add_acq_rel_gpu(&P.counters[u], 1);
            sh_last = (prev == ngrp - 1);
            if (sh_last) P.counters[u] = 0;
          }
          __syncthreads();
          if (sh_last)
            merge_slots(static_cast<int64_t>(P.units) * kparts + static_cast<int64_t>(u) * ngrp,
                        1, ngrp, -1);
        }
      }
    }
    __syncthreads();
  };

  const uint32_t ones = 0x3F803F80u;  // bf16x2 (1, 1)
  // Lane-constant ldmatrix row addresses inside a stage: lane L feeds row
  // r = 8*((L>>3)&1) + (L&7) of the warp's 16-row sub-tile, 16-byte chunk
  // c + (L>>4), with the TMA swizzle applied (the key of a row does not change
  // by +16 rows, so one offset per chunk pair serves both sub-tiles).
  constexpr int P_ = Cfg::P;
  uint32_t m_off[NCH / 2];
  {
    const int r = WROWS * warp + 8 * ((lane >> 3) & 1) + (lane & 7);
    const int key = (r >> Cfg::SH) & Cfg::SWZ;
#pragma unroll
    for (int cp = 0; cp < NCH / 2; ++cp)
      m_off[cp] = r * P_ + 16 * ((2 * cp + (lane >> 4)) ^ key);
  }
  // K: one x4 load per chunk covers rows g, g+8, 16+g, 24+g (lane L feeds
  // row L of the warp's 32 rows); the swizzle key of a row depends on
  // row mod 8 only.
  uint32_t k_off[NCH];
  {
    const int r = WROWS * warp + lane;
    const int key = (r >> Cfg::SH) & Cfg::SWZ;
#pragma unroll
    for (int c = 0; c < NCH; ++c) k_off[c] = r * P_ + 16 * (c ^ key);
  }
  const uint32_t s_row0 = (WROWS * warp + g) * Cfg::SROW;        // scale row of token row g

  // f16 V operands (MODE 0 and 2): keep the step's largest V scale times
  // 2^vexp within [2^-6, 2^6] (P <= 2^8, so P * v_scale * 2^vexp stays in
  // the f16 range with full precision); when it leaves that range, move
  // vexp and rescale the accumulators exactly.  Returns 2^vexp.
  auto adjust_vexp = [&](float vmax) -> float {
    const uint32_t vbits = __reduce_max_sync(0xffffffffu, __float_as_uint(vmax));
    if (vbits != 0u) {
      const int e = static_cast<int>((vbits >> 23) & 0xFFu) - 127 + vexp;
      if (e < -6 || e > 6) {  // warp-uniform
        const int nexp = max(-120, min(120, vexp - e));
        const float r = __int_as_float((127 + max(-126, min(127, nexp - vexp))) << 23);
#pragma unroll
        for (int c = 0; c < NCH; ++c)
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) o_acc[c][j][k] *= r;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi)
#pragma unroll
          for (int k = 0; k < 4; ++k) sp_acc[gi][k] *= r;
        vexp = nexp;
      }
    }
    return __int_as_float((127 + vexp) << 23);
  };

  load_unit();  // q loads overlap the first TMA loads already in flight
  __syncwarp();  // the bias quads written by lanes g == 0 are read by the whole warp
  int stage = -1;
  uint32_t phase = 1;
  for (int i = 0; i < ntiles; ++i) {
    const int ti = t_begin + i;
    if (++stage == Cfg::STAGES) stage = 0;
    if (stage == 0) phase ^= 1u;
    if (!*reinterpret_cast<volatile int *>(&sh_abort) &&
        !mbar_wait_bounded(bar_base + 8 * stage, phase, P.wait_limit)) {
      atomicOr(&g_device_error, DEV_ERR_MBAR_TIMEOUT);
      sh_abort = 1;  // later waits are skipped; results are garbage, the flag reports it
    }
    const uint32_t kp = smem_base + stage * Cfg::STAGE;
    const uint32_t vp = kp + Cfg::KP;
    const uint32_t ksb = kp + 2 * Cfg::KP;
    const uint32_t vsb = ksb + Cfg::KS;
    const int tok0 = ti * TOK + WROWS * warp;  // first token row of this warp
    if (i * NWARP + warp == app_key) {
      // the staged copy of the new row came from HBM before (or while) it was
      // written: quantize the row and overwrite the staged copy (and, once
      // per (b, kvh), write it to the cache)
      uint32_t kw, vw;
      float ksf, vsf;
      quant_row_regs<D, G>(app_k, P.app_tie, kw, ksf);
      quant_row_regs<D, G>(app_v, P.app_tie, vw, vsf);
      const ST kst = from_f32<ST>(ksf), vst = from_f32<ST>(vsf);
      const int r = P.app_row - ti * TOK;
      const int o = NBL * lane;
      const uint32_t off = r * P_ + 16 * ((o >> 4) ^ ((r >> Cfg::SH) & Cfg::SWZ)) + (o & 15);
      st_bytes_shared<NBL>(kp + off, kw);
      st_bytes_shared<NBL>(vp + off, vw);
      const bool lead = (DPL * lane) % G == 0;
      const int so = (DPL * lane / G) * static_cast<int>(sizeof(ST));
      if (lead) {
        st_scale_shared<ST>(ksb + r * Cfg::SROW + so, kst);
        st_scale_shared<ST>(vsb + r * Cfg::SROW + so, vst);
      }
      if (u_hc == 0) {  // one writer per (b, kvh) row
        const int64_t rr = P.app_row;
        st_bytes_global<NBL>(P.kpw + u_b * P.kp_sb + u_kvh * P.kp_sh + rr * P.kp_st + o, kw);
        st_bytes_global<NBL>(P.vpw + u_b * P.vp_sb + u_kvh * P.vp_sh + rr * P.vp_st + o, vw);
        if (lead) {
          *reinterpret_cast<ST *>(const_cast<char *>(P.ks) + u_b * P.ks_sb + u_kvh * P.ks_sh +
                                  rr * Cfg::SROW + so) = kst;
          *reinterpret_cast<ST *>(const_cast<char *>(P.vs) + u_b * P.vs_sb + u_kvh * P.vs_sh +
                                  rr * Cfg::SROW + so) = vst;
        }
      }
      // order these generic writes before the TMA refill of the stage
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
    }
    if constexpr (PAIR) {
      // ---- paired columns (at most 4 q columns per KV head) ---------------
      // The 8 MMA columns hold the 4 columns twice: columns 0-3 score the
      // warp's rows 0-15 (slab 0), columns 4-7 its rows 16-31 (slab 1), by
      // running slab 0 against q in lanes g < 4 only (qfA) and slab 1
      // against q in lanes g >= 4 only (qfB) into ONE accumulator.  Every
      // accumulator element is then a real (token, column) pair: lane
      // (g, tg) holds rows g, g+8 of slab tg / 2 for columns 2tg, 2tg+1
      // (column c is q column c & 3).
      const int slab = tg >> 1;
      const int rbase = WROWS * warp + 16 * slab + g;  // the lane's rows: rbase, rbase + 8
      float s2[2][2] = {};
      SRow<NG, ST> krow2[2];
      krow2[0].load(ksb + rbase * Cfg::SROW);
      krow2[1].load(ksb + (rbase + 8) * Cfg::SROW);
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        float acc[4];
#pragma unroll
        for (int cc = 0; cc < CPG; ++cc) {
          const int c = gi * CPG + cc;
          uint32_t xr[4];  // rows g, g+8 of slab 0, then of slab 1
          ldsm_x4(kp + k_off[c], xr);
          const uint32_t y0 = xr[0] >> 8, y1 = xr[1] >> 8, y2 = xr[2] >> 8, y3 = xr[3] >> 8;
          if (cc == 0) {
            float bq[4];
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(bq[0]), "=f"(bq[1]), "=f"(bq[2]), "=f"(bq[3])
                         : "r"(bias_s + ((warp * NG + gi) * 4 + tg) * 16));
            mma_f16_16816_c(acc, h_lo(xr[0]), h_lo(xr[1]), h_hi(xr[0]), h_hi(xr[1]),
                            qf[c][0][0], qf[c][0][1], bq[0], bq[1], bq[2], bq[3]);
          } else {
            mma_f16_16816(acc, h_lo(xr[0]), h_lo(xr[1]), h_hi(xr[0]), h_hi(xr[1]), qf[c][0][0],
                          qf[c][0][1]);
          }
          mma_f16_16816(acc, h_lo(y0), h_lo(y1), h_hi(y0), h_hi(y1), qf[c][1][0], qf[c][1][1]);
          mma_f16_16816(acc, h_lo(xr[2]), h_lo(xr[3]), h_hi(xr[2]), h_hi(xr[3]), qfl[c][0][0],
                        qfl[c][0][1]);
          mma_f16_16816(acc, h_lo(y2), h_lo(y3), h_hi(y2), h_hi(y3), qfl[c][1][0], qfl[c][1][1]);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float ks = krow2[r].get(gi);
          s2[r][0] = fmaf(ks, acc[2 * r], s2[r][0]);
          s2[r][1] = fmaf(ks, acc[2 * r + 1], s2[r][1]);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        s2[r][0] *= col_inv[0];
        s2[r][1] *= col_inv[1];
      }
      const int tokr = tok0 + 16 * slab + g;  // token of row 0 (row 1: + 8)
      if (tok0 + WROWS > lim_min) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int t = tokr + 8 * r;
          if (t >= col_lim[0]) s2[r][0] = kNegInf;
          if (t >= col_lim[1]) s2[r][1] = kNegInf;
          if (t >= sk_u && (tg & 1) == 0) {  // zero the row's V scales (see below)
            const uint32_t row = vsb + (rbase + 8 * r) * Cfg::SROW;
#pragma unroll
            for (int e = 0; e < Cfg::SROW / 2; ++e)
              asm volatile("st.shared.u16 [%0], %1;" ::"r"(row + 2 * e), "r"(0u) : "memory");
          }
        }
      }
      if (tok0 + WROWS > sk_u) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      // online softmax: column c's 32 rows are in lanes with tg = c/2 and
      // c/2 + 2 (xor 2), all g (xor 4, 8, 16)
      float mx[2];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        mx[cc] = fmaxf(s2[0][cc], s2[1][cc]);
        mx[cc] = fmaxf(mx[cc], __shfl_xor_sync(0xffffffffu, mx[cc], 2));
#pragma unroll
        for (int o = 4; o <= 16; o <<= 1)
          mx[cc] = fmaxf(mx[cc], __shfl_xor_sync(0xffffffffu, mx[cc], o));
      }
      const bool need = (mx[0] > m_run[0] + 8.0f) || (mx[1] > m_run[1] + 8.0f);
      if (__any_sync(0xffffffffu, need)) {
        float alpha[2];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const float mn = fmaxf(m_run[cc], mx[cc]);
          alpha[cc] = (mn == kNegInf) ? 1.0f : fast_exp2(m_run[cc] - mn);
          m_run[cc] = mn;
          l_run[cc] *= alpha[cc];
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            o_acc[c][j][0] *= alpha[0];
            o_acc[c][j][1] *= alpha[1];
            o_acc[c][j][2] *= alpha[0];
            o_acc[c][j][3] *= alpha[1];
          }
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          sp_acc[gi][0] *= alpha[0];
          sp_acc[gi][1] *= alpha[1];
          sp_acc[gi][2] *= alpha[0];
          sp_acc[gi][3] *= alpha[1];
        }
      }
      const float me[2] = {(m_run[0] == kNegInf) ? 0.0f : m_run[0],
                           (m_run[1] == kNegInf) ? 0.0f : m_run[1]};
      float p2[2][2];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          p2[r][cc] = fast_exp2(s2[r][cc] - me[cc]);
          l_run[cc] += p2[r][cc];
        }
      // P'' = P * v_scale * 2^vexp in fp32, one rounding to f16 (V codes
      // enter the MMAs as f16 magic-number operands, 5 integer ops per 8
      // codes), transposed into the B layout: lane (g, tg) then holds column
      // g; slab 0's MMAs take the columns g < 4, slab 1's the columns g >= 4.
      // vexp is a per-warp power-of-two exponent that keeps the step's
      // largest V scale times 2^vexp within [2^-6, 2^6], so P'' (P <= 2^8)
      // stays inside the f16 range with full precision; when a step falls
      // outside, vexp moves and the accumulators are rescaled exactly.
      uint32_t pb[NG][2];
      {
        SRow<NG, ST> va, vc;
        va.load(vsb + rbase * Cfg::SROW);
        vc.load(vsb + (rbase + 8) * Cfg::SROW);
        float vs0[NG], vs1[NG];
        float vmax = 0.0f;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          vs0[gi] = va.get(gi);
          vs1[gi] = vc.get(gi);
          vmax = fmaxf(vmax, fmaxf(vs0[gi], vs1[gi]));
        }
        const float vf = adjust_vexp(vmax);
        const float q00 = p2[0][0] * vf, q01 = p2[0][1] * vf;
        const float q10 = p2[1][0] * vf, q11 = p2[1][1] * vf;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          pb[gi][0] = movmatrix_trans(pack_f16x2(q00 * vs0[gi], q01 * vs0[gi]));
          pb[gi][1] = movmatrix_trans(pack_f16x2(q10 * vs1[gi], q11 * vs1[gi]));
        }
      }
      const uint32_t mask_a = g < 4 ? 0xFFFFFFFFu : 0u;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t msk = h == 0 ? mask_a : ~mask_a;
#pragma unroll
        for (int cp = 0; cp < NCH / 2; ++cp) {
          uint32_t wr[4];
          ldsm_x4_trans(vp + m_off[cp] + h * 16 * P_, wr);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 2 * cp + e;
            const int gi = c / CPG;
            const uint32_t b0 = pb[gi][0] & msk, b1 = pb[gi][1] & msk;
            // rows g: even dims (1024 + code), rows g + 8: odd dims (1024 + 16 code)
            const uint32_t wab = wr[2 * e], wcd = wr[2 * e + 1];
            const uint32_t yab = wab >> 8, ycd = wcd >> 8;
            mma_f16_16816(o_acc[c][0], h_lo(wab), h_hi(wab), h_lo(wcd), h_hi(wcd), b0, b1);
            mma_f16_16816(o_acc[c][1], h_lo(yab), h_hi(yab), h_lo(ycd), h_hi(ycd), b0, b1);
          }
        }
      }
      const uint32_t ones16 = 0x3C003C00u;  // f16x2 (1, 1)
#pragma unroll
      for (int gi = 0; gi < NG; ++gi)
        mma_f16_16816(sp_acc[gi], ones16, ones16, ones16, ones16, pb[gi][0], pb[gi][1]);
    } else {
    // ---------------- scores S^T[token][col] for two m16 sub-tiles -------
    // Per scale group: partial dot products on the tensor cores (the first
    // MMA of a group takes the -136*sum(q) bias as its C input), then the
    // group's K scale in fp32 into s[h][r][cc] (sub-tile h, row g / g+8,
    // column 2tg+cc).
    float s[2][2][2] = {};
    SRow<NG, ST> krow[2][2];  // K scale rows g, g+8 of both sub-tiles
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int r = 0; r < 2; ++r) krow[h][r].load(ksb + s_row0 + (16 * h + 8 * r) * Cfg::SROW);
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) {
      float acc[2][4];
#pragma unroll
      for (int cc = 0; cc < CPG; ++cc) {
        const int c = gi * CPG + cc;
        uint32_t xr[4];  // rows g, g+8 of sub-tile 0, then of sub-tile 1
        ldsm_x4(kp + k_off[c], xr);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t x0 = xr[2 * h], x1 = xr[2 * h + 1];
          float bq[4];
          if (cc == 0)
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(bq[0]), "=f"(bq[1]), "=f"(bq[2]), "=f"(bq[3])
                         : "r"(bias_s + ((warp * NG + gi) * 4 + tg) * 16));
          if constexpr (SPLIT) {
            const uint32_t a0 = nib_lo0(x0), a1 = nib_lo0(x1), a2 = nib_hi0(x0), a3 = nib_hi0(x1);
            const uint32_t a4 = nib_lo1(x0), a5 = nib_lo1(x1), a6 = nib_hi1(x0), a7 = nib_hi1(x1);
            if (cc == 0)
              mma_bf16_16816_c(acc[h], a0, a1, a2, a3, qf[c][0][0], qf[c][0][1], bq[0], bq[1],
                               bq[2], bq[3]);
            else
              mma_bf16_16816(acc[h], a0, a1, a2, a3, qf[c][0][0], qf[c][0][1]);
            mma_bf16_16816(acc[h], a4, a5, a6, a7, qf[c][1][0], qf[c][1][1]);
            mma_bf16_16816(acc[h], a0, a1, a2, a3, qfl[c][0][0], qfl[c][0][1]);
            mma_bf16_16816(acc[h], a4, a5, a6, a7, qfl[c][1][0], qfl[c][1][1]);
          } else {
            const uint32_t y0 = x0 >> 8, y1 = x1 >> 8;
            if (cc == 0)
              mma_f16_16816_c(acc[h], h_lo(x0), h_lo(x1), h_hi(x0), h_hi(x1), qf[c][0][0],
                              qf[c][0][1], bq[0], bq[1], bq[2], bq[3]);
            else
              mma_f16_16816(acc[h], h_lo(x0), h_lo(x1), h_hi(x0), h_hi(x1), qf[c][0][0],
                            qf[c][0][1]);
            mma_f16_16816(acc[h], h_lo(y0), h_lo(y1), h_hi(y0), h_hi(y1), qf[c][1][0],
                          qf[c][1][1]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float ks = krow[h][r].get(gi);
          s[h][r][0] = fmaf(ks, acc[h][2 * r], s[h][r][0]);
          s[h][r][1] = fmaf(ks, acc[h][2 * r + 1], s[h][r][1]);
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        s[h][r][0] *= col_inv[0];
        s[h][r][1] *= col_inv[1];
      }
    if (tok0 + WROWS > lim_min) {  // only rows that reach past a key limit need masks
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int t = tok0 + 16 * h + 8 * r + g;
          if (t >= col_lim[0]) s[h][r][0] = kNegInf;
          if (t >= col_lim[1]) s[h][r][1] = kNegInf;
          if (t >= sk_u && tg == 0) {
            // past the cache end the scale bulk copy (rounded up to 16 bytes)
            // may have brought in bytes from beyond the view: zero the row's V
            // scales so that P (= 0) times them stays 0
            const uint32_t row = vsb + s_row0 + (16 * h + 8 * r) * Cfg::SROW;
#pragma unroll
            for (int e = 0; e < Cfg::SROW / 2; ++e)
              asm volatile("st.shared.u16 [%0], %1;" ::"r"(row + 2 * e), "r"(0u) : "memory");
          }
        }
    }
    // (the zeroed scale rows are read by other lanes of the warp; the next TMA
    // into this stage is ordered after the writes by the proxy fence)
    if (tok0 + WROWS > sk_u) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
    }
    // ---------------- online softmax over 32 rows (lazy rescale) --------
    float mx[2];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      mx[cc] = fmaxf(fmaxf(s[0][0][cc], s[0][1][cc]), fmaxf(s[1][0][cc], s[1][1][cc]));
#pragma unroll
      for (int o = 4; o <= 16; o <<= 1)
        mx[cc] = fmaxf(mx[cc], __shfl_xor_sync(0xffffffffu, mx[cc], o));
    }
    const bool need = (mx[0] > m_run[0] + 8.0f) || (mx[1] > m_run[1] + 8.0f);
    if (__any_sync(0xffffffffu, need)) {
      float alpha[2];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const float mn = fmaxf(m_run[cc], mx[cc]);
        alpha[cc] = (mn == kNegInf) ? 1.0f : fast_exp2(m_run[cc] - mn);
        m_run[cc] = mn;
        l_run[cc] *= alpha[cc];
      }
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          o_acc[c][j][0] *= alpha[0];
          o_acc[c][j][1] *= alpha[1];
          o_acc[c][j][2] *= alpha[0];
          o_acc[c][j][3] *= alpha[1];
        }
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        sp_acc[gi][0] *= alpha[0];
        sp_acc[gi][1] *= alpha[1];
        sp_acc[gi][2] *= alpha[0];
        sp_acc[gi][3] *= alpha[1];
      }
    }
    const float me[2] = {(m_run[0] == kNegInf) ? 0.0f : m_run[0],
                         (m_run[1] == kNegInf) ? 0.0f : m_run[1]};
    float p[2][2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          p[h][r][cc] = fast_exp2(s[h][r][cc] - me[cc]);
          l_run[cc] += p[h][r][cc];
        }

    // ---------------- per sub-tile: P' = P * v_scale, then O^T += V^T P' -
    // (MODE 0: V codes as f16 operands, P'' = P * v_scale * 2^vexp)
    [[maybe_unused]] SRow<NG, ST> vrow[2][2];
    [[maybe_unused]] float vfac = 1.0f;
    if constexpr (!SPLIT) {
      float vmax = 0.0f;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          vrow[h][r].load(vsb + s_row0 + (16 * h + 8 * r) * Cfg::SROW);
#pragma unroll
          for (int gi = 0; gi < NG; ++gi) vmax = fmaxf(vmax, vrow[h][r].get(gi));
        }
      vfac = adjust_vexp(vmax);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t pb[NG][2];
      uint32_t pbl[SPLIT ? NG : 1][2];
      if constexpr (SPLIT) {
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          constexpr int SS = static_cast<int>(sizeof(ST));
          const float vs0 = lds_scale<ST>(vsb + s_row0 + (16 * h) * Cfg::SROW + gi * SS);
          const float vs1 = lds_scale<ST>(vsb + s_row0 + (16 * h + 8) * Cfg::SROW + gi * SS);
          const float a0 = p[h][0][0] * vs0, a1 = p[h][0][1] * vs0;
          const float c0 = p[h][1][0] * vs1, c1 = p[h][1][1] * vs1;
          const uint32_t u0 = pack_bf16x2(a0, a1);
          const uint32_t u1 = pack_bf16x2(c0, c1);
          pb[gi][0] = movmatrix_trans(u0);
          pb[gi][1] = movmatrix_trans(u1);
          const uint32_t l0 = pack_bf16x2(a0 - bf16lo_to_f32(u0), a1 - bf16hi_to_f32(u0));
          const uint32_t l1 = pack_bf16x2(c0 - bf16lo_to_f32(u1), c1 - bf16hi_to_f32(u1));
          pbl[gi][0] = movmatrix_trans(l0);
          pbl[gi][1] = movmatrix_trans(l1);
        }
      } else {
        // P'' = P * v_scale * 2^vexp in fp32, one rounding to f16, then
        // transposed into the B layout
        const float q00 = p[h][0][0] * vfac, q01 = p[h][0][1] * vfac;
        const float q10 = p[h][1][0] * vfac, q11 = p[h][1][1] * vfac;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          const float vs0 = vrow[h][0].get(gi), vs1 = vrow[h][1].get(gi);
          pb[gi][0] = movmatrix_trans(pack_f16x2(q00 * vs0, q01 * vs0));
          pb[gi][1] = movmatrix_trans(pack_f16x2(q10 * vs1, q11 * vs1));
        }
      }
#pragma unroll
      for (int cp = 0; cp < NCH / 2; ++cp) {
        // transposed loads give [t.B0, t.B1, t+1.B0, t+1.B1] words directly:
        // tokens 2tg, 2tg+1 (then +8, +9), bytes 2g, 2g+1 of the chunk
        uint32_t wr[4];
        ldsm_x4_trans(vp + m_off[cp] + h * 16 * P_, wr);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = 2 * cp + e;
          const int gi = c / CPG;
          const uint32_t wab = wr[2 * e], wcd = wr[2 * e + 1];
          if constexpr (SPLIT) {
            const uint32_t v0 = nib_lo0(wab), v1 = nib_hi0(wab), v2 = nib_lo0(wcd), v3 = nib_hi0(wcd);
            const uint32_t v4 = nib_lo1(wab), v5 = nib_hi1(wab), v6 = nib_lo1(wcd), v7 = nib_hi1(wcd);
            mma_bf16_16816(o_acc[c][0], v0, v1, v2, v3, pb[gi][0], pb[gi][1]);
            mma_bf16_16816(o_acc[c][1], v4, v5, v6, v7, pb[gi][0], pb[gi][1]);
            mma_bf16_16816(o_acc[c][0], v0, v1, v2, v3, pbl[gi][0], pbl[gi][1]);
            mma_bf16_16816(o_acc[c][1], v4, v5, v6, v7, pbl[gi][0], pbl[gi][1]);
          } else {
            const uint32_t yab = wab >> 8, ycd = wcd >> 8;
            mma_f16_16816(o_acc[c][0], h_lo(wab), h_hi(wab), h_lo(wcd), h_hi(wcd), pb[gi][0],
                          pb[gi][1]);
            mma_f16_16816(o_acc[c][1], h_lo(yab), h_hi(yab), h_lo(ycd), h_hi(ycd), pb[gi][0],
                          pb[gi][1]);
          }
        }
      }
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        if constexpr (SPLIT) {
          mma_bf16_16816(sp_acc[gi], ones, ones, ones, ones, pb[gi][0], pb[gi][1]);
          mma_bf16_16816(sp_acc[gi], ones, ones, ones, ones, pbl[gi][0], pbl[gi][1]);
        } else {
          constexpr uint32_t ones16 = 0x3C003C00u;  // f16x2 (1, 1)
          mma_f16_16816(sp_acc[gi], ones16, ones16, ones16, ones16, pb[gi][0], pb[gi][1]);
        }
      }
    }

    }  // PAIR / unpaired

    // ---------------- release the stage, refill, flush at unit end ------
    // Each warp counts itself out of the stage (acq_rel: its reads of the
    // stage happen before); the LAST warp to finish refills it at once, so
    // no warp ever waits for the others.  Counters only grow: the last
    // arrival of round r of a stage sees NWARP * (r + 1) - 1.
    __syncwarp();
    if (lane == 0) {
      uint32_t old;
      asm volatile(KV4_RELEASE_ATOM " %0, [%1], 1;"
                   : "=r"(old)
                   : "r"(smem_u32(&sh_done[stage]))
                   : "memory");
      if (old == static_cast<uint32_t>(NWARP * (i / Cfg::STAGES + 1) - 1) &&
          i + Cfg::STAGES < ntiles)
        issue(i + Cfg::STAGES);
    }
  }
  flush();
  if (sh_abort && tid == 0) {
    // drain: wait (bounded) for the loads this CTA may still have in flight
    for (int i = max(0, ntiles - Cfg::STAGES); i < ntiles; ++i) {
      const int s = i % Cfg::STAGES;
      mbar_wait_bounded(bar_base + 8 * s, (i / Cfg::STAGES) & 1, 4 * P.wait_limit);
    }
  }
}

// ===========================================================================
// merge of shard partials (multi-GPU sequence sharding)
// ===========================================================================
struct LseParams {
  const float *po;
  const float *pl;
  int64_t nparts, rows;
  int d;
  void *out;
  int64_t os[4];
  int out_dtype;
  int64_t n1, n2;  // out dims 1, 2
};

__global__ void __launch_bounds__(128) kv4_lse_merge(const LseParams P) {
  const int64_t r = blockIdx.x;
  float M = kNegInf;
  for (int64_t p = 0; p < P.nparts; ++p) M = fmaxf(M, P.pl[p * P.rows + r]);
  float W = 0.0f;
  for (int64_t p = 0; p < P.nparts; ++p)
    W += (M == kNegInf) ? 0.0f : expf(P.pl[p * P.rows + r] - M);
  const float invW = W > 0.0f ? 1.0f / W : 0.0f;
  const int64_t i2 = r % P.n2, i01 = r / P.n2, i1 = i01 % P.n1, i0 = i01 / P.n1;
  for (int dd = threadIdx.x; dd < P.d; dd += blockDim.x) {
    float o = 0.0f;
    for (int64_t p = 0; p < P.nparts; ++p) {
      const float lp = P.pl[p * P.rows + r];
      const float w = (M == kNegInf) ? 0.0f : expf(lp - M);
      o += w * P.po[(p * P.rows + r) * P.d + dd];
    }
    store_from_f32(P.out, P.out_dtype, i0 * P.os[0] + i1 * P.os[1] + i2 * P.os[2] + dd * P.os[3],
                   o * invW);
  }
}

// ===========================================================================
// host side
// ===========================================================================
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct Shape {
  int64_t B, Hq, Hkv, sq, sk, d, pw, ng;
  int G;
};

static bool is_float(int dt) { return dt == KV4_F32 || dt == KV4_F16 || dt == KV4_BF16; }

static int validate(const kv4_tensor *q, const kv4_tensor *kp, const kv4_tensor *ks,
                    const kv4_tensor *vp, const kv4_tensor *vs, int G, Shape &S) {
  if (!q || !kp || !ks || !vp || !vs) return KV4_ERR_INVALID;
  if (G <= 0) return KV4_ERR_INVALID;
  if (!is_float(q->dtype) || kp->dtype != KV4_U8 || vp->dtype != KV4_U8 || !is_float(ks->dtype) ||
      ks->dtype != vs->dtype)
    return KV4_ERR_DTYPE;
  for (int i = 0; i < 4; ++i) {
    if (kp->shape[i] != vp->shape[i] || ks->shape[i] != vs->shape[i]) return KV4_ERR_SHAPE;
    if (i < 3 && kp->shape[i] != ks->shape[i]) return KV4_ERR_SHAPE;
  }
  S.B = q->shape[0];
  S.Hq = q->shape[1];
  S.sq = q->shape[2];
  S.d = q->shape[3];
  S.Hkv = kp->shape[1];
  S.sk = kp->shape[2];
  S.pw = kp->shape[3];
  S.ng = ks->shape[3];
  S.G = G;
  if (kp->shape[0] != S.B) return KV4_ERR_SHAPE;
  if (S.Hkv <= 0 || S.Hq <= 0 || S.Hq % S.Hkv != 0) return KV4_ERR_INVALID;
  if (S.pw < (S.d + 1) / 2 || S.ng < (S.d + G - 1) / G) return KV4_ERR_SHAPE;
  if (S.d > 512) return KV4_ERR_UNSUPPORTED;
  return KV4_OK;
}

struct Plan {
  int path;  // 1 fast, 2 generic
  int D, sdt;
  bool split;
  int mode;  // kernel MODE: 0 bf16 q, 1 split q, 2 paired columns
  int cs;    // cluster size of the split-K merge (1: no clusters)
  int hc, ncols, tpu, L, maxp, ctas, units;
  int64_t total_tiles;
  size_t ws_bytes;
  bool need_merge;
};

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static bool fast_eligible(const kv4_tensor *q, const kv4_tensor *kp, const kv4_tensor *ks,
                          const kv4_tensor *vp, const kv4_tensor *vs, const Shape &S) {
  if (!(S.d == 64 || S.d == 128 || S.d == 256)) return false;
  if (!(S.G == 32 || S.G == 64 || S.G == 128) || S.G > S.d || S.d % S.G) return false;
  if (S.sk <= 0 || S.sk >= (1LL << 31) / 8) return false;
  if (S.B * S.Hkv * ((S.Hq / S.Hkv * S.sq + NCOL - 1) / NCOL) * ((S.sk + TOK - 1) / TOK) >=
      (1LL << 31))
    return false;
  const int64_t ng = S.d / S.G;
  const int ss = dtype_size(ks->dtype);
  for (const kv4_tensor *t : {kp, vp}) {
    if (!aligned16(t->data) || t->stride[3] != 1 || t->stride[2] % 16) return false;
    if (t->shape[1] > 1 && t->stride[1] % 16) return false;
    if (t->shape[0] > 1 && t->stride[0] % 16) return false;
  }
  for (const kv4_tensor *t : {ks, vs}) {
    if (!aligned16(t->data) || t->stride[3] != 1 || t->shape[3] != ng || t->stride[2] != ng)
      return false;
    if (t->shape[1] > 1 && (t->stride[1] * ss) % 16) return false;
    if (t->shape[0] > 1 && (t->stride[0] * ss) % 16) return false;
  }
  if (S.Hq / S.Hkv * S.sq > 8 * NCOL) return false;  // long query blocks: generic
  (void)q;
  return get_encode() != nullptr;
}

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  return dev;
}

// Occupancy of a fast-path instantiation on the current device.  The dynamic
// shared-memory attribute is per device (per context), so it is set, and the
// occupancy queried, once for every device that launches the kernel.
template <int D, int G, typename ST, int MODE, bool PAGED = false>
static int occupancy_of() {
  static std::atomic<int> occ[64];
  static std::mutex mu;
  const int dev = current_device();
  int o = occ[dev].load(std::memory_order_acquire);
  if (o > 0) return o;
  std::lock_guard<std::mutex> lock(mu);
  if ((o = occ[dev].load(std::memory_order_relaxed)) > 0) return o;
  using Cfg = FastCfg<D, G, ST>;
  cudaFuncSetAttribute(kv4_attn_fast<D, G, ST, MODE, PAGED>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  o = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kv4_attn_fast<D, G, ST, MODE, PAGED>, 128,
                                                    Cfg::SMEM) != cudaSuccess ||
      o < 1)
    o = 1;
  occ[dev].store(o, std::memory_order_release);
  return o;
}

static int sm_count() {  // per device, queried once
  static std::atomic<int> cache[64];
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return n;
  if (dev >= 0 && dev < 64 && (n = cache[dev].load(std::memory_order_relaxed)) > 0) return n;
  n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

static int fast_occupancy(int D, int G, int sdt, int mode) {
#define KV4_OCC(DD, GG, STT)                                                     \
  if (D == DD && G == GG)                                                        \
    return mode == 1 ? occupancy_of<DD, GG, STT, 1>()                            \
                     : (mode == 2 ? occupancy_of<DD, GG, STT, 2>() : occupancy_of<DD, GG, STT, 0>());
#define KV4_OCC_S(STT)                                                               \
  KV4_OCC(64, 32, STT) KV4_OCC(64, 64, STT) KV4_OCC(128, 32, STT) KV4_OCC(128, 64, STT) \
      KV4_OCC(128, 128, STT) KV4_OCC(256, 32, STT) KV4_OCC(256, 64, STT)              \
          KV4_OCC(256, 128, STT)
#ifdef KV4_DEV_SUBSET
  if (sdt == KV4_BF16) { KV4_OCC(128, 32, __nv_bfloat16) }
#else
  if (sdt == KV4_BF16) { KV4_OCC_S(__nv_bfloat16) }
  else if (sdt == KV4_F16) { KV4_OCC_S(__half) }
  else { KV4_OCC_S(float) }
#endif
#undef KV4_OCC_S
#undef KV4_OCC
  return 1;
}

// Split-K workspace: partial slots [units * parts] then first-level group
// slots [units * groups] (more than one group only), each NCOL x (D + 1)
// floats; the counters sit at the END of the caller's buffer: [units][groups]
// first-level counters, then [units] unit counters.
static int merge_groups(int parts) {
  const int g = (parts + MERGE_GROUP - 1) / MERGE_GROUP;
  return g > 1 ? g : 0;
}
static size_t counter_bytes_of(int units, int parts) {
  return static_cast<size_t>(units) * (1 + merge_groups(parts)) * sizeof(int);
}
static size_t ws_bytes_of(int units, int parts, int D) {
  if (parts <= 1) return 0;
  const size_t slots = static_cast<size_t>(units) * (parts + merge_groups(parts));
  return (counter_bytes_of(units, parts) + 15) / 16 * 16 +
         slots * NCOL * (static_cast<size_t>(D) + 1) * sizeof(float);
}

// Split-K parts of a unit merge inside one thread-block cluster (through
// distributed shared memory) when there are at most kMaxCluster of them;
// more parts merge through global memory in two levels (measured: clusters
// of 8 plus a global level were slower than the global two-level merge).
constexpr int kMaxCluster = 8;
static int cluster_size_of(int64_t k) {
  return static_cast<int>(k > 1 && k <= kMaxCluster ? k : 1);
}

static void make_plan(const kv4_tensor *q, const kv4_tensor *kp, const kv4_tensor *ks,
                      const kv4_tensor *vp, const kv4_tensor *vs, const Shape &S,
                      const kv4_attn_opts *opts, Plan &pl) {
  pl = Plan{};
  const bool force_generic = opts && opts->force_generic;
  if (!force_generic && fast_eligible(q, kp, ks, vp, vs, S)) {
    pl.path = 1;
    pl.D = static_cast<int>(S.d);
    pl.sdt = ks->dtype;
    pl.split = q->dtype != KV4_BF16;
    const int R = static_cast<int>(S.Hq / S.Hkv);
    pl.ncols = R * static_cast<int>(S.sq);
    pl.hc = (pl.ncols + NCOL - 1) / NCOL;
    pl.units = static_cast<int>(S.B * S.Hkv * pl.hc);
    pl.tpu = static_cast<int>((S.sk + TOK - 1) / TOK);
    pl.total_tiles = static_cast<int64_t>(pl.units) * pl.tpu;
    pl.mode = pl.split ? 1 : (pl.ncols <= 4 ? 2 : 0);
    const int occ = fast_occupancy(pl.D, S.G, pl.sdt, pl.mode);
    int64_t target = static_cast<int64_t>(sm_count()) * occ;
    if (opts && opts->max_ctas > 0) target = std::min<int64_t>(target, opts->max_ctas);
    // split-K: kparts CTAs per unit, as many as fit one wave of resident CTAs
    int64_t k = std::max<int64_t>(1, target / pl.units);
    // at least 4 tiles per CTA: shorter parts spend more time in their
    // prologue and merge than in streaming (measured: batch-1 16K context
    // takes 17.5 us with 32 parts of 4 tiles, 24 us with 74 parts) -- except
    // that up to 8 parts of >= 2 tiles, which merge inside one cluster, pay
    // (measured: batch-1 2K context 9.7 us with 4 parts, 7.9 us with 8)
    k = std::min<int64_t>(
        k, std::max<int64_t>({1, pl.tpu / 4, std::min<int64_t>(kMaxCluster, pl.tpu / 2)}));
    if (opts && opts->tiles_per_cta > 0) k = (pl.tpu + opts->tiles_per_cta - 1) / opts->tiles_per_cta;
    k = std::min<int64_t>(k, pl.tpu);
    pl.cs = cluster_size_of(k);
    pl.maxp = static_cast<int>(k);
    pl.L = static_cast<int>((pl.tpu + k - 1) / k);
    pl.ctas = static_cast<int>(static_cast<int64_t>(pl.units) * k);
    pl.need_merge = k > 1;
    pl.ws_bytes = ws_bytes_of(pl.units, pl.maxp, pl.D);
  } else {
    pl.path = 2;
    pl.ws_bytes = 0;
    pl.ctas = static_cast<int>(S.B * S.Hq * S.sq);
    pl.need_merge = false;
  }
}

// Packed K/V map: 4-D {row bytes, token, head, batch}, box {P, TOK, 1, 1},
// swizzled by the row width (32/64/128 B) so fragment loads are bank-conflict free.
static int encode_packed(CUtensorMap *tm, const kv4_tensor *t, int row_bytes, int tokens) {
  auto enc = get_encode();
  const int64_t sh = t->shape[1] > 1 ? t->stride[1] : t->stride[2] * t->shape[2];
  const int64_t sb = t->shape[0] > 1 ? t->stride[0] : sh * t->shape[1];
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(t->shape[3]), static_cast<cuuint64_t>(t->shape[2]),
                        static_cast<cuuint64_t>(t->shape[1]),
                        static_cast<cuuint64_t>(t->shape[0])};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t->stride[2]),
                           static_cast<cuuint64_t>((sh + 15) / 16 * 16),
                           static_cast<cuuint64_t>((sb + 15) / 16 * 16)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(row_bytes), static_cast<cuuint32_t>(tokens), 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUtensorMapSwizzle sw = row_bytes == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                          : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, t->data, dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KV4_OK : KV4_ERR_LAYOUT;
}


// The last few encoded maps, keyed by everything the encoding reads: a decode
// loop calls with the same cache views again and again, and encoding is a
// driver call on every launch otherwise.
static int encode_packed_cached(CUtensorMap *tm, const kv4_tensor *t, int row_bytes, int tokens) {
  struct Entry {
    const void *data;
    int64_t shape[4], stride[4];
    int row_bytes, tokens;
    CUtensorMap map;
    bool used;
  };
  static Entry ring[16];
  static int next = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (Entry &e : ring)
    if (e.used && e.data == t->data && e.row_bytes == row_bytes && e.tokens == tokens &&
        std::memcmp(e.shape, t->shape, sizeof(e.shape)) == 0 &&
        std::memcmp(e.stride, t->stride, sizeof(e.stride)) == 0) {
      *tm = e.map;
      return KV4_OK;
    }
  const int rc = encode_packed(tm, t, row_bytes, tokens);
  if (rc) return rc;
  Entry &e = ring[next];
  next = (next + 1) % 16;
  e.data = t->data;
  std::memcpy(e.shape, t->shape, sizeof(e.shape));
  std::memcpy(e.stride, t->stride, sizeof(e.stride));
  e.row_bytes = row_bytes;
  e.tokens = tokens;
  e.map = *tm;
  e.used = true;
  return KV4_OK;
}

template <int D, int G, typename ST, int MODE, bool PAGED>
static int launch_fast_t(const FastParams &FP, const Plan &pl, const kv4_tensor *kp,
                         const kv4_tensor *ks, const kv4_tensor *vp, const kv4_tensor *vs,
                         cudaStream_t st) {
  using Cfg = FastCfg<D, G, ST>;
  CUtensorMap tkp, tvp;
  int rc;
  const int box_rows = FP.page > 0 ? FP.page : TOK;  // paged: one box per page
  if ((rc = encode_packed_cached(&tkp, kp, Cfg::P, box_rows))) return rc;
  if ((rc = encode_packed_cached(&tvp, vp, Cfg::P, box_rows))) return rc;
  occupancy_of<D, G, ST, MODE, PAGED>();  // sets the smem attribute once
  int smem = Cfg::SMEM;
  if (FP.page > 0) {  // room for the block-table slice after the staged append row
    smem += 16 + FP.bt_slots * 4;
    // the attribute is per device: remember the largest size set on each
    static std::atomic<int> smem_set[64];
    const int dev = current_device();
    if (smem > std::max(smem_set[dev].load(std::memory_order_acquire), Cfg::SMEM)) {
      static std::mutex mu;
      std::lock_guard<std::mutex> lock(mu);
      if (smem > smem_set[dev].load(std::memory_order_relaxed)) {
        rc = cuda_status(cudaFuncSetAttribute(kv4_attn_fast<D, G, ST, MODE, PAGED>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        if (rc) return rc;
        smem_set[dev].store(smem, std::memory_order_release);
      }
    }
  }
  if (FP.cs > 1 || FP.early) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(pl.ctas));
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    unsigned na = 0;
    if (FP.cs > 1) {  // the split-K parts of a unit merge inside a thread-block cluster
      attr[na].id = cudaLaunchAttributeClusterDimension;
      attr[na].val.clusterDim.x = static_cast<unsigned>(FP.cs);
      attr[na].val.clusterDim.y = 1;
      attr[na].val.clusterDim.z = 1;
      ++na;
    }
    if (FP.early) {  // may start while the previous kernel in the stream drains
      attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[na].val.programmaticStreamSerializationAllowed = 1;
      ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    rc = cuda_status(cudaLaunchKernelEx(&cfg, kv4_attn_fast<D, G, ST, MODE, PAGED>, FP, tkp, tvp));
    if (rc) return rc;
  } else {
    kv4_attn_fast<D, G, ST, MODE, PAGED><<<pl.ctas, 128, smem, st>>>(FP, tkp, tvp);
  }
  rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  return rc;
}

template <int D, int G, typename ST>
static int launch_fast_s(const FastParams &FP, const Plan &pl, const kv4_tensor *kp,
                         const kv4_tensor *ks, const kv4_tensor *vp, const kv4_tensor *vs,
                         cudaStream_t st) {
  if (FP.page > 0) {
    if (pl.mode == 1) return launch_fast_t<D, G, ST, 1, true>(FP, pl, kp, ks, vp, vs, st);
    if (pl.mode == 2) return launch_fast_t<D, G, ST, 2, true>(FP, pl, kp, ks, vp, vs, st);
    return launch_fast_t<D, G, ST, 0, true>(FP, pl, kp, ks, vp, vs, st);
  }
  if (pl.mode == 1) return launch_fast_t<D, G, ST, 1, false>(FP, pl, kp, ks, vp, vs, st);
  if (pl.mode == 2) return launch_fast_t<D, G, ST, 2, false>(FP, pl, kp, ks, vp, vs, st);
  return launch_fast_t<D, G, ST, 0, false>(FP, pl, kp, ks, vp, vs, st);
}

template <typename ST>
static int launch_fast_st(const FastParams &FP, const Plan &pl, const kv4_tensor *kp,
                          const kv4_tensor *ks, const kv4_tensor *vp, const kv4_tensor *vs,
                          cudaStream_t st) {
  const int D = pl.D, G = FP.c.G;
#define KV4_L(DD, GG) \
  if (D == DD && G == GG) return launch_fast_s<DD, GG, ST>(FP, pl, kp, ks, vp, vs, st);
#ifdef KV4_DEV_SUBSET  // development builds: the Llama decode shape only
  KV4_L(128, 32)
#else
  KV4_L(64, 32) KV4_L(64, 64) KV4_L(128, 32) KV4_L(128, 64) KV4_L(128, 128) KV4_L(256, 32)
      KV4_L(256, 64) KV4_L(256, 128)
#endif
#undef KV4_L
  return KV4_ERR_UNSUPPORTED;
}

// Paged cache: page pools plus a block table and per-sequence lengths.
struct PagedJob {
  const int32_t *bt;
  int64_t bt_stride, max_blocks;
  const int32_t *seq_lens;
  int64_t max_seq_len;
};

static bool page_size_ok(int64_t p) { return p == 8 || p == 16 || p == 32 || p == 64 || p == 128; }

static int validate_paged(const kv4_tensor *q, const kv4_tensor *kp, const kv4_tensor *ks,
                          const kv4_tensor *vp, const kv4_tensor *vs, int G, const PagedJob &J,
                          Shape &S) {
  if (!q || !kp || !ks || !vp || !vs || !J.bt || !J.seq_lens) return KV4_ERR_INVALID;
  if (G <= 0) return KV4_ERR_INVALID;
  if (!is_float(q->dtype) || kp->dtype != KV4_U8 || vp->dtype != KV4_U8 || !is_float(ks->dtype) ||
      ks->dtype != vs->dtype)
    return KV4_ERR_DTYPE;
  for (int i = 0; i < 4; ++i) {
    if (kp->shape[i] != vp->shape[i] || ks->shape[i] != vs->shape[i]) return KV4_ERR_SHAPE;
    if (i < 3 && kp->shape[i] != ks->shape[i]) return KV4_ERR_SHAPE;
  }
  S.B = q->shape[0];
  S.Hq = q->shape[1];
  S.sq = q->shape[2];
  S.d = q->shape[3];
  S.Hkv = kp->shape[1];
  S.sk = J.max_seq_len;
  S.pw = kp->shape[3];
  S.ng = ks->shape[3];
  S.G = G;
  if (S.Hkv <= 0 || S.Hq <= 0 || S.Hq % S.Hkv != 0) return KV4_ERR_INVALID;
  if (S.pw < (S.d + 1) / 2 || S.ng < (S.d + G - 1) / G) return KV4_ERR_SHAPE;
  if (!page_size_ok(kp->shape[2])) return KV4_ERR_UNSUPPORTED;
  if (J.max_seq_len < 1 || J.max_blocks < 1 || J.max_seq_len > J.max_blocks * kp->shape[2] ||
      J.bt_stride < J.max_blocks)
    return KV4_ERR_SHAPE;
  if (kp->shape[0] < 1 || kp->shape[0] > INT_MAX) return KV4_ERR_SHAPE;
  return KV4_OK;
}

// Recompute the split-dependent fields of a fast plan for kparts = k.
static void set_parts(Plan &pl, int64_t k) {
  k = std::max<int64_t>(1, std::min<int64_t>(k, pl.tpu));
  pl.cs = cluster_size_of(k);
  pl.maxp = static_cast<int>(k);
  pl.L = static_cast<int>((pl.tpu + k - 1) / k);
  pl.ctas = static_cast<int>(static_cast<int64_t>(pl.units) * k);
  pl.need_merge = k > 1;
  pl.ws_bytes = ws_bytes_of(pl.units, pl.maxp, pl.D);
}

// paged: keep each CTA's block-table slice within 48 KB of shared memory
constexpr int kMaxBtBytes = 48 << 10;
static void paged_plan(Plan &pl, int page) {
  const int ppt = TOK / page;
  int64_t k = pl.maxp;
  while (static_cast<int64_t>((pl.tpu + k - 1) / k) * ppt * 4 > kMaxBtBytes && k < pl.tpu) ++k;
  if (k != pl.maxp) set_parts(pl, k);
}

// New tokens appended into the last rows of the cache views before attention.
struct AppendJob {
  const kv4_tensor *k, *v;  // [B, Hkv, n, d]
  int tie;
};

static int check_append(const AppendJob &A, const Shape &S) {
  if (!A.k || !A.v) return KV4_ERR_INVALID;
  if (!tie_mode_ok(A.tie)) return KV4_ERR_INVALID;
  if (!is_float(A.k->dtype) || A.v->dtype != A.k->dtype) return KV4_ERR_DTYPE;
  for (int i = 0; i < 4; ++i)
    if (A.k->shape[i] != A.v->shape[i]) return KV4_ERR_SHAPE;
  if (A.k->shape[0] != S.B || A.k->shape[1] != S.Hkv || A.k->shape[3] != S.d)
    return KV4_ERR_SHAPE;
  if (A.k->shape[2] < 1 || A.k->shape[2] > S.sk) return KV4_ERR_SHAPE;
  return KV4_OK;
}

static int run_attention(const kv4_tensor *q, const kv4_tensor *kp, const kv4_tensor *ks,
                         const kv4_tensor *vp, const kv4_tensor *vs, const kv4_tensor *out,
                         const kv4_tensor *lse, int mode, int64_t k_offset, int64_t sk_total,
                         int G, int is_causal, float sm_scale, void *ws, size_t ws_bytes,
                         const kv4_attn_opts *opts, cudaStream_t st,
                         const AppendJob *app = nullptr, const PagedJob *pgj = nullptr) {
  Shape S;
  int rc = pgj ? validate_paged(q, kp, ks, vp, vs, G, *pgj, S) : validate(q, kp, ks, vp, vs, G, S);
  if (rc) return rc;
  if (pgj && (app || mode != OUT_FINAL)) return KV4_ERR_UNSUPPORTED;
  if (app && (rc = check_append(*app, S))) return rc;
  if (!out) return KV4_ERR_INVALID;
  for (int i = 0; i < 4; ++i)
    if (out->shape[i] != q->shape[i]) return KV4_ERR_SHAPE;
  if (mode == OUT_FINAL) {
    if (out->dtype != q->dtype) return KV4_ERR_DTYPE;
  } else {
    if (out->dtype != KV4_F32 || !lse || lse->dtype != KV4_F32) return KV4_ERR_DTYPE;
    for (int i = 0; i < 3; ++i)
      if (lse->shape[i] != q->shape[i]) return KV4_ERR_SHAPE;
  }
  if (S.B == 0 || S.Hq == 0 || S.sq == 0 || S.d == 0) return KV4_OK;

  AttnCommon Cm{};
  Cm.q = q->data;
  Cm.q_dtype = q->dtype;
  Cm.out = out->data;
  Cm.out_dtype = out->dtype;
  for (int i = 0; i < 4; ++i) {
    Cm.qs[i] = q->stride[i];
    Cm.os[i] = out->stride[i];
  }
  if (lse) {
    Cm.lse = static_cast<float *>(lse->data);
    for (int i = 0; i < 3; ++i) Cm.ls[i] = lse->stride[i];
  }
  Cm.mode = mode;
  Cm.B = static_cast<int>(S.B);
  Cm.Hq = static_cast<int>(S.Hq);
  Cm.Hkv = static_cast<int>(S.Hkv);
  Cm.R = static_cast<int>(S.Hq / S.Hkv);
  Cm.sq = static_cast<int>(S.sq);
  Cm.sk = static_cast<int>(S.sk);
  Cm.d = static_cast<int>(S.d);
  Cm.G = G;
  Cm.causal = is_causal ? 1 : 0;
  Cm.k_offset = mode == OUT_PARTIAL ? k_offset : 0;
  Cm.sk_total = mode == OUT_PARTIAL ? sk_total : S.sk;
  const float sc = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(static_cast<float>(S.d));
  Cm.scale_log2 = sc * kLog2e;

  Plan pl;
  make_plan(q, kp, ks, vp, vs, S, opts, pl);
  if (pgj) {  // the paged layout runs on the fast path only
    if (pl.path != 1) return KV4_ERR_UNSUPPORTED;
    paged_plan(pl, static_cast<int>(kp->shape[2]));
  }
  // one new token on the fast path is quantized inside the attention launch;
  // anything else is appended by the quantize kernel first (same stream)
  const bool fuse_app = app && pl.path == 1 && app->k->shape[2] == 1 &&
                        app->k->stride[3] == 1 && app->v->stride[3] == 1;
  if (pl.path == 1 && pl.ws_bytes > 0 && (ws == nullptr || ws_bytes < pl.ws_bytes))
    return KV4_ERR_WORKSPACE;
  if (app && !fuse_app) {
    rc = kv4_append_kv(app->k, app->v, kp, ks, vp, vs, S.sk - app->k->shape[2], G, app->tie, st);
    if (rc) return rc;
  }
  if (pl.path == 1) {
    FastParams FP{};
    FP.app_row = -1;
    if (pgj) {
      FP.page = static_cast<int>(kp->shape[2]);
      FP.npages = static_cast<int>(kp->shape[0]);
      FP.bt = pgj->bt;
      FP.bt_stride = pgj->bt_stride;
      FP.seq_lens = pgj->seq_lens;
      FP.bt_slots = pl.L * (TOK / FP.page);
    }
    if (fuse_app) {
      FP.app_row = static_cast<int>(S.sk - 1);
      FP.app_tie = app->tie;
      FP.kn_dtype = app->k->dtype;
      FP.kn = app->k->data;
      FP.vn = app->v->data;
      FP.kn_sb = app->k->stride[0];
      FP.kn_sh = app->k->stride[1];
      FP.vn_sb = app->v->stride[0];
      FP.vn_sh = app->v->stride[1];
      FP.kpw = static_cast<uint8_t *>(kp->data);
      FP.vpw = static_cast<uint8_t *>(vp->data);
      FP.kp_sb = kp->stride[0];
      FP.kp_sh = kp->stride[1];
      FP.kp_st = kp->stride[2];
      FP.vp_sb = vp->stride[0];
      FP.vp_sh = vp->stride[1];
      FP.vp_st = vp->stride[2];
    }
    FP.c = Cm;
    FP.ncols = pl.ncols;
    FP.hc = pl.hc;
    FP.tpu = pl.tpu;
    FP.L = pl.L;
    FP.total_tiles = pl.total_tiles;
    FP.maxp = pl.maxp;
    {
      const int ss = dtype_size(ks->dtype);
      FP.ks = static_cast<const char *>(ks->data);
      FP.vs = static_cast<const char *>(vs->data);
      FP.ks_sb = ks->stride[0] * ss;
      FP.ks_sh = ks->stride[1] * ss;
      FP.vs_sb = vs->stride[0] * ss;
      FP.vs_sh = vs->stride[1] * ss;
    }
    // workspace: partial o, then lse from the front; the per-unit counters
    // (zero between calls) are the LAST units*4 bytes of the caller's buffer.
    FP.ws_o = static_cast<float *>(ws);
    FP.counters = pl.ws_bytes ? reinterpret_cast<int *>(
                                    static_cast<char *>(ws) +
                                    ((ws_bytes - static_cast<size_t>(pl.units) * 4) & ~size_t(3)))
                              : nullptr;
    FP.units = pl.units;
    FP.cs = pl.cs;
    FP.drop_last = (opts && opts->debug_drop_last_tile) ? 1 : 0;
    // (not behind the separate append kernel this call launches itself)
    FP.early = (opts && opts->early_start && FP.page == 0 && !(app && !fuse_app)) ? 1 : 0;
    // long parts merged inside a cluster leave no head or tail worth
    // overlapping (measured: the 8B batch-16 step, 3 parts of 11 tiles, was
    // 0.6 us slower with early start; every global-merge or short-part plan
    // measured faster)
    if (pl.cs > 1 && pl.L >= 8) FP.early = 0;
    FP.wait_limit = FP.drop_last ? 16u : (1u << 14);
    FP.ws_lse = pl.ws_bytes ? FP.ws_o + static_cast<size_t>(pl.units) *
                                            (pl.maxp + merge_groups(pl.maxp)) * NCOL * pl.D
                            : nullptr;
    if (pl.sdt == KV4_BF16) return launch_fast_st<__nv_bfloat16>(FP, pl, kp, ks, vp, vs, st);
#ifndef KV4_DEV_SUBSET
    if (pl.sdt == KV4_F16) return launch_fast_st<__half>(FP, pl, kp, ks, vp, vs, st);
    return launch_fast_st<float>(FP, pl, kp, ks, vp, vs, st);
#else
    return KV4_ERR_UNSUPPORTED;
#endif
  }
  // generic
  GenParams GP{};
  GP.c = Cm;
  GP.kp = static_cast<const uint8_t *>(kp->data);
  GP.vp = static_cast<const uint8_t *>(vp->data);
  GP.ks = ks->data;
  GP.vs = vs->data;
  for (int i = 0; i < 4; ++i) {
    GP.kps[i] = kp->stride[i];
    GP.vps[i] = vp->stride[i];
    GP.kss[i] = ks->stride[i];
    GP.vss[i] = vs->stride[i];
  }
  GP.s_dtype = ks->dtype;
  dim3 grid(static_cast<unsigned>(S.B * S.Hq), static_cast<unsigned>(S.sq));
  if (S.d <= 64) kv4_attn_generic<2><<<grid, 128, 0, st>>>(GP);
  else if (S.d <= 128) kv4_attn_generic<4><<<grid, 128, 0, st>>>(GP);
  else if (S.d <= 256) kv4_attn_generic<8><<<grid, 128, 0, st>>>(GP);
  else kv4_attn_generic<16><<<grid, 128, 0, st>>>(GP);
  return cuda_status(cudaGetLastError());
}

}  // namespace kv4

using namespace kv4;

extern "C" int kv4_attention(const kv4_tensor *q, const kv4_tensor *k_packed,
                             const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                             const kv4_tensor *v_scales, const kv4_tensor *out, int group_size,
                             int is_causal, float sm_scale, void *workspace,
                             size_t workspace_bytes, const kv4_attn_opts *opts, void *stream) {
  return run_attention(q, k_packed, k_scales, v_packed, v_scales, out, nullptr, OUT_FINAL, 0, 0,
                       group_size, is_causal, sm_scale, workspace, workspace_bytes, opts,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int kv4_append_attention(const kv4_tensor *q, const kv4_tensor *k_new,
                                    const kv4_tensor *v_new, const kv4_tensor *k_packed,
                                    const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                                    const kv4_tensor *v_scales, const kv4_tensor *out,
                                    int group_size, int tie_mode, int is_causal, float sm_scale,
                                    void *workspace, size_t workspace_bytes,
                                    const kv4_attn_opts *opts, void *stream) {
  const AppendJob app{k_new, v_new, tie_mode};
  return run_attention(q, k_packed, k_scales, v_packed, v_scales, out, nullptr, OUT_FINAL, 0, 0,
                       group_size, is_causal, sm_scale, workspace, workspace_bytes, opts,
                       static_cast<cudaStream_t>(stream), &app);
}

extern "C" int kv4_attention_paged(const kv4_tensor *q, const kv4_tensor *k_pages,
                                   const kv4_tensor *k_scale_pages, const kv4_tensor *v_pages,
                                   const kv4_tensor *v_scale_pages, const int32_t *block_table,
                                   int64_t block_table_stride, int64_t max_blocks,
                                   const int32_t *seq_lens, int64_t max_seq_len,
                                   const kv4_tensor *out, int group_size, int is_causal,
                                   float sm_scale, void *workspace, size_t workspace_bytes,
                                   const kv4_attn_opts *opts, void *stream) {
  const PagedJob pj{block_table, block_table_stride, max_blocks, seq_lens, max_seq_len};
  return run_attention(q, k_pages, k_scale_pages, v_pages, v_scale_pages, out, nullptr, OUT_FINAL,
                       0, 0, group_size, is_causal, sm_scale, workspace, workspace_bytes, opts,
                       static_cast<cudaStream_t>(stream), nullptr, &pj);
}

extern "C" int kv4_attention_paged_plan(const kv4_tensor *q, const kv4_tensor *k_pages,
                                        const kv4_tensor *k_scale_pages,
                                        const kv4_tensor *v_pages,
                                        const kv4_tensor *v_scale_pages, int64_t max_blocks,
                                        int64_t max_seq_len, int group_size,
                                        const kv4_attn_opts *opts, kv4_attn_plan *plan) {
  if (!plan) return KV4_ERR_INVALID;
  static const int32_t dummy = 0;
  const PagedJob pj{&dummy, max_blocks, max_blocks, &dummy, max_seq_len};
  Shape S;
  int rc = validate_paged(q, k_pages, k_scale_pages, v_pages, v_scale_pages, group_size, pj, S);
  if (rc) return rc;
  Plan pl;
  make_plan(q, k_pages, k_scale_pages, v_pages, v_scale_pages, S, opts, pl);
  if (pl.path != 1) return KV4_ERR_UNSUPPORTED;
  paged_plan(pl, static_cast<int>(k_pages->shape[2]));
  plan->path = pl.path;
  plan->ctas = pl.ctas;
  plan->tiles_per_cta = pl.L;
  plan->units = pl.units;
  plan->max_parts = pl.maxp;
  plan->kernels = 1;
  plan->workspace_bytes = static_cast<int64_t>(pl.ws_bytes);
  return KV4_OK;
}

extern "C" int kv4_attention_partial(const kv4_tensor *q, const kv4_tensor *k_packed,
                                     const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                                     const kv4_tensor *v_scales, const kv4_tensor *part_o,
                                     const kv4_tensor *part_lse, int64_t k_offset,
                                     int64_t sk_total, int group_size, int is_causal,
                                     float sm_scale, void *workspace, size_t workspace_bytes,
                                     const kv4_attn_opts *opts, void *stream) {
  if (k_offset < 0 || sk_total < k_offset + (k_packed ? k_packed->shape[2] : 0))
    return KV4_ERR_INVALID;
  return run_attention(q, k_packed, k_scales, v_packed, v_scales, part_o, part_lse, OUT_PARTIAL,
                       k_offset, sk_total, group_size, is_causal, sm_scale, workspace,
                       workspace_bytes, opts, static_cast<cudaStream_t>(stream));
}

extern "C" int kv4_attention_plan(const kv4_tensor *q, const kv4_tensor *k_packed,
                                  const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                                  const kv4_tensor *v_scales, const kv4_tensor *out,
                                  int group_size, int is_causal, const kv4_attn_opts *opts,
                                  kv4_attn_plan *plan) {
  (void)out;
  (void)is_causal;
  if (!plan) return KV4_ERR_INVALID;
  Shape S;
  int rc = validate(q, k_packed, k_scales, v_packed, v_scales, group_size, S);
  if (rc) return rc;
  Plan pl;
  make_plan(q, k_packed, k_scales, v_packed, v_scales, S, opts, pl);
  plan->path = pl.path;
  plan->ctas = pl.ctas;
  plan->tiles_per_cta = pl.L;
  plan->units = pl.units;
  plan->max_parts = pl.maxp;
  plan->kernels = 1;
  plan->workspace_bytes = static_cast<int64_t>(pl.ws_bytes);
  return KV4_OK;
}

extern "C" int kv4_lse_combine(const float *parts_o, const float *parts_lse, int64_t n_parts,
                               const kv4_tensor *out, void *stream) {
  if (!parts_o || !parts_lse || !out || n_parts <= 0) return KV4_ERR_INVALID;
  if (!is_float(out->dtype)) return KV4_ERR_DTYPE;
  const int64_t rows = out->shape[0] * out->shape[1] * out->shape[2];
  if (rows == 0 || out->shape[3] == 0) return KV4_OK;
  if (rows > 0x7fffffff) return KV4_ERR_UNSUPPORTED;
  LseParams P{};
  P.po = parts_o;
  P.pl = parts_lse;
  P.nparts = n_parts;
  P.rows = rows;
  P.d = static_cast<int>(out->shape[3]);
  P.out = out->data;
  for (int i = 0; i < 4; ++i) P.os[i] = out->stride[i];
  P.out_dtype = out->dtype;
  P.n1 = out->shape[1];
  P.n2 = out->shape[2];
  kv4_lse_merge<<<static_cast<unsigned>(rows), 128, 0, static_cast<cudaStream_t>(stream)>>>(P);
  return cuda_status(cudaGetLastError());
}

namespace kv4 {
int prefill_take_device_error(int *v);  // prefill.cu
}

extern "C" int kv4_device_error(void *stream, int *flag_out) {
  if (!flag_out) return KV4_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = cuda_status(cudaStreamSynchronize(st));
  if (rc) return rc;
  int v = 0, zero = 0;
  rc = cuda_status(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  if (rc) return rc;
  rc = cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  if (rc) return rc;
  int pv = 0;
  rc = prefill_take_device_error(&pv);
  *flag_out = v | pv;
  return rc;
}

// ===========================================================================
// Allocation-free variant of kv4_attention
// ===========================================================================
// Some callers cannot allocate device memory when they call us: code running
// inside a memory-pool-less runtime or an embedding host whose allocator is
// not reachable from this call site, or a step that must not touch the
// device allocator while it is recording or serving.  For them,
// kv4_attention_noalloc uses a fixed scratch area compiled into this
// library instead of a caller-provided workspace.  Every GPU that loads the
// library holds this array until the process exits.
namespace kv4 {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;   // 4 MiB in total
constexpr size_t kNoAllocCounterBytes = size_t(64) << 10;  // tail: up to 16384 work units
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The array's name is only a host-side stand-in in host code; the device
// address is looked up once per device, with that device current.
static void *noalloc_scratch_ptr(int dev, int *status) {
  static std::mutex mu;
  static void *ptrs[64] = {};
  if (dev < 0 || dev >= 64) {
    *status = KV4_ERR_UNSUPPORTED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *status = cuda_status(e);
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *status = KV4_OK;
  return ptrs[dev];
}

}  // namespace kv4

extern "C" int kv4_attention_noalloc(const kv4_tensor *q, const kv4_tensor *k_packed,
                                     const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                                     const kv4_tensor *v_scales, const kv4_tensor *out,
                                     int group_size, int is_causal, float sm_scale,
                                     void *stream) {
  kv4_attn_plan plan;
  int rc = kv4_attention_plan(q, k_packed, k_scales, v_packed, v_scales, out, group_size,
                              is_causal, nullptr, &plan);
  if (rc) return rc;
  if (plan.workspace_bytes == 0)  // nothing to scratch: identical to kv4_attention
    return kv4_attention(q, k_packed, k_scales, v_packed, v_scales, out, group_size, is_causal,
                         sm_scale, nullptr, 0, nullptr, stream);
  const size_t counters = counter_bytes_of(plan.units, plan.max_parts);
  const size_t data = static_cast<size_t>(plan.workspace_bytes) - ((counters + 15) / 16 * 16);
  if (counters > kNoAllocCounterBytes || data > kNoAllocScratchBytes - kNoAllocCounterBytes)
    return KV4_ERR_SCRATCH_LIMIT;
  int dev = 0;
  rc = cuda_status(cudaGetDevice(&dev));
  if (rc) return rc;
  // The scratch address below belongs to the current device; a stream of
  // another device would make the kernel write to the wrong GPU's array.
  if (stream != nullptr) {
    int sdev = -1;
    rc = cuda_status(cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev));
    if (rc) return rc;
    if (sdev != dev) return KV4_ERR_INVALID;
  }
  void *scratch = noalloc_scratch_ptr(dev, &rc);
  if (rc) return rc;
  // The counters (the last `counters` bytes of the area) must start at zero;
  // clear them on this stream in case an earlier call did not complete.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = cuda_status(cudaMemsetAsync(static_cast<char *>(scratch) + kNoAllocScratchBytes - counters,
                                   0, counters, st));
  if (rc) return rc;
  return kv4_attention(q, k_packed, k_scales, v_packed, v_scales, out, group_size, is_causal,
                       sm_scale, scratch, kNoAllocScratchBytes, nullptr, stream);
}

// ===========================================================================
// Sequence-shard exchange over peer memory (one kernel: push + merge)
// ===========================================================================
// Every rank holds a buffer of kv4_lse_exchange_bytes() bytes at the same
// size on every GPU (e.g. symmetric memory), and a device array with the
// addresses of all ranks' buffers as seen from this GPU.  Each value travels
// with the call's epoch in one 8-byte store ({value bits, epoch}, written
// and read as single 8-byte accesses), so a reader knows a value has
// landed when its epoch matches: no fences and no separate flags.  Layout:
//   uint2 [2][world][rows][d + 1]   (parity of the call, source rank, row,
//                                    d values then the lse)
// Call k uses parity k & 1: a rank can only be one call ahead of a peer
// (its call k + 1 cannot end before the peer's call k values arrived, and
// the peer pushes call k + 1 only after it read call k), so two parities keep
// a slot from being overwritten while it is read.
namespace kv4 {

constexpr int kXBlocks = 64;                  // blocks of the exchange kernel (max)
constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // 2 s per call

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct XchgParams {
  const float *po;
  const float *pl;
  int64_t rows;
  int d;
  void *const *peers;  // device array [world]
  int world, rank;
  uint32_t *state;  // this rank's [calls so far, blocks done] (device, zeroed once)
  void *out;
  int64_t os[4];
  int out_dtype;
  int64_t n1, n2;
};

__global__ void __launch_bounds__(256) kv4_lse_exchange_kernel(const XchgParams P) {
  const int nb = gridDim.x, bid = blockIdx.x, tid = threadIdx.x;
  // this call's epoch: calls so far + 1 (the last block of the call advances
  // the count, so the next call, ordered after this one, sees it)
  const uint32_t epoch = __ldcv(P.state) + 1u;
  const int par = static_cast<int>(epoch & 1u);
  const int64_t r0 = P.rows * bid / nb, r1 = P.rows * (bid + 1) / nb;
  const int64_t rw = P.d + 1;                 // words per row
  const int64_t slot = P.rows * rw;           // words per (parity, source)
  auto at = [&](void *base, int src, int64_t r, int w) {
    return reinterpret_cast<uint2 *>(base) + (static_cast<int64_t>(par) * P.world + src) * slot +
           r * rw + w;
  };
  // 1. push this rank's rows [r0, r1) into slot `rank` of every rank's buffer
  for (int q = 0; q < P.world; ++q) {
    void *dst = P.peers[q];
    for (int64_t i = tid; i < (r1 - r0) * rw; i += blockDim.x) {
      const int64_t r = r0 + i / rw;
      const int w = static_cast<int>(i - (r - r0) * rw);
      const float v = w < P.d ? P.po[r * P.d + w] : P.pl[r];
      asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(at(dst, P.rank, r, w)),
                   "r"(__float_as_uint(v)), "r"(epoch)
                   : "memory");
    }
  }
  // 2. read every rank's rows [r0, r1) from this rank's buffer once they have
  // landed (bounded wait), and merge them
  void *mine = P.peers[P.rank];
  const unsigned long long t0 = globaltimer_ns();
  bool late = false;
  auto fetch = [&](int src, int64_t r, int w) -> float {
    uint32_t v, e;
    while (true) {
      asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];"
                   : "=r"(v), "=r"(e)
                   : "l"(at(mine, src, r, w))
                   : "memory");
      if (e == epoch || late) break;
      if (globaltimer_ns() - t0 > kPeerWaitNs) {
        late = true;
        atomicOr(&g_device_error, DEV_ERR_PEER_TIMEOUT);
        break;
      }
    }
    return __uint_as_float(v);
  };
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t i2 = r % P.n2, i01 = r / P.n2, i1 = i01 % P.n1, i0 = i01 / P.n1;
    for (int dd = tid; dd < P.d; dd += blockDim.x) {
      float M = kNegInf;
      for (int k = 0; k < P.world; ++k) M = fmaxf(M, fetch(k, r, P.d));
      float W = 0.0f, o = 0.0f;
      for (int k = 0; k < P.world; ++k) {
        const float l = fetch(k, r, P.d), v = fetch(k, r, dd);
        const float w = (M == kNegInf) ? 0.0f : expf(l - M);
        W += w;
        o += w * v;
      }
      store_from_f32(P.out, P.out_dtype,
                     i0 * P.os[0] + i1 * P.os[1] + i2 * P.os[2] + dd * P.os[3],
                     W > 0.0f ? o / W : 0.0f);
    }
  }
  __syncthreads();
  if (tid == 0) {  // every block has read the epoch before the last one advances it
    if (atomicAdd(&P.state[1], 1u) == static_cast<uint32_t>(nb) - 1u) {
      P.state[1] = 0u;
      __threadfence();
      atomicExch(&P.state[0], epoch);
    }
  }
}

}  // namespace kv4

extern "C" int64_t kv4_lse_exchange_bytes(int64_t rows, int d, int world) {
  if (rows <= 0 || d <= 0 || world <= 0 || world > 64) return 0;
  return 2 * static_cast<int64_t>(world) * rows * (d + 1) * 8;
}

extern "C" int kv4_lse_exchange(const float *part_o, const float *part_lse, int64_t rows,
                                int d, void *const *peer_bufs, int world, int rank,
                                uint32_t *state, const kv4_tensor *out, void *stream) {
  if (!part_o || !part_lse || !peer_bufs || !out || !state || world <= 0 || world > 64 ||
      rank < 0 || rank >= world || rows <= 0 || d <= 0)
    return KV4_ERR_INVALID;
  if (!is_float(out->dtype)) return KV4_ERR_DTYPE;
  if (out->shape[0] * out->shape[1] * out->shape[2] != rows || out->shape[3] != d)
    return KV4_ERR_SHAPE;
  XchgParams P{};
  P.po = part_o;
  P.pl = part_lse;
  P.rows = rows;
  P.d = d;
  P.peers = peer_bufs;
  P.world = world;
  P.rank = rank;
  P.state = state;
  P.out = out->data;
  for (int i = 0; i < 4; ++i) P.os[i] = out->stride[i];
  P.out_dtype = out->dtype;
  P.n1 = out->shape[1];
  P.n2 = out->shape[2];
  const int nb = static_cast<int>(std::min<int64_t>(kXBlocks, rows));
  kv4_lse_exchange_kernel<<<nb, 256, 0, static_cast<cudaStream_t>(stream)>>>(P);
  return cuda_status(cudaGetLastError());
}
