// Fused causal prefill over the packed INT4 cache on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// Semantics follow kernels/llama3/attention_quant.py:24-152 of the reference
// for query blocks (sq > 1): out[b, h, i] = softmax_j(q[b,h,i] . K[b,h/R,j] *
// sm_scale) . V[b,h/R,j], K/V = (code - 8) * scale, bottom-right causal
// (keys j <= sk - sq + i visible) or none.
//
// One CTA = 4 warps = 128 rows = (q head of the GQA group, query) pairs of
// one (batch, KV head); it walks the key tiles of 128 tokens:
//   * a bulk copy streams the packed K/V rows of the next tile into one
//     staging buffer (mbarrier); scales are read per row from global memory;
//   * each thread dequantizes one key row of K and of V into f16 tiles in
//     shared memory, in the canonical 128-byte-swizzled layout of the MMA
//     descriptors (the 8 dims of a packed word are stored in the order
//     0,4,1,5,2,6,3,7 -- the same permutation is applied to q, and undone on
//     the output columns);
//   * one thread issues S = Q K^T (M 128, N 128, K 128) into tensor memory;
//   * every thread reads its row of S, runs the online softmax (lazy
//     rescale), rescales its row of O in tensor memory when the running max
//     moved far, and writes P (f16 pairs) over the first 64 columns of S;
//   * one thread issues O += P V (P from tensor memory, V an MN-major
//     shared-memory operand).
// Tensor memory: 256 columns (S / P: 0..127, O: 128..255).  Shared memory
// 112 KB, so two CTAs share an SM and one's softmax and dequantization
// overlap the other's MMAs.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace kv4 {

namespace pf {

constexpr int ROWS = 128;   // MMA M
constexpr int KT = 128;     // keys per tile (MMA N of S, K of P.V)
constexpr int D = 128;      // head dim (MMA K of S, N of P.V)
constexpr int P_BYTES = D / 2;
constexpr int PANEL = ROWS * 128;  // one 64-element-wide panel of a 16-bit tile (bytes)
constexpr int TILE = 2 * PANEL;    // a 128 x 128 16-bit tile: 32 KB
constexpr uint32_t TMEM_COLS = 256;

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) |
         (static_cast<uint64_t>(lbo >> 4) << 16) | (static_cast<uint64_t>(sbo >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: f32 accumulate, f16 A and B, M = 128, N = 128,
// A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1).
__host__ __device__ constexpr uint32_t instr_desc(uint32_t b_mn) {
  return (1u << 4) | (b_mn << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u)
      : "memory");
}

// A from tensor memory (M rows on the lanes, 16-bit K pairs per column)
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
      : "memory");
}

// 32 consecutive fp32 columns of this thread's row (lane) of tensor memory
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(addr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t addr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(addr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32u(uint32_t addr, const uint32_t (&v)[32]) {
  float f[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
  tmem_st32(addr, f);
}

// byte offset of 16-byte chunk c (0..15) of row r in a swizzled 128 x 128 16-bit tile
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * PANEL + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

}  // namespace pf
}  // namespace kv4

namespace kv4 {
namespace pf {

// device error word of this kernel: DEV_ERR_MBAR_TIMEOUT (a bounded mbarrier
// wait expired), DEV_ERR_F16_RANGE (a scale above 65504 / 8: K/V values
// outside the f16 range of the operands, the output is not valid)
__device__ int g_prefill_error = 0;

struct Params {
  const __nv_bfloat16 *q;
  int64_t qs[3];  // batch, head, query strides (elements; dims contiguous)
  const uint8_t *kp, *vp;
  int64_t kps[2], vps[2];  // batch, head strides (bytes; tokens of 64 bytes contiguous)
  const __nv_bfloat16 *ks, *vs;
  int64_t kss[2], vss[2];  // batch, head strides (elements; tokens of D/G contiguous)
  __nv_bfloat16 *out;
  int64_t os[3];
  int Hkv, R, QB, sq, sk, causal;
  uint32_t wait_limit;
  float scale_log2;
};

constexpr int STAGE = KT * 2 * P_BYTES;  // packed K rows then packed V rows of one tile
constexpr int SMEM_BYTES = 3 * TILE + STAGE + 64;  // Q, K, V tiles; the stage; barriers

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// f16 pairs (1024 + code) of the 8 nibbles of x, in the dim pairs (0,4), (1,5), (2,6), (3,7)
__device__ __forceinline__ uint32_t nib_pair(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(0x000F000Fu), "r"(0x64006400u));
  return r;
}

// largest scale whose products (code - 8) * scale stay finite in f16
constexpr float kMaxF16Scale = 65504.0f / 8.0f;

// NG scales (bf16) of one token row as f16 (exact: 8 significant bits fit in
// 11), each duplicated into both halves of a word; `big` is set when a scale
// would overflow the f16 products
template <int NG>
__device__ __forceinline__ void load_scales(const __nv_bfloat16 *p, bool valid, uint32_t (&s)[NG],
                                            bool &big) {
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const float f = valid ? __bfloat162float(__ldg(p + g)) : 0.0f;
    big |= fabsf(f) > kMaxF16Scale;
    const uint32_t h = __half_as_ushort(__float2half_rn(f));
    s[g] = h | (h << 16);
  }
}

// Dequantize one packed row (64 bytes at smem address `src`) into row r of a
// swizzled f16 tile: value = (code - 8) * scale, with (1024 + code) - 1032
// exact and the product exact as well (a 4-bit code times an 8-bit scale
// significand fits the 11-bit f16 significand) while it is a normal f16.
template <int G>
__device__ __forceinline__ void dequant_row(uint32_t tile, int r, uint32_t src,
                                            const uint32_t (&s)[D / G]) {
  const uint32_t bias = 0x64086408u;  // f16x2 (1032, 1032)
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w[4];
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "r"(src + 16 * c));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t sc = s[(32 * c + 8 * k) / G];
      uint32_t v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = hmul2(hsub2(nib_pair(w[k] >> (4 * e)), bias), sc);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(tile + tile_off(r, 4 * c + k)),
                   "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
                   : "memory");
    }
  }
}

__device__ __forceinline__ void zero_row(uint32_t tile, int r) {
#pragma unroll
  for (int c = 0; c < 16; ++c)
    asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(tile + tile_off(r, c)), "r"(0u)
                 : "memory");
}

}  // namespace pf
}  // namespace kv4

namespace kv4 {
namespace pf {

template <int G>
__global__ void __launch_bounds__(128, 2) kv4_prefill_tc(const Params P) {
  constexpr int NG = D / G;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  const uint32_t sQ = base, sK = sQ + TILE, sV = sK + TILE, sStage = sV + TILE;
  const uint32_t bar_full = sStage + STAGE, bar_s = bar_full + 8, bar_o = bar_full + 16;
  const uint32_t slot = bar_full + 24;  // tcgen05.alloc writes the TMEM address here
  if (base & 1023u) {  // the swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicOr(&g_prefill_error, DEV_ERR_MBAR_TIMEOUT);
    return;
  }

  const int tid = threadIdx.x, warp = tid >> 5;
  const int bkv = blockIdx.y, b = bkv / P.Hkv, kvh = bkv - b * P.Hkv;
  const int q0 = blockIdx.x * P.QB;
  const int hl = tid / P.QB, qi = q0 + (tid - hl * P.QB);
  const bool row_ok = qi < P.sq;
  const int h = kvh * P.R + hl;
  // keys [0, lim) are visible to this row (bottom-right causal alignment)
  int lim = P.causal ? min(P.sk, P.sk - P.sq + qi + 1) : P.sk;
  if (!row_ok) lim = 0;
  const int last_q = min(q0 + P.QB, P.sq) - 1;
  const int maxlim = P.causal ? min(P.sk, P.sk - P.sq + last_q + 1) : P.sk;
  const int nkt = maxlim > 0 ? (maxlim + KT - 1) / KT : 0;

  if (tid == 0) {
    mbar_init(bar_full, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  uint32_t tmem;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(tmem) : "r"(slot) : "memory");
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  // S (fp32) in columns 0..127; P (f16 pairs) over columns 0..63 once S is
  // read; O (fp32) in columns 128..255
  const uint32_t tS = tmem + lane_base, tO = tmem + 128 + lane_base;

  const uint8_t *kp = P.kp + b * P.kps[0] + kvh * P.kps[1];
  const uint8_t *vp = P.vp + b * P.vps[0] + kvh * P.vps[1];
  const __nv_bfloat16 *ks = P.ks + b * P.kss[0] + kvh * P.kss[1];
  const __nv_bfloat16 *vs = P.vs + b * P.vss[0] + kvh * P.vss[1];

  auto issue = [&](int kt) {  // thread 0: packed rows of tile kt -> the stage
    const int t0 = kt * KT, rem = min(KT, P.sk - t0);
    const uint32_t pb = static_cast<uint32_t>(rem * P_BYTES);
    mbar_arrive_expect_tx(bar_full, 2 * pb);
    bulk_load(sStage, kp + static_cast<int64_t>(t0) * P_BYTES, pb, bar_full);
    bulk_load(sStage + KT * P_BYTES, vp + static_cast<int64_t>(t0) * P_BYTES, pb, bar_full);
  };
  if (tid == 0 && nkt > 0) issue(0);

  // this row of q, times sm_scale * log2(e), as f16 -> Q tile (scores come out
  // of the MMA in the log2 domain); dims of each 8-group in the order
  // 0,4,1,5,2,6,3,7
  {
    const __nv_bfloat16 *qr = P.q + b * P.qs[0] + h * P.qs[1] + static_cast<int64_t>(qi) * P.qs[2];
#pragma unroll
    for (int cq = 0; cq < 16; ++cq) {
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (row_ok) w = __ldg(reinterpret_cast<const uint4 *>(qr + 8 * cq));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      float f[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(ws[e] << 16) * P.scale_log2;
        f[2 * e + 1] = __uint_as_float(ws[e] & 0xFFFF0000u) * P.scale_log2;
      }
      const uint32_t a0 = pack_f16x2(f[0], f[4]), a1 = pack_f16x2(f[1], f[5]);
      const uint32_t a2 = pack_f16x2(f[2], f[6]), a3 = pack_f16x2(f[3], f[7]);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sQ + tile_off(tid, cq)),
                   "r"(a0), "r"(a1), "r"(a2), "r"(a3)
                   : "memory");
    }
  }

  const uint32_t id_s = instr_desc(0), id_o = instr_desc(1);
  float m_run = -INFINITY, l_run = 0.0f;
  bool failed = false, big = false;
  for (int kt = 0; kt < nkt; ++kt) {
    const int t0 = kt * KT, rem = min(KT, P.sk - t0);
    const bool key_ok = tid < rem;  // this thread dequantizes key row t0 + tid
    uint32_t sck[NG], scv[NG];
    load_scales<NG>(ks + static_cast<int64_t>(t0 + tid) * NG, key_ok, sck, big);
    load_scales<NG>(vs + static_cast<int64_t>(t0 + tid) * NG, key_ok, scv, big);
    if (!mbar_wait_bounded(bar_full, static_cast<uint32_t>(kt) & 1u, P.wait_limit)) failed = true;
    if (key_ok) {
      dequant_row<G>(sK, tid, sStage + tid * P_BYTES, sck);
      dequant_row<G>(sV, tid, sStage + KT * P_BYTES + tid * P_BYTES, scv);
    } else {
      zero_row(sK, tid);
      zero_row(sV, tid);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();  // stage consumed; Q (first tile), K and V tiles written
    tc_fence_after();
    if (tid == 0) {
      if (kt + 1 < nkt) issue(kt + 1);
#pragma unroll
      for (int j = 0; j < D / 16; ++j) {  // S = Q K^T, 16 dims per MMA
        const uint32_t off = (j >> 2) * PANEL + (j & 3) * 32;
        mma_f16(tmem, smem_desc(sQ + off, 16, 1024), smem_desc(sK + off, 16, 1024), id_s,
                j > 0 ? 1u : 0u);
      }
      mma_commit(bar_s);
    }
    if (!mbar_wait_bounded(bar_s, static_cast<uint32_t>(kt) & 1u, P.wait_limit)) failed = true;
    tc_fence_after();

    // online softmax of this thread's row (log2 domain)
    float sv[4][32];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, sv[c]);
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float x = (t0 + 32 * c + e < lim) ? sv[c][e] : -INFINITY;
        sv[c][e] = x;
        mx = fmaxf(mx, x);
      }
    // lazy rescale: the running max moves only when a score exceeds it by
    // more than 8, so unnormalised probabilities stay below 2^8
    const bool up = mx > m_run + 8.0f;
    float alpha = 1.0f;
    if (up) {
      alpha = m_run == -INFINITY ? 0.0f : exp2f(m_run - mx);
      l_run *= alpha;
      m_run = mx;
    }
    if (kt > 0 && __any_sync(0xffffffffu, up)) {  // warp-uniform: TMEM access is collective
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tO + 32 * c, ov);
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] *= alpha;
        tmem_st32(tO + 32 * c, ov);
      }
    }
    const float me = m_run == -INFINITY ? 0.0f : m_run;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {  // P as f16 pairs over columns 32 h2 .. 32 h2 + 31
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float p0 = exp2f(sv[2 * h2 + (e >> 4)][2 * (e & 15)] - me);
        const float p1 = exp2f(sv[2 * h2 + (e >> 4)][2 * (e & 15) + 1] - me);
        l_run += p0 + p1;
        pk[e] = pack_f16x2(p0, p1);
      }
      tmem_st32u(tS + 32 * h2, pk);
    }
    tc_fence_before();
    __syncthreads();  // P written, O rescaled
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int j = 0; j < KT / 16; ++j)  // O += P V, 16 keys (8 columns of P) per MMA
        mma_f16_ts(tmem + 128, tmem + 8 * j, smem_desc(sV + j * 16 * 128, PANEL, 1024), id_o,
                   (kt > 0 || j > 0) ? 1u : 0u);
      mma_commit(bar_o);
    }
    if (!mbar_wait_bounded(bar_o, static_cast<uint32_t>(kt) & 1u, P.wait_limit)) failed = true;
    tc_fence_after();
  }
  if (failed) atomicOr(&g_prefill_error, DEV_ERR_MBAR_TIMEOUT);
  if (big) atomicOr(&g_prefill_error, DEV_ERR_F16_RANGE);

  // epilogue: O / l -> out; every lane takes part in the collective TMEM loads
  {
    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
    __nv_bfloat16 *orow = P.out + b * P.os[0] + h * P.os[1] + static_cast<int64_t>(qi) * P.os[2];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float ov[32];
      if (nkt > 0) {
        tmem_ld32(tO + 32 * c, ov);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = 0.0f;
      }
      if (row_ok) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {  // columns 8a.. hold dims 8a + (0,4,1,5,2,6,3,7)
          const float *o8 = ov + 8 * a;
          uint4 w;
          w.x = pack_bf16x2(o8[0] * inv, o8[2] * inv);
          w.y = pack_bf16x2(o8[4] * inv, o8[6] * inv);
          w.z = pack_bf16x2(o8[1] * inv, o8[3] * inv);
          w.w = pack_bf16x2(o8[5] * inv, o8[7] * inv);
          *reinterpret_cast<uint4 *>(orow + 32 * c + 8 * a) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
}

}  // namespace pf

// read-and-clear of this file's device error word (folded into kv4_device_error)
int prefill_take_device_error(int *v) {
  int zero = 0;
  int rc = cuda_status(cudaMemcpyFromSymbol(v, pf::g_prefill_error, sizeof(int)));
  if (rc) return rc;
  return cuda_status(cudaMemcpyToSymbol(pf::g_prefill_error, &zero, sizeof(int)));
}

}  // namespace kv4

// ===========================================================================
// host side
// ===========================================================================
namespace kv4 {
namespace {

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int G>
int launch_prefill(const pf::Params &P, dim3 grid, cudaStream_t st) {
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev]) {
    const int rc = cuda_status(cudaFuncSetAttribute(
        pf::kv4_prefill_tc<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM_BYTES));
    if (rc) return rc;
    configured[dev] = true;
  }
  pf::kv4_prefill_tc<G><<<grid, 128, pf::SMEM_BYTES, st>>>(P);
  return cuda_status(cudaGetLastError());
}

}  // namespace
}  // namespace kv4

extern "C" int kv4_prefill_attention(const kv4_tensor *q, const kv4_tensor *k_packed,
                                     const kv4_tensor *k_scales, const kv4_tensor *v_packed,
                                     const kv4_tensor *v_scales, const kv4_tensor *out,
                                     int group_size, int is_causal, float sm_scale,
                                     void *stream) {
  using namespace kv4;
  const kv4_tensor *kp = k_packed, *ks = k_scales, *vp = v_packed, *vs = v_scales;
  if (!q || !kp || !ks || !vp || !vs || !out) return KV4_ERR_INVALID;
  if (group_size <= 0) return KV4_ERR_INVALID;
  if (q->dtype != KV4_BF16 || out->dtype != KV4_BF16 || ks->dtype != KV4_BF16 ||
      vs->dtype != KV4_BF16 || kp->dtype != KV4_U8 || vp->dtype != KV4_U8)
    return KV4_ERR_DTYPE;
  const int64_t B = q->shape[0], Hq = q->shape[1], sq = q->shape[2], d = q->shape[3];
  const int64_t Hkv = kp->shape[1], sk = kp->shape[2];
  for (int i = 0; i < 4; ++i) {
    if (out->shape[i] != q->shape[i]) return KV4_ERR_SHAPE;
    if (kp->shape[i] != vp->shape[i] || ks->shape[i] != vs->shape[i]) return KV4_ERR_SHAPE;
    if (i < 3 && kp->shape[i] != ks->shape[i]) return KV4_ERR_SHAPE;
  }
  if (kp->shape[0] != B) return KV4_ERR_SHAPE;
  if (Hkv <= 0 || Hq <= 0 || Hq % Hkv) return KV4_ERR_INVALID;
  const int64_t R = Hq / Hkv;
  const int G = group_size;
  if (d != pf::D || !(G == 16 || G == 32 || G == 64 || G == 128)) return KV4_ERR_UNSUPPORTED;
  if (kp->shape[3] != pf::P_BYTES || ks->shape[3] != pf::D / G) return KV4_ERR_UNSUPPORTED;
  if (pf::ROWS % R) return KV4_ERR_UNSUPPORTED;
  if (sq <= 0 || sk <= 0 || sk >= (int64_t(1) << 30) || sq >= (int64_t(1) << 30))
    return KV4_ERR_UNSUPPORTED;
  if (is_causal && sq > sk) return KV4_ERR_UNSUPPORTED;  // rows with no visible key
  if (B * Hkv > 65535) return KV4_ERR_UNSUPPORTED;
  for (const kv4_tensor *t : {q, out}) {
    if (!al16(t->data) || t->stride[3] != 1) return KV4_ERR_LAYOUT;
    for (int i = 0; i < 3; ++i)
      if (t->shape[i] > 1 && (t->stride[i] * 2) % 16) return KV4_ERR_LAYOUT;
  }
  for (const kv4_tensor *t : {kp, vp}) {
    if (!al16(t->data) || t->stride[3] != 1 || t->stride[2] != pf::P_BYTES) return KV4_ERR_LAYOUT;
    for (int i = 0; i < 2; ++i)
      if (t->shape[i] > 1 && t->stride[i] % 16) return KV4_ERR_LAYOUT;
  }
  for (const kv4_tensor *t : {ks, vs}) {
    if ((reinterpret_cast<uintptr_t>(t->data) & 1u) || t->stride[3] != 1 ||
        t->stride[2] != pf::D / G)
      return KV4_ERR_LAYOUT;
  }

  pf::Params P{};
  P.q = static_cast<const __nv_bfloat16 *>(q->data);
  P.out = static_cast<__nv_bfloat16 *>(out->data);
  P.kp = static_cast<const uint8_t *>(kp->data);
  P.vp = static_cast<const uint8_t *>(vp->data);
  P.ks = static_cast<const __nv_bfloat16 *>(ks->data);
  P.vs = static_cast<const __nv_bfloat16 *>(vs->data);
  for (int i = 0; i < 3; ++i) {
    P.qs[i] = q->stride[i];
    P.os[i] = out->stride[i];
  }
  for (int i = 0; i < 2; ++i) {
    P.kps[i] = kp->stride[i];
    P.vps[i] = vp->stride[i];
    P.kss[i] = ks->stride[i];
    P.vss[i] = vs->stride[i];
  }
  P.Hkv = static_cast<int>(Hkv);
  P.R = static_cast<int>(R);
  P.QB = static_cast<int>(pf::ROWS / R);
  P.sq = static_cast<int>(sq);
  P.sk = static_cast<int>(sk);
  P.causal = is_causal ? 1 : 0;
  P.wait_limit = 1u << 14;
  const float sc = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(static_cast<float>(d));
  P.scale_log2 = sc * 1.4426950408889634f;
  const dim3 grid(static_cast<unsigned>((sq + P.QB - 1) / P.QB), static_cast<unsigned>(B * Hkv));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 16: return launch_prefill<16>(P, grid, st);
    case 32: return launch_prefill<32>(P, grid, st);
    case 64: return launch_prefill<64>(P, grid, st);
    default: return launch_prefill<128>(P, grid, st);
  }
}
