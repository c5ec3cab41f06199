// INT4 group quantize (incl. fused K+V quantize-on-append) and dequantize.
//
// Arithmetic follows the reference quantizer exactly
// (kernels/llama3/quantize.py:47-75 Triton kernel, :126-148 torch path):
//   scale = max|x| / 7 in fp32 (1.0 for an all-zero group)
//   q     = x / scale (un-rounded fp32 scale)
//   both divisions as the reference path does them: div.full.f32 like the
//   Triton kernel (default), or IEEE like the torch path
//   code  = clamp(round(q), -8, 7) + 8, round = half-away (Triton) or
//           half-even (torch), packed low nibble = even column
//   the stored scale is the fp32 scale rounded (RN) to the scales dtype.
// One thread owns one group: it makes two passes over the group's elements
// (max, then codes), the second served from L1; loads are 16-byte vectors
// whenever the group is contiguous and aligned.
#include "common.cuh"

namespace kv4 {

struct QJob {
  const void *x;
  int64_t xs[4];  // x strides (elements)
  uint8_t *p;
  int64_t ps[4];  // packed strides (bytes)
  void *s;
  int64_t ss[4];  // scales strides (elements)
  int64_t t_off;  // row offset applied to dim 2 of packed/scales
  // paged destination (slots != nullptr): row (i0, i1, i2) goes to page
  // slots[i0 * n2 + i2] / page, row slots[...] % page of head i1 (negative
  // slots are skipped); dim 0 of packed/scales is then the page
  const int32_t *slots;
  int64_t page, npages;  // slots past the pool are skipped as well
};

struct QParams {
  QJob job[2];
  int njobs;
  int64_t n1, n2;   // x dims 1, 2 (dim 0 implied by rows)
  int64_t rows;     // n0*n1*n2 per job
  int64_t d;        // elements per row
  int G;            // group size
  int ng;           // groups per row
  int pb;           // packed bytes per group = ceil(G/2)
};

template <typename XT>
__device__ __forceinline__ void load8(const XT *p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float *p, float (&v)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4 *>(p));
  float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename H2, typename XT>
__device__ __forceinline__ void load8_16(const XT *p, float (&v)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
  const XT *h = reinterpret_cast<const XT *>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = to_f32(h[i]);
}
template <>
__device__ __forceinline__ void load8<__half>(const __half *p, float (&v)[8]) {
  load8_16<__half2>(p, v);
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16 *p, float (&v)[8]) {
  load8_16<__nv_bfloat162>(p, v);
}

template <typename XT, typename ST, int TIE>
__global__ void __launch_bounds__(256) quantize_kernel(const QParams P) {
  const int64_t per_job = P.rows * P.ng;
  const int64_t total = per_job * P.njobs;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int jid = idx >= per_job ? 1 : 0;
    const QJob &J = P.job[jid];
    const int64_t rem = idx - jid * per_job;
    const int64_t row = rem / P.ng;
    const int grp = static_cast<int>(rem - row * P.ng);
    const int64_t i2 = row % P.n2;
    const int64_t r01 = row / P.n2;
    const int64_t i1 = r01 % P.n1;
    const int64_t i0 = r01 / P.n1;

    const XT *xrow = static_cast<const XT *>(J.x) + i0 * J.xs[0] + i1 * J.xs[1] + i2 * J.xs[2];
    const int64_t c0 = static_cast<int64_t>(grp) * P.G;
    const int64_t rest = P.d - c0;
    const int nvalid = static_cast<int>(rest < P.G ? rest : P.G);  // >= 1
    const XT *xg = xrow + c0 * J.xs[3];
    const bool vec = (J.xs[3] == 1) && (nvalid % 8 == 0) &&
                     ((reinterpret_cast<uintptr_t>(xg) & 15) == 0);

    // pass 1: max |x|
    float mx = 0.0f;
    if (vec) {
      for (int e = 0; e < nvalid; e += 8) {
        float v[8];
        load8<XT>(xg + e, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
      }
    } else {
      for (int e = 0; e < nvalid; ++e) mx = fmaxf(mx, fabsf(to_f32(xg[e * J.xs[3]])));
    }
    const float scale = group_scale<TIE>(mx);

    // destination row: (i0, i1, i2 + t_off), or the paged slot of (i0, i2)
    int64_t d0 = i0, d2 = i2 + J.t_off;
    if (J.slots) {
      const int64_t slot = J.slots[i0 * P.n2 + i2];
      if (slot < 0 || slot >= J.page * J.npages) continue;
      d0 = slot / J.page;
      d2 = slot - d0 * J.page;
    }
    // pass 2: codes, packed two per byte, emitted 4 bytes at a time
    uint8_t *prow = J.p + d0 * J.ps[0] + i1 * J.ps[1] + d2 * J.ps[2];
    uint8_t *pg = prow + static_cast<int64_t>(grp) * P.pb * J.ps[3];
    const bool pvec = (J.ps[3] == 1) && ((reinterpret_cast<uintptr_t>(pg) & 3) == 0) &&
                      (P.pb % 4 == 0);
    if (vec && pvec) {
      for (int e = 0; e < P.G; e += 8) {
        uint32_t w = 0x88888888u;  // padding columns quantize to code 8
        if (e < nvalid) {
          float v[8];
          load8<XT>(xg + e, v);
          w = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) w |= code_of<TIE>(v[i], scale) << (4 * i);
        }
        *reinterpret_cast<uint32_t *>(pg + e / 2) = w;
      }
    } else {
      for (int b = 0; b < P.pb; ++b) {
        const int e0 = 2 * b, e1 = 2 * b + 1;
        uint32_t lo = 8, hi = 8;
        if (e0 < nvalid) lo = code_of<TIE>(to_f32(xg[e0 * J.xs[3]]), scale);
        if (e1 < nvalid) hi = code_of<TIE>(to_f32(xg[e1 * J.xs[3]]), scale);
        if (e1 >= P.G) hi = 0;  // odd group size: the pad nibble is 0
        pg[b * J.ps[3]] = static_cast<uint8_t>(lo | (hi << 4));
      }
    }
    ST *srow = static_cast<ST *>(J.s) + d0 * J.ss[0] + i1 * J.ss[1] + d2 * J.ss[2];
    srow[grp * J.ss[3]] = from_f32<ST>(scale);
  }
}

// ---------------------------------------------------------------------------
struct DQParams {
  const uint8_t *p;
  int64_t ps[4];
  const void *s;
  int64_t ss[4];
  void *o;
  int64_t os[4];
  int64_t n1, n2, rows;
  int d_out;
  int G;
  int slot;  // nibbles per group slot = 2*pw/ng
};

template <typename ST, typename OT>
__global__ void __launch_bounds__(256) dequantize_kernel(const DQParams P) {
  const int64_t total = P.rows * P.d_out;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / P.d_out;
    const int e = static_cast<int>(idx - row * P.d_out);
    const int64_t i2 = row % P.n2;
    const int64_t r01 = row / P.n2;
    const int64_t i1 = r01 % P.n1;
    const int64_t i0 = r01 / P.n1;
    const int grp = e / P.G;
    const int nib = grp * P.slot + (e - grp * P.G);
    const uint8_t byte =
        P.p[i0 * P.ps[0] + i1 * P.ps[1] + i2 * P.ps[2] + (nib >> 1) * P.ps[3]];
    const int code = (nib & 1) ? (byte >> 4) : (byte & 15);
    const float s = to_f32(static_cast<const ST *>(P.s)[i0 * P.ss[0] + i1 * P.ss[1] +
                                                        i2 * P.ss[2] + grp * P.ss[3]]);
    static_cast<OT *>(P.o)[i0 * P.os[0] + i1 * P.os[1] + i2 * P.os[2] + e * P.os[3]] =
        from_f32<OT>(static_cast<float>(code - 8) * s);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static bool is_float_dtype(int dt) { return dt == KV4_F32 || dt == KV4_F16 || dt == KV4_BF16; }

static int grid_for(int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = 148 * 64;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

template <typename XT, typename ST>
static void launch_quant(const QParams &P, int tie, cudaStream_t st) {
  const int threads = 256;
  const int grid = grid_for(P.rows * P.ng * P.njobs, threads);
  if (tie == KV4_TIE_HALF_EVEN)
    quantize_kernel<XT, ST, KV4_TIE_HALF_EVEN><<<grid, threads, 0, st>>>(P);
  else if (tie == KV4_TIE_HALF_AWAY_IEEE)
    quantize_kernel<XT, ST, KV4_TIE_HALF_AWAY_IEEE><<<grid, threads, 0, st>>>(P);
  else
    quantize_kernel<XT, ST, KV4_TIE_HALF_AWAY><<<grid, threads, 0, st>>>(P);
}

template <typename XT>
static void launch_quant_x(const QParams &P, int sdt, int tie, cudaStream_t st) {
  if (sdt == KV4_F32) launch_quant<XT, float>(P, tie, st);
  else if (sdt == KV4_F16) launch_quant<XT, __half>(P, tie, st);
  else launch_quant<XT, __nv_bfloat16>(P, tie, st);
}

static int fill_job(QJob &J, const kv4_tensor *x, const kv4_tensor *p, const kv4_tensor *s,
                    int64_t t_off) {
  J.x = x->data;
  J.p = static_cast<uint8_t *>(p->data);
  J.s = s->data;
  for (int i = 0; i < 4; ++i) {
    J.xs[i] = x->stride[i];
    J.ps[i] = p->stride[i];
    J.ss[i] = s->stride[i];
  }
  J.t_off = t_off;
  return KV4_OK;
}

static int check_quant_args(const kv4_tensor *x, const kv4_tensor *p, const kv4_tensor *s,
                            int64_t t_off, int G, int tie, int64_t &ng, int64_t &pb) {
  if (!x || !p || !s) return KV4_ERR_INVALID;
  if (G <= 0) return KV4_ERR_INVALID;
  if (!tie_mode_ok(tie)) return KV4_ERR_INVALID;
  if (!is_float_dtype(x->dtype) || !is_float_dtype(s->dtype) || p->dtype != KV4_U8)
    return KV4_ERR_DTYPE;
  const int64_t d = x->shape[3];
  ng = (d + G - 1) / G;
  pb = (G + 1) / 2;
  for (int i = 0; i < 2; ++i)
    if (p->shape[i] != x->shape[i] || s->shape[i] != x->shape[i]) return KV4_ERR_SHAPE;
  if (t_off < 0 || t_off + x->shape[2] > p->shape[2] || t_off + x->shape[2] > s->shape[2])
    return KV4_ERR_SHAPE;
  if (p->shape[3] < ng * pb || s->shape[3] < ng) return KV4_ERR_SHAPE;
  return KV4_OK;
}

}  // namespace kv4

using namespace kv4;

extern "C" int kv4_quantize(const kv4_tensor *x, const kv4_tensor *packed,
                            const kv4_tensor *scales, int64_t t_off, int group_size,
                            int tie_mode, void *stream) {
  int64_t ng, pb;
  int rc = check_quant_args(x, packed, scales, t_off, group_size, tie_mode, ng, pb);
  if (rc) return rc;
  const int64_t rows = x->shape[0] * x->shape[1] * x->shape[2];
  if (rows == 0 || x->shape[3] == 0) return KV4_OK;
  QParams P{};
  fill_job(P.job[0], x, packed, scales, t_off);
  P.njobs = 1;
  P.n1 = x->shape[1];
  P.n2 = x->shape[2];
  P.rows = rows;
  P.d = x->shape[3];
  P.G = group_size;
  P.ng = static_cast<int>(ng);
  P.pb = static_cast<int>(pb);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x->dtype == KV4_F32) launch_quant_x<float>(P, scales->dtype, tie_mode, st);
  else if (x->dtype == KV4_F16) launch_quant_x<__half>(P, scales->dtype, tie_mode, st);
  else launch_quant_x<__nv_bfloat16>(P, scales->dtype, tie_mode, st);
  return cuda_status(cudaGetLastError());
}

extern "C" int kv4_append_kv(const kv4_tensor *k, const kv4_tensor *v,
                             const kv4_tensor *k_packed, const kv4_tensor *k_scales,
                             const kv4_tensor *v_packed, const kv4_tensor *v_scales,
                             int64_t pos, int group_size, int tie_mode, void *stream) {
  int64_t ng, pb, ng2, pb2;
  int rc = check_quant_args(k, k_packed, k_scales, pos, group_size, tie_mode, ng, pb);
  if (rc) return rc;
  rc = check_quant_args(v, v_packed, v_scales, pos, group_size, tie_mode, ng2, pb2);
  if (rc) return rc;
  for (int i = 0; i < 4; ++i)
    if (k->shape[i] != v->shape[i]) return KV4_ERR_SHAPE;
  if (k->dtype != v->dtype || k_scales->dtype != v_scales->dtype) return KV4_ERR_DTYPE;
  const int64_t rows = k->shape[0] * k->shape[1] * k->shape[2];
  if (rows == 0 || k->shape[3] == 0) return KV4_OK;
  QParams P{};
  fill_job(P.job[0], k, k_packed, k_scales, pos);
  fill_job(P.job[1], v, v_packed, v_scales, pos);
  P.njobs = 2;
  P.n1 = k->shape[1];
  P.n2 = k->shape[2];
  P.rows = rows;
  P.d = k->shape[3];
  P.G = group_size;
  P.ng = static_cast<int>(ng);
  P.pb = static_cast<int>(pb);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k->dtype == KV4_F32) launch_quant_x<float>(P, k_scales->dtype, tie_mode, st);
  else if (k->dtype == KV4_F16) launch_quant_x<__half>(P, k_scales->dtype, tie_mode, st);
  else launch_quant_x<__nv_bfloat16>(P, k_scales->dtype, tie_mode, st);
  return cuda_status(cudaGetLastError());
}

extern "C" int kv4_append_kv_paged(const kv4_tensor *k, const kv4_tensor *v,
                                   const kv4_tensor *k_pages, const kv4_tensor *k_scale_pages,
                                   const kv4_tensor *v_pages, const kv4_tensor *v_scale_pages,
                                   const int32_t *slot_mapping, int group_size, int tie_mode,
                                   void *stream) {
  if (!k || !v || !k_pages || !k_scale_pages || !v_pages || !v_scale_pages || !slot_mapping)
    return KV4_ERR_INVALID;
  // shape checks as for a contiguous append of B*n rows into one page
  // (dims 0 and 2 of the pools are pages and rows, not batch and tokens)
  for (int i = 0; i < 4; ++i)
    if (k->shape[i] != v->shape[i]) return KV4_ERR_SHAPE;
  if (k->dtype != v->dtype || k_scale_pages->dtype != v_scale_pages->dtype) return KV4_ERR_DTYPE;
  for (int i = 0; i < 4; ++i)
    if (k_pages->shape[i] != v_pages->shape[i] || k_scale_pages->shape[i] != v_scale_pages->shape[i])
      return KV4_ERR_SHAPE;
  if (k_pages->shape[0] != k_scale_pages->shape[0] || k_pages->shape[2] != k_scale_pages->shape[2] ||
      k_pages->shape[1] != k->shape[1] || k_scale_pages->shape[1] != k->shape[1])
    return KV4_ERR_SHAPE;
  if (group_size <= 0) return KV4_ERR_INVALID;
  if (!tie_mode_ok(tie_mode)) return KV4_ERR_INVALID;
  if (!is_float_dtype(k->dtype) || !is_float_dtype(k_scale_pages->dtype) ||
      k_pages->dtype != KV4_U8 || v_pages->dtype != KV4_U8)
    return KV4_ERR_DTYPE;
  const int64_t d = k->shape[3];
  const int64_t ng = (d + group_size - 1) / group_size, pb = (group_size + 1) / 2;
  if (k_pages->shape[3] < ng * pb || k_scale_pages->shape[3] < ng) return KV4_ERR_SHAPE;
  const int64_t rows = k->shape[0] * k->shape[1] * k->shape[2];
  if (rows == 0 || d == 0) return KV4_OK;
  QParams P{};
  fill_job(P.job[0], k, k_pages, k_scale_pages, 0);
  fill_job(P.job[1], v, v_pages, v_scale_pages, 0);
  for (int j = 0; j < 2; ++j) {
    P.job[j].slots = slot_mapping;
    P.job[j].page = k_pages->shape[2];
    P.job[j].npages = k_pages->shape[0];
  }
  P.njobs = 2;
  P.n1 = k->shape[1];
  P.n2 = k->shape[2];
  P.rows = rows;
  P.d = d;
  P.G = group_size;
  P.ng = static_cast<int>(ng);
  P.pb = static_cast<int>(pb);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k->dtype == KV4_F32) launch_quant_x<float>(P, k_scale_pages->dtype, tie_mode, st);
  else if (k->dtype == KV4_F16) launch_quant_x<__half>(P, k_scale_pages->dtype, tie_mode, st);
  else launch_quant_x<__nv_bfloat16>(P, k_scale_pages->dtype, tie_mode, st);
  return cuda_status(cudaGetLastError());
}

template <typename ST>
static void launch_dq(const DQParams &P, int odt, cudaStream_t st) {
  const int threads = 256;
  const int grid = grid_for(P.rows * P.d_out, threads);
  if (odt == KV4_F32) dequantize_kernel<ST, float><<<grid, threads, 0, st>>>(P);
  else if (odt == KV4_F16) dequantize_kernel<ST, __half><<<grid, threads, 0, st>>>(P);
  else dequantize_kernel<ST, __nv_bfloat16><<<grid, threads, 0, st>>>(P);
}

extern "C" int kv4_dequantize(const kv4_tensor *packed, const kv4_tensor *scales,
                              const kv4_tensor *out, int group_size, void *stream) {
  if (!packed || !scales || !out) return KV4_ERR_INVALID;
  if (group_size <= 0) return KV4_ERR_INVALID;
  if (packed->dtype != KV4_U8 || !is_float_dtype(scales->dtype) || !is_float_dtype(out->dtype))
    return KV4_ERR_DTYPE;
  for (int i = 0; i < 3; ++i)
    if (packed->shape[i] != scales->shape[i] || out->shape[i] != packed->shape[i])
      return KV4_ERR_SHAPE;
  const int64_t ng = scales->shape[3];
  const int64_t pw = packed->shape[3];
  if (ng <= 0) return KV4_ERR_SHAPE;
  if ((2 * pw) % ng != 0) return KV4_ERR_SHAPE;
  const int64_t slot = 2 * pw / ng;
  if (slot < group_size) return KV4_ERR_SHAPE;
  if (out->shape[3] > ng * group_size) return KV4_ERR_SHAPE;
  const int64_t rows = packed->shape[0] * packed->shape[1] * packed->shape[2];
  if (rows == 0 || out->shape[3] == 0) return KV4_OK;
  DQParams P{};
  P.p = static_cast<const uint8_t *>(packed->data);
  P.s = scales->data;
  P.o = out->data;
  for (int i = 0; i < 4; ++i) {
    P.ps[i] = packed->stride[i];
    P.ss[i] = scales->stride[i];
    P.os[i] = out->stride[i];
  }
  P.n1 = packed->shape[1];
  P.n2 = packed->shape[2];
  P.rows = rows;
  P.d_out = static_cast<int>(out->shape[3]);
  P.G = group_size;
  P.slot = static_cast<int>(slot);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (scales->dtype == KV4_F32) launch_dq<float>(P, out->dtype, st);
  else if (scales->dtype == KV4_F16) launch_dq<__half>(P, out->dtype, st);
  else launch_dq<__nv_bfloat16>(P, out->dtype, st);
  return cuda_status(cudaGetLastError());
}
