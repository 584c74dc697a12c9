// CSR aggregation kernels for sm_100a: GCNConv's weighted SpMM and GATConv's
// fused SDDMM -> LeakyReLU -> edge softmax -> SpMM, plus the degree-skew plan.
//
// Reference semantics (PyG eager, as captured op by op in
// experiments/gatconv/dumps/gat.1-raw-torch.mlir:25-129):
//   e_k  = leaky_relu(asrc[src_k] + adst[dst_k], 0.2)           (:25-38)
//   m    = scatter_amax_dst(e)  (include_self = false)           (:56-60)
//   p_k  = exp(e_k - m[dst_k])                                    (:61-65)
//   S    = scatter_add_dst(p) + 1e-16                             (:82-87)
//   out  = scatter_add_dst(p_k / S[dst_k] * h[src_k])             (:88-125)
// and for GCN the sparsifier's CSR row loop out[i] = sum_k w_k h[col_k]
// (test/reference/gcn.linalg-on-tensors.mlir:20, gnnc/schedule/sparse.py:47-62).
//
// Layout and schedule
//  * One warp owns one destination row (rows of degree <= cta_threshold).
//    Edges are taken 32 at a time: lane l loads col[k+l] and the edge's
//    logits, the warp reduces the per-head max / exp-sum with shuffles
//    (online across 32-edge chunks), and the chunk's (src, p) pairs go to
//    shared memory. The warp then streams the h[src] rows: each lane loads a
//    16-byte vector (8 bf16 or 4 fp32 features) of every row, so one edge is
//    one fully coalesced row read; loads are unrolled for memory-level
//    parallelism. Logits never leave the SM.
//  * Rows longer than cta_threshold are processed by a whole CTA (its warps
//    split the edge range and combine (max, sum, acc) in shared memory).
//    Rows longer than split_threshold are cut into segments processed by
//    different CTAs; each writes a partial (max, sum, acc) and a merge kernel
//    combines them in slot order, so results are deterministic (no float
//    atomics anywhere).
//  * The grid is persistent (a multiple of the SM count). CTAs first drain the
//    CTA work list (largest items first), then every warp pulls contiguous,
//    edge-balanced row ranges from a second list.
//  * Epilogue, fused: divide by the softmax denominator, concat or mean over
//    heads, + bias, ReLU / ELU, optional row log_softmax, convert, store.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kHMax = 16;
constexpr unsigned kFull = 0xffffffffu;

enum AggMode { MODE_GCN = 0, MODE_GAT = 1, MODE_SCORES = 2 };

struct AggParams {
  const int32_t* rowptr;
  const int32_t* col;
  const float* w;       // GCN edge values [E]
  const float* asrc;    // GAT [n_src, H]
  const float* adst;    // GAT [n_rows, H]
  const float* scores;  // MODE_SCORES [E, H]
  const void* h;
  int64_t ldh;  // elements
  int64_t n_rows, n_src;
  int64_t e_lo, e_hi;  // valid edge index range (from the plan's rowptr)
  int H, C, F, F_pad, HS;
  float slope, eps;
  int mode, concat, act, log_softmax;
  int fast_epilogue;  // concat, no log_softmax, vector-aligned out/bias: register epilogue
  const float* bias;
  void* out;
  int out_dtype;
  int64_t ldo;
  int F_out;
  const int4* cta_items;
  int64_t n_cta_items;
  const int4* split_rows;
  const int32_t* warp_tasks;
  int64_t n_warp_tasks;
  const int2* stream_tasks;  // row ranges [x, y) of warp rows only (wide launches)
  int64_t n_stream_tasks;
  int cta_threshold;
  float* partials;
  int part_stride;
  int* counters;  // [0] next CTA item, [1] next warp task, [2] bad-index flag
  const void* root;  // SAGE root term [n_rows, F_out] added before bias (null: none)
  int root_dtype;
  int64_t ldr;
};

__device__ __forceinline__ float load_val(const void* base, int dtype, size_t idx) {
  return dtype == GNNC_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx])
                            : reinterpret_cast<const float*>(base)[idx];
}

template <typename TH, int VEC>
struct VecLoad;

template <>
struct VecLoad<float, 4> {
  static __device__ __forceinline__ void run(const char* p, float* d) {
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
  }
};
template <>
struct VecLoad<float, 1> {
  static __device__ __forceinline__ void run(const char* p, float* d) {
    d[0] = __ldg(reinterpret_cast<const float*>(p));
  }
};
template <>
struct VecLoad<__nv_bfloat16, 8> {
  static __device__ __forceinline__ void run(const char* p, float* d) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    d[0] = bf16_lo(v.x); d[1] = bf16_hi(v.x); d[2] = bf16_lo(v.y); d[3] = bf16_hi(v.y);
    d[4] = bf16_lo(v.z); d[5] = bf16_hi(v.z); d[6] = bf16_lo(v.w); d[7] = bf16_hi(v.w);
  }
};
template <>
struct VecLoad<__nv_bfloat16, 1> {
  static __device__ __forceinline__ void run(const char* p, float* d) {
    unsigned short v = __ldg(reinterpret_cast<const unsigned short*>(p));
    d[0] = __uint_as_float(uint32_t(v) << 16);
  }
};

// expm1(v) for v <= 0 (ELU's negative branch, which torch computes as expm1),
// without branches. exp(v) - 1 cancels for small |v|: on (-1/64, 0] the Taylor
// polynomial v + v^2/2 + v^3/6 is used instead (truncation below v^4/24, a
// relative 1e-7 of the result there). Below -1/64 exp(v) - 1 is used, whose
// absolute error (that of the fast exponential near 1, a few 1e-7) is a
// relative error of at most ~2e-5 of |expm1(v)| >= 0.0155, falling with |v|.
__device__ __forceinline__ float expm1_nonpos(float v) {
  const float taylor = fmaf(v * v, fmaf(v, 1.f / 6.f, 0.5f), v);
  const float direct = __expf(v) - 1.f;
  return v > -0.015625f ? taylor : direct;
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == GNNC_ACT_RELU) return fmaxf(v, 0.f);
  if (act == GNNC_ACT_ELU) return v > 0.f ? v : expm1_nonpos(v);
  return v;
}

// Final value of output feature c from the aggregated [H*C] row in smem.
__device__ __forceinline__ float out_value(const AggParams& p, int64_t row, const float* s_row,
                                           int c) {
  float v;
  if (p.concat) {
    v = s_row[c];
  } else {
    v = 0.f;
    for (int hd = 0; hd < p.H; ++hd) v += s_row[hd * p.C + c];
    v = v / float(p.H);
  }
  if (p.root) v += load_val(p.root, p.root_dtype, size_t(row) * size_t(p.ldr) + c);
  if (p.bias) v += __ldg(p.bias + c);
  return apply_act(v, p.act);
}

// Epilogue for one row, run by one full warp. s_row holds the aggregated
// (already normalised) [F] values.
__device__ __forceinline__ void warp_epilogue(const AggParams& p, int64_t row, const float* s_row,
                                              int lane) {
  const int Fo = p.F_out;
  if (Fo <= 64) {
    // At most two columns per lane: each output value is formed once and kept
    // in registers (same values and summation order as the loop below).
    const int c0 = lane, c1 = lane + 32;
    const bool ok0 = c0 < Fo, ok1 = c1 < Fo;
    float v0 = ok0 ? out_value(p, row, s_row, c0) : -INFINITY;
    float v1 = ok1 ? out_value(p, row, s_row, c1) : -INFINITY;
    if (p.log_softmax) {
      const float m = warp_max(fmaxf(v0, v1));
      float se = 0.f;
      if (ok0) se += expf(v0 - m);
      if (ok1) se += expf(v1 - m);
      const float l = logf(warp_sum(se));
      v0 = (v0 - m) - l;
      v1 = (v1 - m) - l;
    }
    const size_t base = size_t(row) * size_t(p.ldo);
    if (ok0) store_val(p.out, p.out_dtype, base + c0, v0);
    if (ok1) store_val(p.out, p.out_dtype, base + c1, v1);
    return;
  }
  float mx = 0.f, lse = 0.f;
  if (p.log_softmax) {
    float m = -INFINITY;
    for (int c = lane; c < Fo; c += 32) m = fmaxf(m, out_value(p, row, s_row, c));
    mx = warp_max(m);
    float se = 0.f;
    for (int c = lane; c < Fo; c += 32) se += expf(out_value(p, row, s_row, c) - mx);
    lse = logf(warp_sum(se));
  }
  const size_t base = size_t(row) * size_t(p.ldo);
  for (int c = lane; c < Fo; c += 32) {
    float v = out_value(p, row, s_row, c);
    if (p.log_softmax) v = (v - mx) - lse;
    store_val(p.out, p.out_dtype, base + c, v);
  }
}

// Warp-wide max of a float in one instruction (sm_100a redux.sync).
__device__ __forceinline__ float warp_max_redux(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// Stores VEC consecutive outputs of one row: one 16/8-byte store when VEC >= 4.
template <int VEC>
__device__ __forceinline__ void store_vec(void* out, int dtype, size_t idx, const float* v) {
  if (dtype == GNNC_BF16) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + idx;
    if constexpr (VEC == 8) {
      *reinterpret_cast<uint4*>(o) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    } else if constexpr (VEC == 4) {
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = __float2bfloat16_rn(v[e]);
    }
  } else {
    float* o = reinterpret_cast<float*>(out) + idx;
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int e = 0; e < VEC; e += 4)
        *reinterpret_cast<float4*>(o + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = v[e];
    }
  }
}

// c{0,1} += a * b{0,1} as one packed fp32x2 FMA (same rounding as two fmaf).
__device__ __forceinline__ void ffma2(float& c0, float& c1, float a, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %2};\n\t"
      "mov.b64 rb, {%3, %4};\n\t"
      "mov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a), "f"(b0), "f"(b1));
}

// acc[e] += a * x[e] for one vector of features.
template <int VEC>
__device__ __forceinline__ void fma_vec(float* acc, float a, const float* x) {
  if constexpr (VEC % 2 == 0) {
#pragma unroll
    for (int e = 0; e < VEC; e += 2) ffma2(acc[e], acc[e + 1], a, x[e], x[e + 1]);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = fmaf(a, x[e], acc[e]);
  }
}

template <typename TH, int VEC, int LPG, int NV>
struct Agg {
  static constexpr int G = 32 / LPG;  // edge groups per warp
  static constexpr int U = NV == 1 ? 4 : (NV == 2 ? 2 : 1);

  // Accumulates edges [eb, ee) of `row`. The running per-head max lives in
  // lane hd (m_reg); acc and s_acc (the exp-sum of the lane's head) are the
  // group-partial weighted sums.
  static __device__ __forceinline__ void range(const AggParams& p, int64_t row, int eb, int ee,
                                               float (&acc)[NV][VEC], float (&s_acc)[NV],
                                               float& m_reg, int32_t* s_col, float* s_p,
                                               const int (&hv)[NV], int lane) {
    const int lig = lane % LPG;
    const int grp = lane / LPG;
    const char* hbase = reinterpret_cast<const char*>(p.h);
    const size_t ldh_b = size_t(p.ldh) * sizeof(TH);
    int voff[NV];
    bool vok[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int e0 = (v * LPG + lig) * VEC;
      voff[v] = e0 * int(sizeof(TH));
      vok[v] = e0 < p.F;
    }
    float sc_reg = 1.f;
    // a_dst of this row: lane hd holds head hd's value (broadcast per head below).
    float ad_reg = 0.f;
    if (p.mode == MODE_GAT && lane < p.H) ad_reg = __ldg(p.adst + size_t(row) * p.H + lane);
    for (int cb = eb; cb < ee; cb += 32) {
      const int k = cb + lane;
      bool valid = k < ee;
      int src = valid ? __ldg(p.col + k) : 0;
      if (valid && unsigned(src) >= unsigned(p.n_src)) {
        atomicOr(p.counters + 2, 1);
        valid = false;
        src = 0;
      }
      s_col[lane] = src;
      if (p.mode == MODE_GCN) {
        s_p[lane] = valid ? __ldg(p.w + k) : 0.f;
      } else {
        bool rescale = false;
        const float* as = p.asrc + size_t(src) * p.H;
        const float* sc_row = p.scores + size_t(k) * p.H;
        for (int hd = 0; hd < p.H; ++hd) {
          const float ad = __shfl_sync(kFull, ad_reg, hd);
          float e = -INFINITY;
          if (valid) {
            if (p.mode == MODE_GAT) {
              const float x = __ldg(as + hd) + ad;
              e = x > 0.f ? x : x * p.slope;
            } else {
              e = __ldg(sc_row + hd);
            }
          }
          const float cmax = warp_max_redux(e);
          const float m_old = __shfl_sync(kFull, m_reg, hd);
          const float m_new = fmaxf(m_old, cmax);
          // Fast exponential: relative error ~1e-6 for the arguments here (<= 0).
          const float pr = valid ? __expf(e - m_new) : 0.f;
          const float sc = __expf(m_old - m_new);  // 0 on the first chunk (m_old = -inf)
          if (lane == hd) {
            sc_reg = sc;
            m_reg = m_new;
          }
          rescale |= (cb != eb) && (m_new != m_old);
          s_p[lane * p.HS + hd] = pr;
        }
        if (rescale) {
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const float sc = __shfl_sync(kFull, sc_reg, hv[v]);
            s_acc[v] *= sc;
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[v][e] *= sc;
          }
        }
      }
      __syncwarp();
      const int n = min(32, ee - cb);
      int j = grp;
      for (; j + (U - 1) * G < n; j += U * G) {
        float hvv[U][NV][VEC];
        const char* rows[U];
#pragma unroll
        for (int u = 0; u < U; ++u) rows[u] = hbase + size_t(s_col[j + u * G]) * ldh_b;
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            if (vok[v]) {
              VecLoad<TH, VEC>::run(rows[u] + voff[v], hvv[u][v]);
            } else {
#pragma unroll
              for (int e = 0; e < VEC; ++e) hvv[u][v][e] = 0.f;
            }
          }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const float a = s_p[(j + u * G) * p.HS + hv[v]];
            s_acc[v] += a;
            fma_vec<VEC>(acc[v], a, hvv[u][v]);
          }
      }
      for (; j < n; j += G) {
        const char* r = hbase + size_t(s_col[j]) * ldh_b;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          const float a = s_p[j * p.HS + hv[v]];
          s_acc[v] += a;
          if (!vok[v]) continue;
          float x[VEC];
          VecLoad<TH, VEC>::run(r + voff[v], x);
          fma_vec<VEC>(acc[v], a, x);
        }
      }
      __syncwarp();
    }
  }

  static __device__ __forceinline__ void group_reduce(float (&acc)[NV][VEC], float (&s_acc)[NV]) {
#pragma unroll
    for (int o = LPG; o < 32; o <<= 1)
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        s_acc[v] += __shfl_xor_sync(kFull, s_acc[v], o);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[v][e] += __shfl_xor_sync(kFull, acc[v][e], o);
      }
  }

  // Writes the group-0 lanes' features, scaled by inv[v], into s_row.
  static __device__ __forceinline__ void spill(const AggParams& p, const float (&acc)[NV][VEC],
                                               const float (&inv)[NV], float* s_row, int lane) {
    if (lane < LPG) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int e0 = (v * LPG + lane) * VEC;
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (e0 + e < p.F) s_row[e0 + e] = acc[v][e] * inv[v];
      }
    }
  }

  // Concatenated heads without log_softmax: the epilogue runs in registers
  // and each lane stores its VEC outputs with one vector store.
  static __device__ __forceinline__ void store_row(const AggParams& p, int64_t row,
                                                   const float (&acc)[NV][VEC],
                                                   const float (&inv)[NV], int lane) {
    if (lane >= LPG) return;
    const size_t base = size_t(row) * size_t(p.ldo);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int e0 = (v * LPG + lane) * VEC;
      if (e0 >= p.F) continue;
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = acc[v][e] * inv[v];
      if (p.root) {
        const size_t rb = size_t(row) * size_t(p.ldr) + e0;
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (e0 + e < p.F) o[e] += load_val(p.root, p.root_dtype, rb + e);
      }
      if (p.bias) {
        if constexpr (VEC % 4 == 0) {
#pragma unroll
          for (int e = 0; e < VEC; e += 4) {
            const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + e0 + e));
            o[e] += b.x; o[e + 1] += b.y; o[e + 2] += b.z; o[e + 3] += b.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] += __ldg(p.bias + e0 + e);
        }
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = apply_act(o[e], p.act);
      if (e0 + VEC <= p.F) {
        store_vec<VEC>(p.out, p.out_dtype, base + e0, o);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (e0 + e < p.F) store_val(p.out, p.out_dtype, base + e0 + e, o[e]);
      }
    }
  }
};

// Edge loop specialised for the widest common layout: bf16 h with 8 features
// (one 16-byte load) per lane and the whole warp on one edge at a time
// (F = 256), and a compile-time head count KH (0: GCN edge weights). Same
// arithmetic, in the same order, as Agg<bf16, 8, 32, 1>::range; what changes
// is the instruction count per edge: the head loops unroll, the edges of a
// chunk are visited in groups of eight at constant shared-memory offsets with
// eight row loads in flight, and a row address is one wide multiply-add from
// a per-lane base.
template <int KH>
struct AggFast {
  static constexpr int HS = KH == 0 ? 1 : (KH | 1);

  static __device__ __forceinline__ void fma_row(float (&acc)[8], float a, const uint4& v) {
    ffma2(acc[0], acc[1], a, bf16_lo(v.x), bf16_hi(v.x));
    ffma2(acc[2], acc[3], a, bf16_lo(v.y), bf16_hi(v.y));
    ffma2(acc[4], acc[5], a, bf16_lo(v.z), bf16_hi(v.z));
    ffma2(acc[6], acc[7], a, bf16_lo(v.w), bf16_hi(v.w));
  }

  static __device__ __forceinline__ void range(const AggParams& p, int64_t row, int eb, int ee,
                                               float (&acc)[1][8], float (&s_acc)[1],
                                               float& m_reg, int32_t* s_col, float* s_p,
                                               const int (&hv)[1], int lane) {
    const char* hlane = reinterpret_cast<const char*>(p.h) + lane * 16;
    const uint32_t ldh_b = uint32_t(p.ldh) * 2u;
    const float* s_ph = s_p + hv[0];
    float sc_reg = 1.f;
    float ad_reg = 0.f;
    if (KH > 0 && p.mode == MODE_GAT && lane < KH) ad_reg = __ldg(p.adst + size_t(row) * KH + lane);
    for (int cb = eb; cb < ee; cb += 32) {
      const int k = cb + lane;
      bool valid = k < ee;
      int src = valid ? __ldg(p.col + k) : 0;
      if (valid && unsigned(src) >= unsigned(p.n_src)) {
        atomicOr(p.counters + 2, 1);
        valid = false;
        src = 0;
      }
      s_col[lane] = src;
      if constexpr (KH == 0) {
        s_p[lane] = valid ? __ldg(p.w + k) : 0.f;
      } else {
        // Lanes past the chunk's last edge read a valid row too: a_src of
        // node 0, or the chunk's first score row.
        const float* xs = p.mode == MODE_GAT ? p.asrc + size_t(src) * KH
                                             : p.scores + size_t(valid ? k : cb) * KH;
        float x[KH];
        if constexpr (KH == 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(xs));
          x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else if constexpr (KH == 2) {
          const float2 v = __ldg(reinterpret_cast<const float2*>(xs));
          x[0] = v.x; x[1] = v.y;
        } else {
#pragma unroll
          for (int hd = 0; hd < KH; ++hd) x[hd] = __ldg(xs + hd);
        }
        bool rescale = false;
#pragma unroll
        for (int hd = 0; hd < KH; ++hd) {
          // Every lane takes part in the shuffles and the reduction: `valid`
          // differs across lanes, so they stay outside its branch.
          const float ad = __shfl_sync(kFull, ad_reg, hd);
          float e = -INFINITY;
          if (valid) {
            if (p.mode == MODE_GAT) {
              const float t = x[hd] + ad;
              e = t > 0.f ? t : t * p.slope;
            } else {
              e = x[hd];
            }
          }
          const float cmax = warp_max_redux(e);
          const float m_old = __shfl_sync(kFull, m_reg, hd);
          const float m_new = fmaxf(m_old, cmax);
          const float pr = valid ? __expf(e - m_new) : 0.f;
          const float sc = __expf(m_old - m_new);
          if (lane == hd) {
            sc_reg = sc;
            m_reg = m_new;
          }
          rescale |= (cb != eb) && (m_new != m_old);
          s_p[lane * HS + hd] = pr;
        }
        if (rescale) {  // warp-uniform: m_new and m_old are the same in every lane
          const float sc = __shfl_sync(kFull, sc_reg, hv[0]);
          s_acc[0] *= sc;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[0][e] *= sc;
        }
      }
      __syncwarp();
      const int n = min(32, ee - cb);
      int j = 0;
      for (; j + 8 <= n; j += 8) {
        const int32_t* cj = s_col + j;
        const float* pj = s_ph + j * HS;
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          v[u] = __ldg(reinterpret_cast<const uint4*>(hlane + size_t(uint32_t(cj[u])) * ldh_b));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float a = pj[u * HS];
          s_acc[0] += a;
          fma_row(acc[0], a, v[u]);
        }
      }
      for (; j < n; ++j) {
        const uint4 v =
            __ldg(reinterpret_cast<const uint4*>(hlane + size_t(uint32_t(s_col[j])) * ldh_b));
        const float a = s_ph[j * HS];
        s_acc[0] += a;
        fma_row(acc[0], a, v);
      }
      __syncwarp();
    }
  }
};

// ---------------------------------------------------------------------------
// Prefetched edge stream for the 256-wide bf16 layout (AggFast's lane layout).
//
// Each edge's column index and a_src row (GCN: its weight) used to be loaded
// at the head of the edge's 32-edge chunk, so a row paid three dependent
// memory round trips (col, then a_src, then the h rows) before its first
// FMA. Here a warp walks a contiguous edge range - a task of whole rows, or
// its share of one long row - in 32-edge windows and stages them in shared
// memory with asynchronous copies (cp.async) ahead of use: window w+3's
// column indices and window w+2's a_src rows are in flight while a chunk that
// starts in window w (and may end in w+1) is processed. Rows then start with
// their inputs in shared memory and only the h gathers stay on the critical
// path. Chunks are still counted from each row's first edge, so the
// arithmetic and summation order per row are those of AggFast::range: results
// do not depend on how rows are grouped into tasks.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

template <int KH>
struct AggStream {
  static constexpr int KA = KH == 0 ? 1 : KH;  // floats staged per edge (a_src row or weight)
  // The chunk's softmax weights sit head by head in s_p (s_p[hd * PS + edge]),
  // so that a lane reads four consecutive edges' weights of its head with one
  // 16-byte load; PS = 36 puts the heads' rows 4 banks apart (conflict-free
  // for the lanes of different heads). The buffer holds 32 * (KH | 1) floats.
  static constexpr int PS = KH <= 1 ? 32 : 36;
  static_assert(KH * PS <= 32 * (KH | 1), "s_p capacity");

  // Per-warp shared memory. Window slots are rings indexed by window & 3.
  struct Win {
    float as[4][32 * KA];    // a_src rows (GCN: weights) of windows w .. w+2
    float adst[2][32 * KA];  // a_dst rows of the current / next batch of 31 rows
    int32_t col[4][32];      // column indices of windows w .. w+3
    int32_t rp[2][32];       // row pointers of the current / next batch of 31 rows
  };

  // The stream [s0, s1) and the current window (edges base .. base+32).
  struct Cursor {
    int s0, s1, w, base;
    int epoch;  // counts the waits for all outstanding copies
  };

  static __device__ __forceinline__ void issue_col(const AggParams& p, Win& s, const Cursor& c,
                                                   int w, int lane) {
    const int k = c.s0 + 32 * w + lane;
    if (k < c.s1) cp_async4(&s.col[w & 3][lane], p.col + k);
  }

  // Needs window w's column indices in shared memory.
  static __device__ __forceinline__ void issue_as(const AggParams& p, Win& s, const Cursor& c,
                                                  int w, int lane) {
    const int k = c.s0 + 32 * w + lane;
    if (k >= c.s1) return;
    float* dst = &s.as[w & 3][lane * KA];
    if constexpr (KH == 0) {
      cp_async4(dst, p.w + k);
    } else {
      const int src = s.col[w & 3][lane];
      if (unsigned(src) >= unsigned(p.n_src)) return;  // reported when the edge is processed
      const float* a = p.asrc + size_t(src) * KH;
      if constexpr (KH == 1) {
        cp_async4(dst, a);
      } else if constexpr (KH == 2) {
        cp_async8(dst, a);
      } else if constexpr (KH == 4) {
        cp_async16(dst, a);
      } else {
        cp_async16(dst, a);
        cp_async16(dst + 4, a + 4);
      }
    }
  }

  // Starts the stream [s0, s1) at window 0.
  static __device__ __forceinline__ void begin(const AggParams& p, Win& s, Cursor& c, int s0,
                                               int s1, int lane) {
    c.s0 = s0;
    c.s1 = s1;
    c.epoch = 0;
    for (int w = 0; w < 3; ++w) issue_col(p, s, c, w, lane);
    cp_async_commit();
    cp_async_wait_all();
    __syncwarp();
    issue_as(p, s, c, 0, lane);
    issue_as(p, s, c, 1, lane);
    cp_async_commit();
    advance_to(p, s, c, 0, lane);
  }

  // Window w becomes current. Once this returns, the column indices of
  // windows w .. w+2 and the a_src rows of windows w, w+1 are in shared
  // memory, and window w+2's a_src rows and window w+3's column indices are
  // in flight. A 32-edge chunk that starts in window w ends in w or w+1.
  static __device__ __forceinline__ void advance_to(const AggParams& p, Win& s, Cursor& c, int w,
                                                    int lane) {
    cp_async_wait_all();
    ++c.epoch;
    __syncwarp();
    c.w = w;
    c.base = c.s0 + 32 * w;
    issue_as(p, s, c, w + 2, lane);
    issue_col(p, s, c, w + 3, lane);
    cp_async_commit();
  }

  // Row epilogue for concatenated heads, bf16 output, no root term: the lane's
  // 8 features are scaled, biased and activated as fp32 pairs (f32x2), with
  // the same per-element operations and rounding as Agg::store_row.
  static __device__ __forceinline__ uint64_t pk(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
  }
  static __device__ __forceinline__ void upk(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  }
  static __device__ __forceinline__ void store_bf16(const AggParams& p, int64_t row,
                                                    const float (&acc)[8], float inv, int lane) {
    const int e0 = lane * 8;
    uint64_t o[4];
    const uint64_t ii = pk(inv, inv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[i] = pk(acc[2 * i], acc[2 * i + 1]);
      asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(o[i]) : "l"(ii));
    }
    if (p.bias) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.bias + e0));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.bias + e0 + 4));
      const uint64_t bb[4] = {pk(b0.x, b0.y), pk(b0.z, b0.w), pk(b1.x, b1.y), pk(b1.z, b1.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) asm("add.rn.f32x2 %0, %0, %1;" : "+l"(o[i]) : "l"(bb[i]));
    }
    float v[8];
    if (p.act == GNNC_ACT_ELU) {
      const uint64_t c6 = pk(1.f / 6.f, 1.f / 6.f), c5 = pk(0.5f, 0.5f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // expm1_nonpos on both halves: v + v^2 (1/2 + v/6) and exp(v) - 1
        uint64_t vv, t, taylor;
        asm("mul.rn.f32x2 %0, %1, %1;" : "=l"(vv) : "l"(o[i]));
        asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(t) : "l"(o[i]), "l"(c6), "l"(c5));
        asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(taylor) : "l"(vv), "l"(t), "l"(o[i]));
        float x0, x1, t0, t1;
        upk(o[i], x0, x1);
        upk(taylor, t0, t1);
        const float d0 = __expf(x0) - 1.f, d1 = __expf(x1) - 1.f;
        v[2 * i] = x0 > 0.f ? x0 : (x0 > -0.015625f ? t0 : d0);
        v[2 * i + 1] = x1 > 0.f ? x1 : (x1 > -0.015625f ? t1 : d1);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        upk(o[i], v[2 * i], v[2 * i + 1]);
        v[2 * i] = apply_act(v[2 * i], p.act);
        v[2 * i + 1] = apply_act(v[2 * i + 1], p.act);
      }
    }
    store_vec<8>(p.out, GNNC_BF16, size_t(row) * size_t(p.ldo) + e0, v);
  }

  // R edges (compile-time count): R row loads in flight, then R FMAs in order.
  template <int R>
  static __device__ __forceinline__ void tail(const int32_t* cj, const float* pj,
                                              const char* hlane, uint32_t ldh_b,
                                              float (&acc)[8], float& s_acc) {
    uint4 v[R];
#pragma unroll
    for (int u = 0; u < R; ++u)
      v[u] = __ldg(reinterpret_cast<const uint4*>(hlane + size_t(uint32_t(cj[u])) * ldh_b));
#pragma unroll
    for (int u = 0; u < R; ++u) {
      s_acc += pj[u];
      AggFast<KH>::fma_row(acc, pj[u], v[u]);
    }
  }

  // Accumulates the row's edges [eb, ee), which must be the next edges of
  // the stream, in 32-edge chunks counted from eb. ad_reg: lane hd holds
  // a_dst of head hd. Same arithmetic and order as AggFast<KH>::range.
  static __device__ __forceinline__ void row(const AggParams& p, Win& s, Cursor& c, int eb,
                                             int ee, float ad_reg, float (&acc)[8], float& s_acc,
                                             float& m_reg, int32_t* s_col, float* s_p, int hv,
                                             int lane) {
    const char* hlane = reinterpret_cast<const char*>(p.h) + lane * 16;
    const uint32_t ldh_b = uint32_t(p.ldh) * 2u;
    const float* s_ph = s_p + hv * PS;
    float sc_reg = 1.f;
    for (int cb = eb; cb < ee; cb += 32) {
      if (cb >= c.base + 32) advance_to(p, s, c, c.w + 1, lane);
      const int k = cb + lane;
      bool valid = k < ee;
      const int off = k - c.base;  // < 64 for every valid lane
      const int slot = (c.w + (off >> 5)) & 3, pos = off & 31;
      int src = valid ? s.col[slot][pos] : 0;
      if (valid && unsigned(src) >= unsigned(p.n_src)) {
        atomicOr(p.counters + 2, 1);
        valid = false;
        src = 0;
      }
      s_col[lane] = src;
      const float* xs = &s.as[valid ? slot : 0][(valid ? pos : 0) * KA];
      if constexpr (KH == 0) {
        s_p[lane] = valid ? xs[0] : 0.f;
      } else {
        float x[KH];
        if constexpr (KH == 4) {
          const float4 v = *reinterpret_cast<const float4*>(xs);
          x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else if constexpr (KH == 2) {
          const float2 v = *reinterpret_cast<const float2*>(xs);
          x[0] = v.x; x[1] = v.y;
        } else {
#pragma unroll
          for (int hd = 0; hd < KH; ++hd) x[hd] = xs[hd];
        }
        bool rescale = false;
        if (cb == eb) {
          // A row's first chunk: the running max starts at this chunk's max
          // (the general step below with m_old = -inf, nothing to rescale).
#pragma unroll
          for (int hd = 0; hd < KH; ++hd) {
            const float ad = __shfl_sync(kFull, ad_reg, hd);
            float e = -INFINITY;
            if (valid) {
              const float t = x[hd] + ad;
              e = t > 0.f ? t : t * p.slope;
            }
            const float m_new = warp_max_redux(e);
            const float pr = valid ? __expf(e - m_new) : 0.f;
            if (lane == hd) m_reg = m_new;
            s_p[hd * PS + lane] = pr;
          }
        } else {
#pragma unroll
          for (int hd = 0; hd < KH; ++hd) {
            // every lane takes part in the shuffles and the reduction
            const float ad = __shfl_sync(kFull, ad_reg, hd);
            float e = -INFINITY;
            if (valid) {
              const float t = x[hd] + ad;
              e = t > 0.f ? t : t * p.slope;
            }
            const float cmax = warp_max_redux(e);
            const float m_old = __shfl_sync(kFull, m_reg, hd);
            const float m_new = fmaxf(m_old, cmax);
            const float pr = valid ? __expf(e - m_new) : 0.f;
            const float sc = __expf(m_old - m_new);
            if (lane == hd) {
              sc_reg = sc;
              m_reg = m_new;
            }
            rescale |= m_new != m_old;
            s_p[hd * PS + lane] = pr;
          }
        }
        if (rescale) {  // warp-uniform
          const float sc = __shfl_sync(kFull, sc_reg, hv);
          s_acc *= sc;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] *= sc;
        }
      }
      __syncwarp();
      const int n = min(32, ee - cb);
      int j = 0;
      for (; j + 8 <= n; j += 8) {
        // s_col and s_p rows are 16-byte aligned and j is a multiple of 8
        const int4 c0 = *reinterpret_cast<const int4*>(s_col + j);
        const int4 c1 = *reinterpret_cast<const int4*>(s_col + j + 4);
        const int cj[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          v[u] = __ldg(reinterpret_cast<const uint4*>(hlane + size_t(uint32_t(cj[u])) * ldh_b));
        const float4 q0 = *reinterpret_cast<const float4*>(s_ph + j);
        const float4 q1 = *reinterpret_cast<const float4*>(s_ph + j + 4);
        const float pj[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          s_acc += pj[u];
          AggFast<KH>::fma_row(acc, pj[u], v[u]);
        }
      }
      // The last 1-7 edges: their row loads go out together (one round trip,
      // not one per edge), then fold in edge order. The count is the same in
      // every lane, so each case issues exactly its loads and FMAs.
      switch (n - j) {
        case 1: tail<1>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        case 2: tail<2>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        case 3: tail<3>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        case 4: tail<4>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        case 5: tail<5>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        case 6: tail<6>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        case 7: tail<7>(s_col + j, s_ph + j, hlane, ldh_b, acc, s_acc); break;
        default: break;
      }
      __syncwarp();
    }
  }
};

// Phase 2 with the prefetched stream: a warp takes a task of consecutive warp
// rows (the plan leaves the CTA rows out of these tasks, so the task's edges
// are one contiguous range) and streams through its edges. The row pointers
// and a_dst rows of the next 31 rows are staged the same way, one batch ahead.
template <int KH>
__device__ __forceinline__ void stream_tasks(const AggParams& p, typename AggStream<KH>::Win& s,
                                             int32_t* s_col, float* s_p, float* s_row, int hv,
                                             int lane) {
  using S = AggStream<KH>;
  using A = Agg<__nv_bfloat16, 8, 32, 1>;
  constexpr int KA = S::KA;
  const bool softmax = p.mode != MODE_GCN;
  const bool bf16_epilogue = p.fast_epilogue && !p.root && p.out_dtype == GNNC_BF16;
  for (;;) {
    int t = 0;
    if (lane == 0) t = atomicAdd(p.counters + 1, 1);
    t = __shfl_sync(kFull, t, 0);
    if (t >= p.n_stream_tasks) break;
    const int2 task = p.stream_tasks[t];
    const int r0 = task.x, r1 = task.y;
    int rr = 0;
    if (lane < 2) rr = __ldg(p.rowptr + (lane == 0 ? r0 : r1));
    const int s0 = int(max(int64_t(__shfl_sync(kFull, rr, 0)), p.e_lo));
    const int s1 = int(min(int64_t(__shfl_sync(kFull, rr, 1)), p.e_hi));
    // Row pointers rowptr[rb .. rb+31] and the a_dst rows of rows rb .. rb+30
    // of one batch, into batch slot `slot`.
    auto issue_batch = [&](int slot, int rb) {
      const int nr = min(31, r1 - rb);
      if (lane <= nr) cp_async4(&s.rp[slot][lane], p.rowptr + rb + lane);
      if constexpr (KH > 0) {
        if (lane < nr) {
          const float* a = p.adst + size_t(rb + lane) * KH;
          float* d = &s.adst[slot][lane * KA];
          if constexpr (KH == 1) {
            cp_async4(d, a);
          } else if constexpr (KH == 2) {
            cp_async8(d, a);
          } else if constexpr (KH == 4) {
            cp_async16(d, a);
          } else {
            cp_async16(d, a);
            cp_async16(d + 4, a + 4);
          }
        }
      }
    };
    issue_batch(0, r0);
    cp_async_commit();
    typename S::Cursor c;
    S::begin(p, s, c, s0, s1, lane);  // its waits also land batch 0
    int batch_epoch = c.epoch;
    bool fresh = true;  // batch 0 landed in begin()
    for (int rb = r0, bi = 0; rb < r1; rb += 31, bi ^= 1) {
      if (!fresh && c.epoch == batch_epoch) {  // no window wait since it was issued
        cp_async_wait_all();
        ++c.epoch;
        __syncwarp();
      }
      fresh = false;
      if (rb + 31 < r1) {
        issue_batch(bi ^ 1, rb + 31);
        cp_async_commit();
        batch_epoch = c.epoch;
      }
      const int nr = min(31, r1 - rb);
      const int rpv = s.rp[bi][lane];
      for (int i = 0; i < nr; ++i) {
        const int r = rb + i;
        const int eb = int(max(int64_t(__shfl_sync(kFull, rpv, i)), p.e_lo));
        const int ee = int(min(int64_t(__shfl_sync(kFull, rpv, i + 1)), p.e_hi));
        const float ad_reg = (KH > 0 && lane < KH) ? s.adst[bi][i * KA + lane] : 0.f;
        float acc[1][8], s_acc[1], inv[1];
        s_acc[0] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[0][e] = 0.f;
        float m_reg = -INFINITY;
        if (ee > eb)
          S::row(p, s, c, eb, ee, ad_reg, acc[0], s_acc[0], m_reg, s_col, s_p, hv, lane);
        // correctly rounded reciprocal: the same value as 1.f / x
        inv[0] = (softmax && ee > eb) ? __frcp_rn(s_acc[0] + p.eps) : 1.f;
        if (bf16_epilogue) {
          S::store_bf16(p, r, acc[0], inv[0], lane);
        } else if (p.fast_epilogue) {
          A::store_row(p, r, acc, inv, lane);
        } else {
          A::spill(p, acc, inv, s_row, lane);
          __syncwarp();
          warp_epilogue(p, r, s_row, lane);
          __syncwarp();
        }
      }
    }
    // Nothing may still be landing in this warp's buffers when they are reused.
    cp_async_wait_all();
    __syncwarp();
  }
}

// Edge loop specialised for narrow bf16 rows (32 < F <= 64: one 16-byte load
// per lane, four edges side by side in 8-lane groups) and a compile-time head
// count KH (0: GCN edge weights). The scores are formed as in AggFast; each
// group then takes every fourth edge of the chunk, eight at a time with
// predicated loads, so a partial chunk costs no loop control. Same arithmetic
// per edge, in the same order within a group, as Agg<bf16, 8, 8, 1>::range.
template <int KH>
struct AggNarrow {
  static constexpr int HS = KH == 0 ? 1 : (KH | 1);

  static __device__ __forceinline__ void range(const AggParams& p, int64_t row, int eb, int ee,
                                               float (&acc)[1][8], float (&s_acc)[1],
                                               float& m_reg, int32_t* s_col, float* s_p,
                                               const int (&hv)[1], int lane) {
    const int lig = lane & 7;
    const int grp = lane >> 3;
    const bool vok = lig * 8 < p.F;
    const char* hlane = reinterpret_cast<const char*>(p.h) + lig * 16;
    const uint32_t ldh_b = uint32_t(p.ldh) * 2u;
    const float* s_ph = s_p + hv[0];
    float sc_reg = 1.f;
    float ad_reg = 0.f;
    if (KH > 0 && p.mode == MODE_GAT && lane < KH) ad_reg = __ldg(p.adst + size_t(row) * KH + lane);
    for (int cb = eb; cb < ee; cb += 32) {
      const int k = cb + lane;
      bool valid = k < ee;
      int src = valid ? __ldg(p.col + k) : 0;
      if (valid && unsigned(src) >= unsigned(p.n_src)) {
        atomicOr(p.counters + 2, 1);
        valid = false;
        src = 0;
      }
      s_col[lane] = src;
      if constexpr (KH == 0) {
        s_p[lane] = valid ? __ldg(p.w + k) : 0.f;
      } else {
        const float* xs = p.mode == MODE_GAT ? p.asrc + size_t(src) * KH
                                             : p.scores + size_t(valid ? k : cb) * KH;
        bool rescale = false;
#pragma unroll
        for (int hd = 0; hd < KH; ++hd) {
          const float ad = __shfl_sync(kFull, ad_reg, hd);
          float e = -INFINITY;
          if (valid) {
            const float x = __ldg(xs + hd);
            if (p.mode == MODE_GAT) {
              const float t = x + ad;
              e = t > 0.f ? t : t * p.slope;
            } else {
              e = x;
            }
          }
          const float cmax = warp_max_redux(e);
          const float m_old = __shfl_sync(kFull, m_reg, hd);
          const float m_new = fmaxf(m_old, cmax);
          const float pr = valid ? __expf(e - m_new) : 0.f;
          const float sc = __expf(m_old - m_new);
          if (lane == hd) {
            sc_reg = sc;
            m_reg = m_new;
          }
          rescale |= (cb != eb) && (m_new != m_old);
          s_p[lane * HS + hd] = pr;
        }
        if (rescale) {  // warp-uniform
          const float sc = __shfl_sync(kFull, sc_reg, hv[0]);
          s_acc[0] *= sc;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[0][e] *= sc;
        }
      }
      __syncwarp();
      const int n = min(32, ee - cb);
      uint4 v[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int j = grp + 4 * t;
        v[t] = make_uint4(0u, 0u, 0u, 0u);
        if (vok && j < n)
          v[t] = __ldg(reinterpret_cast<const uint4*>(hlane + size_t(uint32_t(s_col[j])) * ldh_b));
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int j = grp + 4 * t;
        if (j < n) {
          const float a = s_ph[j * HS];
          s_acc[0] += a;
          AggFast<KH>::fma_row(acc[0], a, v[t]);
        }
      }
      __syncwarp();
    }
  }
};

// Phase 2 of agg_kernel for narrow bf16 rows (32 < F <= 64) with one head or
// GCN weights (written for up to four heads): one destination row per 8-lane group,
// four rows per warp at a time, so four rows' chains of dependent loads (col,
// then a_src, then h) overlap instead of running one after another. Within a
// group, lane l scores edge 8c + l of chunk c (group-wide max by xor
// shuffles, online softmax across chunks), then every lane gathers its 16-byte
// slice of the chunk's h rows in edge order and folds it in, as the one-row
// loops do. The warp runs as many chunks as its longest row needs; finished
// groups idle through the rest. Rows above the CTA threshold are skipped.
template <int KH>
__device__ __forceinline__ void narrow_rows(const AggParams& p, int32_t* s_col, float* s_p,
                                            int lane, bool softmax) {
  constexpr int HS = KH == 0 ? 1 : (KH | 1);
  constexpr int KX = KH > 0 ? KH : 1;
  const int lig = lane & 7, grp = lane >> 3;
  const bool vok = lig * 8 < p.F;
  const char* hlane = reinterpret_cast<const char*>(p.h) + lig * 16;
  const uint32_t ldh_b = uint32_t(p.ldh) * 2u;
  const int hv = KH > 1 ? min((lig * 8) / p.C, KH - 1) : 0;
  const float* s_pg = s_p + (grp * 8) * HS + hv;
  const int32_t* s_cg = s_col + grp * 8;
  for (;;) {
    int t = 0;
    if (lane == 0) t = atomicAdd(p.counters + 1, 1);
    t = __shfl_sync(kFull, t, 0);
    if (t >= p.n_warp_tasks) break;
    const int r0 = p.warp_tasks[t], r1 = p.warp_tasks[t + 1];
    for (int rb = r0; rb < r1; rb += 4) {
      const int r = rb + grp;
      int eb = 0, ee = 0;
      bool active = r < r1;
      if (active) {
        eb = int(max(int64_t(__ldg(p.rowptr + r)), p.e_lo));
        ee = int(min(int64_t(__ldg(p.rowptr + r + 1)), p.e_hi));
        if (ee - eb > p.cta_threshold) active = false;
      }
      if (!active) eb = ee = 0;
      float ad[KX], m[KX];
#pragma unroll
      for (int hd = 0; hd < KX; ++hd) {
        ad[hd] = (KH > 0 && active && p.mode == MODE_GAT) ? __ldg(p.adst + size_t(r) * KH + hd)
                                                           : 0.f;
        m[hd] = -INFINITY;
      }
      float acc[8], s_acc = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      const int nch = __reduce_max_sync(kFull, unsigned(ee - eb + 7) >> 3);
      for (int c = 0; c < int(nch); ++c) {
        const int k = eb + c * 8 + lig;
        bool valid = k < ee;
        int src = valid ? __ldg(p.col + k) : 0;
        if (valid && unsigned(src) >= unsigned(p.n_src)) {
          atomicOr(p.counters + 2, 1);
          valid = false;
          src = 0;
        }
        s_col[lane] = src;
        if constexpr (KH == 0) {
          s_p[lane] = valid ? __ldg(p.w + k) : 0.f;
        } else {
          const float* xs = p.mode == MODE_GAT ? p.asrc + size_t(src) * KH
                                               : p.scores + size_t(valid ? k : 0) * KH;
          bool rescale = false;
          float scl = 1.f;
#pragma unroll
          for (int hd = 0; hd < KH; ++hd) {
            float e = -INFINITY;
            if (valid) {
              const float x = __ldg(xs + hd);
              if (p.mode == MODE_GAT) {
                const float tt = x + ad[hd];
                e = tt > 0.f ? tt : tt * p.slope;
              } else {
                e = x;
              }
            }
            float cmax = e;  // group-wide max: the xor partners stay inside the 8-lane group
            cmax = fmaxf(cmax, __shfl_xor_sync(kFull, cmax, 4));
            cmax = fmaxf(cmax, __shfl_xor_sync(kFull, cmax, 2));
            cmax = fmaxf(cmax, __shfl_xor_sync(kFull, cmax, 1));
            const float m_new = fmaxf(m[hd], cmax);
            const float pr = valid ? __expf(e - m_new) : 0.f;
            if (hd == hv) {
              rescale = (c > 0) && (m_new != m[hd]);
              scl = __expf(m[hd] - m_new);
            }
            m[hd] = m_new;
            s_p[lane * HS + hd] = pr;
          }
          if (rescale) {  // uniform within the group; no shuffle below
            s_acc *= scl;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] *= scl;
          }
        }
        __syncwarp();
        const int n = min(8, max(0, ee - (eb + c * 8)));
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          v[u] = make_uint4(0u, 0u, 0u, 0u);
          if (vok && u < n)
            v[u] = __ldg(reinterpret_cast<const uint4*>(hlane + size_t(uint32_t(s_cg[u])) * ldh_b));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (u < n) {
            const float a = s_pg[u * HS];
            s_acc += a;
            AggFast<KH>::fma_row(acc, a, v[u]);
          }
        }
        __syncwarp();
      }
      // Epilogue of the group's row: lane lig holds features [8 lig, 8 lig + 8).
      const float inv = (softmax && ee > eb) ? 1.f / (s_acc + p.eps) : 1.f;
      const int e0 = lig * 8;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const bool ok = active && e0 + e < p.F;
        float v = acc[e] * inv;
        if (ok && p.root) v += load_val(p.root, p.root_dtype, size_t(r) * size_t(p.ldr) + e0 + e);
        if (ok && p.bias) v += __ldg(p.bias + e0 + e);
        o[e] = apply_act(v, p.act);
      }
      if (p.log_softmax) {
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e0 + e < p.F) mx = fmaxf(mx, o[e]);
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
        float se = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e0 + e < p.F) se += expf(o[e] - mx);
        se += __shfl_xor_sync(kFull, se, 4);
        se += __shfl_xor_sync(kFull, se, 2);
        se += __shfl_xor_sync(kFull, se, 1);
        const float lse = logf(se);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = (o[e] - mx) - lse;
      }
      if (active) {
        const size_t base = size_t(r) * size_t(p.ldo) + e0;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e0 + e < p.F) store_val(p.out, p.out_dtype, base + e, o[e]);
      }
    }
  }
}

// Edge loop specialised for fp32 rows of 256 features (two 16-byte loads per
// lane per edge, the Agg<float, 4, 32, 2> layout: lane l holds features
// [4l, 4l+4) and [128+4l, 128+4l+4)) and a compile-time head count KH (0: GCN
// weights): the AggFast scheme (unrolled heads, groups of four edges with
// eight loads in flight, constant shared-memory offsets) with the same
// arithmetic and order as Agg<float, 4, 32, 2>::range.
template <int KH>
struct AggFast32 {
  static constexpr int HS = KH == 0 ? 1 : (KH | 1);

  static __device__ __forceinline__ void fma4(float (&acc)[4], float a, const float4& v) {
    ffma2(acc[0], acc[1], a, v.x, v.y);
    ffma2(acc[2], acc[3], a, v.z, v.w);
  }

  static __device__ __forceinline__ void range(const AggParams& p, int64_t row, int eb, int ee,
                                               float (&acc)[2][4], float (&s_acc)[2],
                                               float& m_reg, int32_t* s_col, float* s_p,
                                               const int (&hv)[2], int lane) {
    const char* hl0 = reinterpret_cast<const char*>(p.h) + lane * 16;
    const char* hl1 = hl0 + 512;
    const size_t ldh_b = size_t(p.ldh) * 4u;
    const float* s_ph0 = s_p + hv[0];
    const float* s_ph1 = s_p + hv[1];
    float sc_reg = 1.f;
    float ad_reg = 0.f;
    if (KH > 0 && p.mode == MODE_GAT && lane < KH) ad_reg = __ldg(p.adst + size_t(row) * KH + lane);
    for (int cb = eb; cb < ee; cb += 32) {
      const int k = cb + lane;
      bool valid = k < ee;
      int src = valid ? __ldg(p.col + k) : 0;
      if (valid && unsigned(src) >= unsigned(p.n_src)) {
        atomicOr(p.counters + 2, 1);
        valid = false;
        src = 0;
      }
      s_col[lane] = src;
      if constexpr (KH == 0) {
        s_p[lane] = valid ? __ldg(p.w + k) : 0.f;
      } else {
        const float* xs = p.mode == MODE_GAT ? p.asrc + size_t(src) * KH
                                             : p.scores + size_t(valid ? k : cb) * KH;
        bool rescale = false;
#pragma unroll
        for (int hd = 0; hd < KH; ++hd) {
          const float ad = __shfl_sync(kFull, ad_reg, hd);  // every lane: outside `valid`
          float e = -INFINITY;
          if (valid) {
            const float x = __ldg(xs + hd);
            if (p.mode == MODE_GAT) {
              const float t = x + ad;
              e = t > 0.f ? t : t * p.slope;
            } else {
              e = x;
            }
          }
          const float cmax = warp_max_redux(e);
          const float m_old = __shfl_sync(kFull, m_reg, hd);
          const float m_new = fmaxf(m_old, cmax);
          const float pr = valid ? __expf(e - m_new) : 0.f;
          const float sc = __expf(m_old - m_new);
          if (lane == hd) {
            sc_reg = sc;
            m_reg = m_new;
          }
          rescale |= (cb != eb) && (m_new != m_old);
          s_p[lane * HS + hd] = pr;
        }
        if (rescale) {  // warp-uniform
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const float sc = __shfl_sync(kFull, sc_reg, hv[v]);
            s_acc[v] *= sc;
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[v][e] *= sc;
          }
        }
      }
      __syncwarp();
      const int n = min(32, ee - cb);
      int j = 0;
      for (; j + 4 <= n; j += 4) {
        float4 v0[4], v1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const size_t off = size_t(uint32_t(s_col[j + u])) * ldh_b;
          v0[u] = __ldg(reinterpret_cast<const float4*>(hl0 + off));
          v1[u] = __ldg(reinterpret_cast<const float4*>(hl1 + off));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float a0 = s_ph0[(j + u) * HS], a1 = s_ph1[(j + u) * HS];
          s_acc[0] += a0;
          fma4(acc[0], a0, v0[u]);
          s_acc[1] += a1;
          fma4(acc[1], a1, v1[u]);
        }
      }
      for (; j < n; ++j) {
        const size_t off = size_t(uint32_t(s_col[j])) * ldh_b;
        const float4 v0 = __ldg(reinterpret_cast<const float4*>(hl0 + off));
        const float4 v1 = __ldg(reinterpret_cast<const float4*>(hl1 + off));
        const float a0 = s_ph0[j * HS], a1 = s_ph1[j * HS];
        s_acc[0] += a0;
        fma4(acc[0], a0, v0);
        s_acc[1] += a1;
        fma4(acc[1], a1, v1);
      }
      __syncwarp();
    }
  }
};

// Selects the edge loop: the specialised one for KH >= 0, the generic otherwise.
template <typename TH, int VEC, int LPG, int NV, int KH>
struct EdgeLoop {
  using type = Agg<TH, VEC, LPG, NV>;
};
template <int KH>
struct EdgeLoop<__nv_bfloat16, 8, 32, 1, KH> {
  using type = AggFast<KH>;
};
template <>
struct EdgeLoop<__nv_bfloat16, 8, 32, 1, -1> {
  using type = Agg<__nv_bfloat16, 8, 32, 1>;
};
template <int KH>
struct EdgeLoop<float, 4, 32, 2, KH> {
  using type = AggFast32<KH>;
};
template <>
struct EdgeLoop<float, 4, 32, 2, -1> {
  using type = Agg<float, 4, 32, 2>;
};
template <int KH>
struct EdgeLoop<__nv_bfloat16, 8, 8, 1, KH> {
  using type = AggNarrow<KH>;
};
template <>
struct EdgeLoop<__nv_bfloat16, 8, 8, 1, -1> {
  using type = Agg<__nv_bfloat16, 8, 8, 1>;
};

// Phase 2 of agg_kernel without the edge stream: warps pull edge-balanced row
// ranges and process their rows one at a time with the layout's edge loop.
template <typename TH, int VEC, int LPG, int NV, int KH>
__device__ __forceinline__ void warp_rows(const AggParams& p, int32_t* s_col, float* s_p,
                                          float* s_row, const int (&hv)[NV], int lane) {
  using A = Agg<TH, VEC, LPG, NV>;
  using L = typename EdgeLoop<TH, VEC, LPG, NV, KH>::type;
  const bool softmax = p.mode != MODE_GCN;
  // (one head or GCN weights: measured faster than the one-row loop; with
  // four heads the per-head group reductions cost more than the overlap gains)
  if constexpr (KH >= 0 && KH <= 1 && LPG == 8 && NV == 1 && VEC == 8) {
    if (p.concat || p.H == 1) {
      narrow_rows<KH>(p, s_col, s_p, lane, softmax);
      return;
    }
  }
  for (;;) {
    int t = 0;
    if (lane == 0) t = atomicAdd(p.counters + 1, 1);
    t = __shfl_sync(kFull, t, 0);
    if (t >= p.n_warp_tasks) break;
    const int r0 = p.warp_tasks[t], r1 = p.warp_tasks[t + 1];
    // The task's row pointers come in with one load per 31 rows (lane i holds
    // rowptr[rb + i]) instead of two dependent loads at the head of each row.
    for (int rb = r0; rb < r1; rb += 31) {
      const int nr = min(31, r1 - rb);
      const int rpv = lane <= nr ? __ldg(p.rowptr + rb + lane) : 0;
      for (int i = 0; i < nr; ++i) {
        const int r = rb + i;
        const int eb = max(int64_t(__shfl_sync(kFull, rpv, i)), p.e_lo);
        const int ee = min(int64_t(__shfl_sync(kFull, rpv, i + 1)), p.e_hi);
        if (ee - eb > p.cta_threshold) continue;
        float acc[NV][VEC], s_acc[NV], inv[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          s_acc[v] = 0.f;
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[v][e] = 0.f;
        }
        float m_reg = -INFINITY;
        if (ee > eb) {
          L::range(p, r, eb, ee, acc, s_acc, m_reg, s_col, s_p, hv, lane);
          A::group_reduce(acc, s_acc);
        }
        const bool divide = softmax && ee > eb;
#pragma unroll
        for (int v = 0; v < NV; ++v) inv[v] = divide ? 1.f / (s_acc[v] + p.eps) : 1.f;
        if (p.fast_epilogue) {
          A::store_row(p, r, acc, inv, lane);
        } else {
          A::spill(p, acc, inv, s_row, lane);
          __syncwarp();
          warp_epilogue(p, r, s_row, lane);
          __syncwarp();
        }
      }
    }
  }
}

// Floats of the shared-memory carve-up below, before the stream buffers.
__host__ __device__ constexpr int agg_smem_floats(int F_pad, int HS) {
  return kWarps * 32 + kWarps * 32 * HS + kWarps * F_pad + 2 * kWarps * kHMax + F_pad +
         2 * kHMax;
}

// STREAM: the 256-wide bf16 layout with the prefetched edge stream (AggStream)
// in both phases; KH >= 0 and GAT or GCN mode only.
template <typename TH, int VEC, int LPG, int NV, int KH = -1, bool STREAM = false>
__global__ void __launch_bounds__(kThreads, 4) agg_kernel(const AggParams p) {
  using A = Agg<TH, VEC, LPG, NV>;
  using L = typename EdgeLoop<TH, VEC, LPG, NV, KH>::type;
  static_assert(!STREAM || (KH >= 0 && LPG == 32 && NV == 1 && VEC == 8), "stream layout");
  using Win = typename AggStream<(KH >= 0 ? KH : 0)>::Win;
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Shared memory carve-up (floats).
  int32_t* s_col_all = reinterpret_cast<int32_t*>(smem);            // kWarps*32
  float* s_p_all = smem + kWarps * 32;                                // kWarps*32*HS
  float* s_row_all = s_p_all + kWarps * 32 * p.HS;                   // kWarps*F_pad
  float* s_wm = s_row_all + kWarps * p.F_pad;                         // kWarps*kHMax
  float* s_ws = s_wm + kWarps * kHMax;                                // kWarps*kHMax
  float* s_fin = s_ws + kWarps * kHMax;                               // F_pad
  float* s_hm = s_fin + p.F_pad;                                      // kHMax
  float* s_hs = s_hm + kHMax;                                         // kHMax
  // stream buffers, one per warp, 16-byte aligned
  Win* s_win = reinterpret_cast<Win*>(
      reinterpret_cast<char*>(smem) + ((agg_smem_floats(p.F_pad, p.HS) * 4 + 15) & ~15));
  __shared__ int s_item;

  int32_t* s_col = s_col_all + warp * 32;
  float* s_p = s_p_all + warp * 32 * p.HS;
  float* s_row = s_row_all + warp * p.F_pad;
  const bool softmax = p.mode != MODE_GCN;

  int hv[NV];
  bool head_start[NV];  // this lane's vector v begins head hv[v]
  {
    const int lig = lane % LPG;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int e0 = (v * LPG + lig) * VEC;
      hv[v] = softmax ? min(e0 / p.C, p.H - 1) : 0;
      head_start[v] = softmax && lane < LPG && e0 < p.F && (e0 % p.C) == 0;
    }
  }

  // ---- Phase 1: CTA items (long rows and segments of split rows) ----
  for (;;) {
    if (threadIdx.x == 0) s_item = atomicAdd(p.counters + 0, 1);
    __syncthreads();
    const int it = s_item;
    if (it >= p.n_cta_items) break;
    const int4 item = p.cta_items[it];
    const int64_t row = item.x;
    const int eb = int(max(int64_t(item.y), p.e_lo)), ee = int(min(int64_t(item.z), p.e_hi));
    const int slot = item.w;
    const int len = ee - eb;
    const int sub = ((len + kWarps - 1) / kWarps + 31) & ~31;
    const int wb = min(ee, eb + warp * sub), we = min(ee, wb + sub);
    float acc[NV][VEC], s_acc[NV], one[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      s_acc[v] = 0.f;
      one[v] = 1.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[v][e] = 0.f;
    }
    float m_reg = -INFINITY;
    if constexpr (STREAM) {
      if (wb < we) {
        using S = AggStream<(KH >= 0 ? KH : 0)>;
        const float ad_reg =
            (KH > 0 && lane < KH) ? __ldg(p.adst + size_t(row) * (KH > 0 ? KH : 1) + lane) : 0.f;
        typename S::Cursor c;
        S::begin(p, s_win[warp], c, wb, we, lane);
        S::row(p, s_win[warp], c, wb, we, ad_reg, acc[0], s_acc[0], m_reg, s_col, s_p, hv[0],
               lane);
        cp_async_wait_all();  // nothing left landing in the buffers
        __syncwarp();
      }
    } else {
      L::range(p, row, wb, we, acc, s_acc, m_reg, s_col, s_p, hv, lane);
    }
    A::group_reduce(acc, s_acc);
    A::spill(p, acc, one, s_row, lane);
    if (lane < kHMax) s_wm[warp * kHMax + lane] = m_reg;
#pragma unroll
    for (int v = 0; v < NV; ++v)
      if (head_start[v]) s_ws[warp * kHMax + hv[v]] = s_acc[v];
    __syncthreads();
    if (softmax && threadIdx.x < p.H) {
      const int hd = threadIdx.x;
      float M = -INFINITY;
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_wm[w * kHMax + hd]);
      float S = 0.f;
      for (int w = 0; w < kWarps; ++w) S += s_ws[w * kHMax + hd] * expf(s_wm[w * kHMax + hd] - M);
      s_hm[hd] = M;
      s_hs[hd] = S;
    }
    __syncthreads();
    float* dst = slot >= 0 ? p.partials + size_t(slot) * p.part_stride : nullptr;
    for (int c = threadIdx.x; c < p.F; c += kThreads) {
      float a = 0.f;
      if (softmax) {
        const int hd = c / p.C;
        const float M = s_hm[hd];
        for (int w = 0; w < kWarps; ++w)
          a += s_row_all[w * p.F_pad + c] * expf(s_wm[w * kHMax + hd] - M);
      } else {
        for (int w = 0; w < kWarps; ++w) a += s_row_all[w * p.F_pad + c];
      }
      if (dst) {
        dst[2 * kHMax + c] = a;
      } else {
        s_fin[c] = softmax ? a / (s_hs[c / p.C] + p.eps) : a;
      }
    }
    if (dst && threadIdx.x < kHMax) {
      dst[threadIdx.x] = softmax ? s_hm[threadIdx.x] : 0.f;
      dst[kHMax + threadIdx.x] = softmax ? s_hs[threadIdx.x] : 0.f;
    }
    __syncthreads();
    if (!dst && warp == 0) warp_epilogue(p, row, s_fin, lane);
    __syncthreads();
  }

  // ---- Phase 2: one warp per short row, edge-balanced row ranges ----
  if constexpr (STREAM) {
    stream_tasks<(KH >= 0 ? KH : 0)>(p, s_win[warp], s_col, s_p, s_row, hv[0], lane);
  } else {
    warp_rows<TH, VEC, LPG, NV, KH>(p, s_col, s_p, s_row, hv, lane);
  }
}


// Combines the partial (max, sum, acc) slots of every split row in slot order.
__global__ void __launch_bounds__(kThreads) merge_kernel(const AggParams p) {
  extern __shared__ float smem[];
  float* s_fin = smem;               // F_pad
  float* s_hm = s_fin + p.F_pad;     // kHMax
  float* s_hs = s_hm + kHMax;        // kHMax
  const int4 sr = p.split_rows[blockIdx.x];
  const int64_t row = sr.x;
  const int first = sr.y, ns = sr.z;
  const bool softmax = p.mode != MODE_GCN;
  if (softmax && threadIdx.x < p.H) {
    const int hd = threadIdx.x;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, p.partials[size_t(first + s) * p.part_stride + hd]);
    float S = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float* q = p.partials + size_t(first + s) * p.part_stride;
      S += q[kHMax + hd] * expf(q[hd] - M);
    }
    s_hm[hd] = M;
    s_hs[hd] = S;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < p.F; c += kThreads) {
    float a = 0.f;
    if (softmax) {
      const int hd = c / p.C;
      for (int s = 0; s < ns; ++s) {
        const float* q = p.partials + size_t(first + s) * p.part_stride;
        a += q[2 * kHMax + c] * expf(q[hd] - s_hm[hd]);
      }
      a = a / (s_hs[hd] + p.eps);
    } else {
      for (int s = 0; s < ns; ++s) a += p.partials[size_t(first + s) * p.part_stride + 2 * kHMax + c];
    }
    s_fin[c] = a;
  }
  __syncthreads();
  if (threadIdx.x < 32) warp_epilogue(p, row, s_fin, threadIdx.x);
}

using KernelFn = void (*)(const AggParams);

template <typename TH, int VEC>
KernelFn pick_layout(int lpg, int nv) {
  if (nv == 1) {
    switch (lpg) {
      case 1: return agg_kernel<TH, VEC, 1, 1>;
      case 2: return agg_kernel<TH, VEC, 2, 1>;
      case 4: return agg_kernel<TH, VEC, 4, 1>;
      case 8: return agg_kernel<TH, VEC, 8, 1>;
      case 16: return agg_kernel<TH, VEC, 16, 1>;
      case 32: return agg_kernel<TH, VEC, 32, 1>;
    }
  } else if (lpg == 32) {
    switch (nv) {
      case 2: return agg_kernel<TH, VEC, 32, 2>;
      case 4: return agg_kernel<TH, VEC, 32, 4>;
      case 8: return agg_kernel<TH, VEC, 32, 8>;
    }
  }
  return nullptr;
}

// The register epilogue stores VEC outputs per lane with one vector store and
// reads bias as float4s: it needs concatenated heads, no log_softmax, and
// out / ldo / bias aligned for those accesses.
bool fast_epilogue_ok(const AggParams& p, int vec) {
  if (!p.concat || p.log_softmax) return false;
  const uintptr_t o = reinterpret_cast<uintptr_t>(p.out);
  const size_t osz = p.out_dtype == GNNC_BF16 ? 2 : 4;
  const size_t vbytes = osz * size_t(vec);
  const size_t need = vbytes >= 16 ? 16 : vbytes;  // store width per instruction
  if (vec > 1 && (o % need != 0 || (size_t(p.ldo) * osz) % need != 0)) return false;
  if (vec % 4 == 0 && p.bias && reinterpret_cast<uintptr_t>(p.bias) % 16 != 0) return false;
  return true;
}

// Softmax probabilities are staged as s_p[edge * HS + head]; an odd stride
// keeps the per-lane stores and the per-head loads free of bank conflicts.
int head_stride(int mode, int H) { return mode == MODE_GCN ? 1 : (H | 1); }

// stream_kh: the head count of a stream kernel (its per-warp buffers), -1 for none.
size_t agg_smem_bytes(int F_pad, int HS, int stream_kh = -1) {
  size_t b = sizeof(float) * size_t(agg_smem_floats(F_pad, HS));
  if (stream_kh < 0) return b;
  size_t win = 0;
  switch (stream_kh) {
    case 0: win = sizeof(AggStream<0>::Win); break;
    case 1: win = sizeof(AggStream<1>::Win); break;
    case 2: win = sizeof(AggStream<2>::Win); break;
    case 4: win = sizeof(AggStream<4>::Win); break;
    default: win = sizeof(AggStream<8>::Win); break;
  }
  return gnnc::align_up(b, 16) + size_t(kWarps) * win;
}

int part_stride_floats(int F) { return int(gnnc::align_up(size_t(2 * kHMax + F), 4)); }

// Lanes per edge group and vectors per lane for feature width F at vector width vec.
void row_layout(int F, int vec, int* lpg_out, int* nv_out) {
  const int lanes = (F + vec - 1) / vec;
  int lpg = 1;
  while (lpg < lanes && lpg < 32) lpg <<= 1;
  int nv = (lanes + 31) / 32;
  if (nv > 1) nv = nv <= 2 ? 2 : (nv <= 4 ? 4 : (nv <= 8 ? 8 : 16));
  *lpg_out = lpg;
  *nv_out = nv;
}

int padded_width(int F, int vec) {
  int lpg, nv;
  row_layout(F, vec, &lpg, &nv);
  return int(gnnc::align_up(size_t(lpg * vec * nv), 4));
}

struct Launch {
  const gnnc_plan_t* plan;
  const void* h;
  int h_dtype;
  int64_t ldh;
};

// The aggregation kernel for a layout: the specialised edge loops where they
// apply (compile-time head counts for 256-wide bf16 / fp32 rows and narrow
// bf16 rows), the generic template otherwise; nullptr if there is none.
KernelFn choose_kernel(const AggParams& p, int h_dtype, int vec, int lpg, int nv,
                       int* stream_kh = nullptr) {
  KernelFn fn = nullptr;
  if (stream_kh) *stream_kh = -1;
  if (h_dtype == GNNC_BF16 && vec == 8 && lpg == 8 && nv == 1) {
    // Narrow rows (32 < F <= 64): specialised loop for a compile-time head count.
    switch (p.mode == MODE_GCN ? 0 : p.H) {
      case 0: fn = agg_kernel<__nv_bfloat16, 8, 8, 1, 0>; break;
      case 1: fn = agg_kernel<__nv_bfloat16, 8, 8, 1, 1>; break;
      case 2: fn = agg_kernel<__nv_bfloat16, 8, 8, 1, 2>; break;
      case 4: fn = agg_kernel<__nv_bfloat16, 8, 8, 1, 4>; break;
      case 8: fn = agg_kernel<__nv_bfloat16, 8, 8, 1, 8>; break;
      default: break;
    }
  }
  if (!fn && h_dtype == GNNC_F32 && vec == 4 && p.F == 256) {
    // fp32 rows of 256: specialised loop for a compile-time head count
    switch (p.mode == MODE_GCN ? 0 : p.H) {
      case 0: fn = agg_kernel<float, 4, 32, 2, 0>; break;
      case 1: fn = agg_kernel<float, 4, 32, 2, 1>; break;
      case 2: fn = agg_kernel<float, 4, 32, 2, 2>; break;
      case 4: fn = agg_kernel<float, 4, 32, 2, 4>; break;
      case 8: fn = agg_kernel<float, 4, 32, 2, 8>; break;
      default: break;
    }
  }
  if (!fn && h_dtype == GNNC_BF16 && vec == 8 && p.F == 256 && p.mode != MODE_SCORES) {
    // The prefetched edge stream: a_src / a_dst rows are copied whole
    // (4, 8 or 16-byte cp.async), so both tables must be aligned to that.
    const int kh = p.mode == MODE_GCN ? 0 : p.H;
    const size_t row_align = kh == 1 ? 4 : (kh == 2 ? 8 : 16);
    const bool ok = kh == 0 || (reinterpret_cast<uintptr_t>(p.asrc) % row_align == 0 &&
                                reinterpret_cast<uintptr_t>(p.adst) % row_align == 0);
    switch (ok ? kh : -1) {
      case 0: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 0, true>; break;
      case 1: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 1, true>; break;
      case 2: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 2, true>; break;
      case 4: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 4, true>; break;
      case 8: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 8, true>; break;
      default: break;
    }
    if (fn && stream_kh) *stream_kh = kh;
  }
  if (!fn && h_dtype == GNNC_BF16 && vec == 8 && p.F == 256) {
    // Specialised edge loop for a compile-time head count. It reads a_src
    // rows (or score rows) as one vector: they must be aligned to it.
    const int kh = p.mode == MODE_GCN ? 0 : p.H;
    const uintptr_t xs = reinterpret_cast<uintptr_t>(p.mode == MODE_GAT ? p.asrc : p.scores);
    const bool xs_ok = kh == 4 ? xs % 16 == 0 : (kh == 2 ? xs % 8 == 0 : true);
    switch (xs_ok ? kh : -1) {
      case 0: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 0>; break;
      case 1: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 1>; break;
      case 2: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 2>; break;
      case 4: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 4>; break;
      case 8: fn = agg_kernel<__nv_bfloat16, 8, 32, 1, 8>; break;
      default: break;
    }
  }
  if (fn) return fn;
  if (h_dtype == GNNC_BF16)
    return vec == 8 ? pick_layout<__nv_bfloat16, 8>(lpg, nv) : pick_layout<__nv_bfloat16, 1>(lpg, nv);
  return vec == 4 ? pick_layout<float, 4>(lpg, nv) : pick_layout<float, 1>(lpg, nv);
}

int run_aggregate(gnnc_ctx_t* ctx, const Launch& L, AggParams p) {
  const gnnc_plan_t* plan = L.plan;
  // Vector width: 16-byte loads when the row stride, base pointer and (for
  // multi-head softmax) the head width allow it; scalar loads otherwise.
  const int vmax = L.h_dtype == GNNC_BF16 ? 8 : 4;
  const bool heads_ok = (p.mode == MODE_GCN) || p.H == 1 || (p.C % vmax == 0);
  const bool align_ok = (reinterpret_cast<uintptr_t>(L.h) % 16 == 0) && (L.ldh % vmax == 0);
  const int vec = (heads_ok && align_ok) ? vmax : 1;
  int lpg, nv;
  row_layout(p.F, vec, &lpg, &nv);
  if (nv > 8)
    return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED,
                           "feature width %d too large for the row kernel (vector width %d)", p.F,
                           vec);
  int stream_kh = -1;
  KernelFn fn = choose_kernel(p, L.h_dtype, vec, lpg, nv, &stream_kh);
  if (!fn) return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED, "no kernel for layout");

  p.F_pad = int(gnnc::align_up(size_t(lpg * vec * nv), 4));
  p.HS = head_stride(p.mode, p.H);
  p.fast_epilogue = fast_epilogue_ok(p, vec);
  p.part_stride = part_stride_floats(p.F_pad);
  p.cta_items = plan->cta_items;
  const bool wide = lpg == 32;  // a whole warp per edge
  p.n_cta_items = wide ? plan->n_cta_items_wide : plan->n_cta_items;
  p.split_rows = plan->split_rows;
  p.warp_tasks = plan->warp_tasks;
  p.n_warp_tasks = plan->n_warp_tasks;
  p.stream_tasks = plan->stream_tasks;
  p.n_stream_tasks = plan->n_stream_tasks;
  p.cta_threshold = wide ? plan->wide_threshold : plan->cta_threshold;
  p.counters = ctx->dev_words;
  p.partials = nullptr;
  if (plan->n_segments > 0) {
    const size_t need = size_t(plan->n_segments) * p.part_stride * sizeof(float);
    int st = gnnc::ensure_workspace(ctx, need);
    if (st) return st;
    p.partials = reinterpret_cast<float*>(ctx->ws);
  }
  const size_t smem = agg_smem_bytes(p.F_pad, p.HS, stream_kh);
  if (smem > 48 * 1024)
    GNNC_CUDA_TRY(ctx, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(smem)));
  int per_sm = 0;
  GNNC_CUDA_TRY(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem));
  if (per_sm < 1) per_sm = 1;
  const int grid = ctx->num_sms * per_sm;
  GNNC_CUDA_TRY(ctx, cudaMemsetAsync(ctx->dev_words, 0, 2 * sizeof(int), ctx->stream));
  fn<<<grid, kThreads, smem, ctx->stream>>>(p);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  if (plan->n_split_rows > 0) {
    const size_t msmem = sizeof(float) * (p.F_pad + 2 * kHMax);
    merge_kernel<<<unsigned(plan->n_split_rows), kThreads, msmem, ctx->stream>>>(p);
    GNNC_CUDA_TRY(ctx, cudaGetLastError());
  }
  return GNNC_OK;
}

int check_common(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, const int32_t* rowptr,
                 const int32_t* col, const void* h, int h_dtype, int64_t ldh, int64_t n_rows,
                 int64_t n_src, int64_t F, int act, void* out, int out_dtype, int64_t ldo,
                 int64_t F_out) {
  GNNC_CHECK_ARG(ctx, plan != nullptr, "plan is null");
  GNNC_CHECK_ARG(ctx, plan->n_rows == n_rows, "plan was built for %lld rows, call has %lld",
                 (long long)plan->n_rows, (long long)n_rows);
  GNNC_CHECK_ARG(ctx, plan->device == ctx->device, "plan belongs to another device");
  GNNC_CHECK_ARG(ctx, n_rows >= 0 && n_src >= 0 && F > 0, "bad sizes");
  GNNC_CHECK_ARG(ctx, n_rows == 0 || (rowptr && out), "null rowptr/out");
  GNNC_CHECK_ARG(ctx, h != nullptr || n_src == 0, "null h");
  GNNC_CHECK_ARG(ctx, h_dtype == GNNC_F32 || h_dtype == GNNC_BF16, "bad h dtype");
  GNNC_CHECK_ARG(ctx, out_dtype == GNNC_F32 || out_dtype == GNNC_BF16, "bad out dtype");
  GNNC_CHECK_ARG(ctx, act >= GNNC_ACT_NONE && act <= GNNC_ACT_ELU, "bad activation");
  GNNC_CHECK_ARG(ctx, ldh >= F, "ldh (%lld) < F (%lld)", (long long)ldh, (long long)F);
  GNNC_CHECK_ARG(ctx, ldo >= F_out, "ldo (%lld) < F_out (%lld)", (long long)ldo,
                 (long long)F_out);
  GNNC_CHECK_ARG(ctx, n_src < (int64_t(1) << 31), "n_src exceeds int32 indexing");
  (void)col;
  return GNNC_OK;
}

AggParams base_params(const gnnc_plan_t* plan) {
  AggParams p{};
  p.e_lo = plan->e_begin;
  p.e_hi = plan->e_end;
  return p;
}

}  // namespace

// ---------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------

extern "C" int gnnc_plan_create(gnnc_ctx_t* ctx, const int32_t* rowptr, int64_t n_rows,
                                int32_t cta_threshold, int32_t split_threshold,
                                gnnc_plan_t** out_plan) {
  if (!ctx || !out_plan) return GNNC_ERR_INVALID;
  *out_plan = nullptr;
  GNNC_CHECK_ARG(ctx, n_rows >= 0 && n_rows < (int64_t(1) << 31), "bad n_rows");
  GNNC_CHECK_ARG(ctx, rowptr != nullptr, "null rowptr");
  const bool default_cta = cta_threshold <= 0;
  const bool default_split = split_threshold <= 0;
  if (cta_threshold <= 0) cta_threshold = 256;
  if (split_threshold <= 0) split_threshold = 4096;
  GNNC_CHECK_ARG(ctx, split_threshold >= cta_threshold, "split_threshold < cta_threshold");
  // With the default thresholds, launches on wide rows (256 features: a whole
  // warp per edge) give rows of up to 1024 edges to the warp path, which is
  // faster there than the CTA path (measured on the c4 graph); narrow rows
  // keep the CTA path from 257 edges up.
  const int wide_threshold =
      default_cta ? std::min(1024, split_threshold) : cta_threshold;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  std::vector<int32_t> rp(size_t(n_rows) + 1);
  GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(rp.data(), rowptr, rp.size() * sizeof(int32_t),
                                     cudaMemcpyDeviceToHost, ctx->stream));
  GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  if (rp[0] < 0)
    return gnnc::set_error(ctx, GNNC_ERR_BOUNDS, "rowptr[0] = %d is negative", rp[0]);
  for (int64_t r = 0; r < n_rows; ++r)
    if (rp[r + 1] < rp[r])
      return gnnc::set_error(ctx, GNNC_ERR_BOUNDS, "rowptr decreases at row %lld",
                             (long long)r);

  if (default_split) {
    // Split a row across CTAs only when one CTA alone would take a sizeable
    // share of the launch: longer than the edges per resident CTA over two
    // (at least 4096). Splitting costs partials and a merge launch; on the c4
    // graph (max degree 6,853) no row needs it, on the scale-24 R-MAT graph
    // the hub rows of ~370k edges do.
    const int64_t per = (int64_t(rp[size_t(n_rows)]) - rp[0]) / (2 * int64_t(ctx->num_sms) * 4);
    split_threshold = int(std::min<int64_t>(std::max<int64_t>(4096, per), int64_t(1) << 30));
  }
  std::vector<int4> items, splits;
  std::vector<int32_t> tasks;
  int64_t n_warp = 0, n_cta = 0, n_seg = 0;
  int max_deg = 0;
  // Warp tasks: contiguous row ranges of roughly equal cost (edges + a fixed
  // per-row overhead); rows taken by the CTA path cost one unit. A task costs
  // 768 units, or less on small launches (a rank's share of a partitioned
  // graph) so that every resident warp gets about eight tasks and the last
  // ones finish together.
  const int64_t kRowCost = 6;
  const int64_t total_cost = (int64_t(rp[size_t(n_rows)]) - rp[0]) + kRowCost * n_rows;
  const int64_t kTaskCost = std::min<int64_t>(
      768, std::max<int64_t>(192, total_cost / (int64_t(ctx->num_sms) * 32 * 8)));
  int64_t cost = 0;
  tasks.push_back(0);
  for (int64_t r = 0; r < n_rows; ++r) {
    const int deg = rp[r + 1] - rp[r];
    max_deg = std::max(max_deg, deg);
    if (deg > split_threshold) {
      const int ns = (deg + split_threshold - 1) / split_threshold;
      splits.push_back(make_int4(int(r), int(n_seg), ns, 0));
      for (int s = 0; s < ns; ++s) {
        const int eb = rp[r] + s * split_threshold;
        const int ee = std::min(rp[r + 1], eb + split_threshold);
        items.push_back(make_int4(int(r), eb, ee, int(n_seg + s)));
      }
      n_seg += ns;
      cost += 1;
    } else if (deg > cta_threshold) {
      items.push_back(make_int4(int(r), rp[r], rp[r + 1], -1));
      ++n_cta;
      cost += deg <= wide_threshold ? deg + kRowCost : 1;
    } else {
      ++n_warp;
      cost += deg + kRowCost;
    }
    if (cost >= kTaskCost) {
      tasks.push_back(int32_t(r + 1));
      cost = 0;
    }
  }
  if (tasks.back() != n_rows) tasks.push_back(int32_t(n_rows));
  // Stream tasks (wide launches with the prefetched edge stream): runs of
  // consecutive rows that the wide launches give to warps, cut at every row
  // they leave to the CTA path, so each task's edges are contiguous.
  std::vector<int2> stasks;
  {
    int64_t c = 0;
    int64_t start = -1;
    for (int64_t r = 0; r < n_rows; ++r) {
      const int deg = rp[r + 1] - rp[r];
      if (deg > wide_threshold) {
        if (start >= 0) stasks.push_back(make_int2(int(start), int(r)));
        start = -1;
        c = 0;
        continue;
      }
      if (start < 0) start = r;
      c += deg + kRowCost;
      if (c >= kTaskCost) {
        stasks.push_back(make_int2(int(start), int(r + 1)));
        start = -1;
        c = 0;
      }
    }
    if (start >= 0) stasks.push_back(make_int2(int(start), int(n_rows)));
  }
  // Largest CTA items first, so the long ones do not form the tail; whole
  // rows the wide launches leave to warps go last.
  auto warp_on_wide = [&](const int4& it) { return it.w < 0 && it.z - it.y <= wide_threshold; };
  std::stable_sort(items.begin(), items.end(), [&](const int4& a, const int4& b) {
    const bool wa = warp_on_wide(a), wb = warp_on_wide(b);
    if (wa != wb) return wb;
    return (a.z - a.y) > (b.z - b.y);
  });
  int64_t n_items_wide = 0;
  for (const int4& it : items) n_items_wide += warp_on_wide(it) ? 0 : 1;

  gnnc_plan_t* plan = new gnnc_plan_t();
  plan->n_rows = n_rows;
  plan->cta_threshold = cta_threshold;
  plan->split_threshold = split_threshold;
  plan->n_warp_rows = n_warp;
  plan->n_cta_rows = n_cta;
  plan->n_split_rows = int64_t(splits.size());
  plan->n_segments = n_seg;
  plan->n_cta_items = int64_t(items.size());
  plan->wide_threshold = wide_threshold;
  plan->n_cta_items_wide = n_items_wide;
  plan->n_warp_tasks = int64_t(tasks.size()) - 1;
  plan->n_stream_tasks = int64_t(stasks.size());
  plan->max_degree = max_deg;
  plan->device = ctx->device;
  plan->e_begin = rp[0];
  plan->e_end = rp[size_t(n_rows)];
  auto upload = [&](void** dst, const void* src, size_t bytes) -> cudaError_t {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(dst, bytes);
    if (e != cudaSuccess) return e;
    if (src) return cudaMemcpyAsync(*dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
    return cudaSuccess;
  };
  cudaError_t e = upload(reinterpret_cast<void**>(&plan->cta_items),
                         items.empty() ? nullptr : items.data(), items.size() * sizeof(int4));
  if (e == cudaSuccess)
    e = upload(reinterpret_cast<void**>(&plan->split_rows),
               splits.empty() ? nullptr : splits.data(), splits.size() * sizeof(int4));
  if (e == cudaSuccess)
    e = upload(reinterpret_cast<void**>(&plan->warp_tasks), tasks.data(),
               tasks.size() * sizeof(int32_t));
  if (e == cudaSuccess)
    e = upload(reinterpret_cast<void**>(&plan->stream_tasks),
               stasks.empty() ? nullptr : stasks.data(), stasks.size() * sizeof(int2));
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    gnnc_plan_destroy(plan);
    return gnnc::cuda_status(ctx, e, "plan upload");
  }
  *out_plan = plan;
  return GNNC_OK;
}

extern "C" int gnnc_plan_destroy(gnnc_plan_t* plan) {
  if (!plan) return GNNC_OK;
  cudaSetDevice(plan->device);
  if (plan->cta_items) cudaFree(plan->cta_items);
  if (plan->split_rows) cudaFree(plan->split_rows);
  if (plan->warp_tasks) cudaFree(plan->warp_tasks);
  if (plan->stream_tasks) cudaFree(plan->stream_tasks);
  delete plan;
  return GNNC_OK;
}

extern "C" int gnnc_plan_info(const gnnc_plan_t* plan, int64_t* info) {
  if (!plan || !info) return GNNC_ERR_INVALID;
  info[0] = plan->n_rows;
  info[1] = plan->n_warp_rows;
  info[2] = plan->n_cta_rows;
  info[3] = plan->n_split_rows;
  info[4] = plan->n_segments;
  info[5] = plan->max_degree;
  return GNNC_OK;
}

extern "C" int gnnc_workspace_query(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, int64_t F,
                                    size_t* bytes) {
  if (!ctx || !plan || !bytes || F <= 0) return GNNC_ERR_INVALID;
  const int F_pad = std::max(padded_width(int(F), 1), std::max(padded_width(int(F), 4),
                                                                padded_width(int(F), 8)));
  *bytes = size_t(plan->n_segments) * part_stride_floats(F_pad) * sizeof(float);
  return GNNC_OK;
}

// ---------------------------------------------------------------------------
// Aggregation entry points
// ---------------------------------------------------------------------------

extern "C" int gnnc_gcn_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan,
                                  const int32_t* rowptr, const int32_t* col, const float* w,
                                  const void* h, int h_dtype, int64_t ldh, int64_t n_rows,
                                  int64_t n_src, int64_t F, const float* bias, int act,
                                  int log_softmax, void* out, int out_dtype, int64_t ldo) {
  if (!ctx) return GNNC_ERR_INVALID;
  int st = check_common(ctx, plan, rowptr, col, h, h_dtype, ldh, n_rows, n_src, F, act, out,
                        out_dtype, ldo, F);
  if (st) return st;
  if (n_rows == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  AggParams p = base_params(plan);
  p.rowptr = rowptr; p.col = col; p.w = w; p.h = h; p.ldh = ldh;
  p.n_rows = n_rows; p.n_src = n_src;
  p.H = 1; p.C = int(F); p.F = int(F); p.F_out = int(F);
  p.mode = MODE_GCN; p.concat = 1; p.act = act; p.log_softmax = log_softmax;
  p.bias = bias; p.out = out; p.out_dtype = out_dtype; p.ldo = ldo; p.eps = 0.f;
  return run_aggregate(ctx, Launch{plan, h, h_dtype, ldh}, p);
}

extern "C" int gnnc_sage_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan,
                                   const int32_t* rowptr, const int32_t* col, const float* w,
                                   const void* h, int h_dtype, int64_t ldh, const void* root,
                                   int root_dtype, int64_t ldr, int64_t n_rows, int64_t n_src,
                                   int64_t F, const float* bias, int act, int log_softmax,
                                   void* out, int out_dtype, int64_t ldo) {
  if (!ctx) return GNNC_ERR_INVALID;
  int st = check_common(ctx, plan, rowptr, col, h, h_dtype, ldh, n_rows, n_src, F, act, out,
                        out_dtype, ldo, F);
  if (st) return st;
  GNNC_CHECK_ARG(ctx, root != nullptr || n_rows == 0, "null root");
  GNNC_CHECK_ARG(ctx, root_dtype == GNNC_F32 || root_dtype == GNNC_BF16, "bad root dtype");
  GNNC_CHECK_ARG(ctx, ldr >= F, "ldr (%lld) < F (%lld)", (long long)ldr, (long long)F);
  if (n_rows == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  AggParams p = base_params(plan);
  p.rowptr = rowptr; p.col = col; p.w = w; p.h = h; p.ldh = ldh;
  p.n_rows = n_rows; p.n_src = n_src;
  p.H = 1; p.C = int(F); p.F = int(F); p.F_out = int(F);
  p.mode = MODE_GCN; p.concat = 1; p.act = act; p.log_softmax = log_softmax;
  p.bias = bias; p.out = out; p.out_dtype = out_dtype; p.ldo = ldo; p.eps = 0.f;
  p.root = root; p.root_dtype = root_dtype; p.ldr = ldr;
  return run_aggregate(ctx, Launch{plan, h, h_dtype, ldh}, p);
}

static int gat_like(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, int mode, const int32_t* rowptr,
                    const int32_t* col, const float* scores, const void* h, int h_dtype,
                    int64_t ldh, const float* asrc, const float* adst, int64_t n_rows,
                    int64_t n_src, int64_t H, int64_t C, float slope, float eps, int concat,
                    const float* bias, int act, int log_softmax, void* out, int out_dtype,
                    int64_t ldo) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, H >= 1 && C >= 1, "bad heads/channels");
  if (H > kHMax)
    return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED, "at most %d heads supported", kHMax);
  const int64_t F = H * C, F_out = concat ? F : C;
  int st = check_common(ctx, plan, rowptr, col, h, h_dtype, ldh, n_rows, n_src, F, act, out,
                        out_dtype, ldo, F_out);
  if (st) return st;
  if (n_rows == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  AggParams p = base_params(plan);
  p.rowptr = rowptr; p.col = col; p.scores = scores; p.asrc = asrc; p.adst = adst;
  p.h = h; p.ldh = ldh; p.n_rows = n_rows; p.n_src = n_src;
  p.H = int(H); p.C = int(C); p.F = int(F); p.F_out = int(F_out);
  p.mode = mode; p.concat = concat; p.act = act; p.log_softmax = log_softmax;
  p.slope = slope; p.eps = eps; p.bias = bias; p.out = out; p.out_dtype = out_dtype; p.ldo = ldo;
  return run_aggregate(ctx, Launch{plan, h, h_dtype, ldh}, p);
}

extern "C" int gnnc_gat_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan,
                                  const int32_t* rowptr, const int32_t* col, const void* h,
                                  int h_dtype, int64_t ldh, const float* asrc, const float* adst,
                                  int64_t n_rows, int64_t n_src, int64_t H, int64_t C,
                                  float negative_slope, int concat, const float* bias, int act,
                                  int log_softmax, void* out, int out_dtype, int64_t ldo) {
  if (ctx && n_rows > 0 && (!asrc || !adst))
    return gnnc::set_error(ctx, GNNC_ERR_INVALID, "null attention coefficients");
  return gat_like(ctx, plan, MODE_GAT, rowptr, col, nullptr, h, h_dtype, ldh, asrc, adst, n_rows,
                  n_src, H, C, negative_slope, 1e-16f, concat, bias, act, log_softmax, out,
                  out_dtype, ldo);
}

extern "C" int gnnc_softmax_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan,
                                      const int32_t* rowptr, const int32_t* col, const float* s,
                                      const void* h, int h_dtype, int64_t ldh, int64_t n_rows,
                                      int64_t n_src, int64_t H, int64_t C, float eps, int concat,
                                      const float* bias, int act, int log_softmax, void* out,
                                      int out_dtype, int64_t ldo) {
  if (ctx && n_rows > 0 && !s) return gnnc::set_error(ctx, GNNC_ERR_INVALID, "null scores");
  return gat_like(ctx, plan, MODE_SCORES, rowptr, col, s, h, h_dtype, ldh, nullptr, nullptr,
                  n_rows, n_src, H, C, 0.f, eps, concat, bias, act, log_softmax, out, out_dtype,
                  ldo);
}

// ---------------------------------------------------------------------------
// GAT aggregation that allocates nothing
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory while a layer runs: a serving
// process that reserves its whole memory budget at start-up (a cudaMalloc in
// the middle of a request can fail because the device is already full, and
// cudaMalloc / cudaFree synchronise the device), or a host runtime that owns
// all device memory through its own pool and forbids libraries from
// allocating behind its back. gnnc_gat_aggregate may grow the context
// workspace with cudaMalloc when a plan needs more split-row partials than it
// has seen before; gnnc_gat_aggregate_noalloc never allocates. Its scratch -
// the scheduling counters, the bad-index flag and the split-row partials -
// lives in the fixed array below, which every GPU that loads this library
// holds until the process exits. gnnc_init looks up the array's device
// address for its context (with lazy module loading that lookup is what loads
// this library's device code on the device and reserves the array), so no
// call of the entry point itself allocates.

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr size_t kStaticCounterBytes = 256;               // counters first, partials after

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// ORs the call's bad-index flag into the context's flag word, which
// gnnc_synchronize reports.
__global__ void fold_flag_kernel(const int* from, int* into) {
  if (*from) atomicOr(into, 1);
}

}  // namespace

namespace gnnc {

cudaError_t resolve_static_scratch(gnnc_ctx_t* ctx) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  ctx->static_scratch = e == cudaSuccess ? p : nullptr;
  return e;
}

}  // namespace gnnc

extern "C" int gnnc_gat_aggregate_noalloc(gnnc_ctx_t* ctx, const gnnc_plan_t* plan,
                                          const int32_t* rowptr, const int32_t* col,
                                          const void* h, int h_dtype, int64_t ldh,
                                          const float* asrc, const float* adst, int64_t n_rows,
                                          int64_t n_src, int64_t H, int64_t C,
                                          float negative_slope, int concat, const float* bias,
                                          int act, int log_softmax, void* out, int out_dtype,
                                          int64_t ldo) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, H >= 1 && C >= 1, "bad heads/channels");
  if (H > kHMax)
    return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED, "at most %d heads supported", kHMax);
  const int64_t F = H * C, F_out = concat ? F : C;
  int st = check_common(ctx, plan, rowptr, col, h, h_dtype, ldh, n_rows, n_src, F, act, out,
                        out_dtype, ldo, F_out);
  if (st) return st;
  if (n_rows == 0) return GNNC_OK;
  GNNC_CHECK_ARG(ctx, asrc && adst, "null attention coefficients");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  // The array's device address, looked up once by gnnc_init. In host code the
  // name g_static_scratch is only a host-side stand-in, never passed to a kernel.
  unsigned char* scratch = reinterpret_cast<unsigned char*>(ctx->static_scratch);
  if (!scratch)
    return gnnc::set_error(ctx, GNNC_ERR_CUDA, "fixed scratch address was not resolved");

  AggParams p = base_params(plan);
  p.rowptr = rowptr; p.col = col; p.scores = nullptr; p.asrc = asrc; p.adst = adst;
  p.h = h; p.ldh = ldh; p.n_rows = n_rows; p.n_src = n_src;
  p.H = int(H); p.C = int(C); p.F = int(F); p.F_out = int(F_out);
  p.mode = MODE_GAT; p.concat = concat; p.act = act; p.log_softmax = log_softmax;
  p.slope = negative_slope; p.eps = 1e-16f; p.bias = bias; p.out = out; p.out_dtype = out_dtype;
  p.ldo = ldo;

  // Same kernel choice as gnnc_gat_aggregate (choose_kernel).
  const int vmax = h_dtype == GNNC_BF16 ? 8 : 4;
  const bool heads_ok = p.H == 1 || (p.C % vmax == 0);
  const bool align_ok = (reinterpret_cast<uintptr_t>(h) % 16 == 0) && (ldh % vmax == 0);
  const int vec = (heads_ok && align_ok) ? vmax : 1;
  int lpg, nv;
  row_layout(p.F, vec, &lpg, &nv);
  if (nv > 8)
    return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED,
                           "feature width %d too large for the row kernel (vector width %d)", p.F,
                           vec);
  int stream_kh = -1;
  KernelFn fn = choose_kernel(p, h_dtype, vec, lpg, nv, &stream_kh);
  if (!fn) return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED, "no kernel for layout");
  p.F_pad = int(gnnc::align_up(size_t(lpg * vec * nv), 4));
  p.HS = head_stride(p.mode, p.H);
  p.fast_epilogue = fast_epilogue_ok(p, vec);
  p.part_stride = part_stride_floats(p.F_pad);
  p.cta_items = plan->cta_items;
  const bool wide = lpg == 32;  // a whole warp per edge
  p.n_cta_items = wide ? plan->n_cta_items_wide : plan->n_cta_items;
  p.split_rows = plan->split_rows;
  p.warp_tasks = plan->warp_tasks;
  p.n_warp_tasks = plan->n_warp_tasks;
  p.stream_tasks = plan->stream_tasks;
  p.n_stream_tasks = plan->n_stream_tasks;
  p.cta_threshold = wide ? plan->wide_threshold : plan->cta_threshold;

  const size_t need = size_t(plan->n_segments) * p.part_stride * sizeof(float);
  if (need > kStaticScratchBytes - kStaticCounterBytes)
    return gnnc::set_error(ctx, GNNC_ERR_UNSUPPORTED,
                           "this plan's %lld split-row segments need %zu bytes of scratch; the "
                           "fixed scratch holds %zu (raise split_threshold or use "
                           "gnnc_gat_aggregate)",
                           (long long)plan->n_segments, need,
                           kStaticScratchBytes - kStaticCounterBytes);
  p.counters = reinterpret_cast<int*>(scratch);
  p.partials = reinterpret_cast<float*>(scratch + kStaticCounterBytes);

  const size_t smem = agg_smem_bytes(p.F_pad, p.HS, stream_kh);
  if (smem > 48 * 1024)
    GNNC_CUDA_TRY(ctx, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(smem)));
  int per_sm = 0;
  GNNC_CUDA_TRY(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem));
  if (per_sm < 1) per_sm = 1;
  // The array keeps the previous call's contents: the two work counters and
  // the bad-index flag must start at zero. Partials are written before read.
  GNNC_CUDA_TRY(ctx, cudaMemsetAsync(p.counters, 0, 3 * sizeof(int), ctx->stream));
  fn<<<ctx->num_sms * per_sm, kThreads, smem, ctx->stream>>>(p);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  if (plan->n_split_rows > 0) {
    const size_t msmem = sizeof(float) * (p.F_pad + 2 * kHMax);
    merge_kernel<<<unsigned(plan->n_split_rows), kThreads, msmem, ctx->stream>>>(p);
    GNNC_CUDA_TRY(ctx, cudaGetLastError());
  }
  fold_flag_kernel<<<1, 1, 0, ctx->stream>>>(p.counters + 2, ctx->dev_words + 2);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}
