// Dense projection h = x . w^T with GATConv's attention coefficients fused
// into the epilogue (experiments/gatconv/dumps/gat.1-raw-torch.mlir:5-24:
// aten.linear, view [N,H,C], mul by att_src / att_dst, sum over C).
//
// This file holds the CUDA-core path (fp32 FMA, any K, any F, fp32 or bf16
// operands). It is the exact-fp32 path the fp32 configurations need (tensor
// cores would round operands to tf32). The bf16 tensor-core path lives in
// proj_tc.cu and is selected by gnnc_proj when the shapes allow it.
//
// One CTA owns BM rows and walks every column tile of the output, so the
// per-head dot products with att_src / att_dst are summed inside the CTA in a
// fixed order (deterministic, no atomics).
#include "common.cuh"
#include "proj_tc.cuh"

namespace {

constexpr int BM = 64, BN = 64, BK = 16;
constexpr int kThreads = 256;

struct ProjParams {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  int64_t N, K, F;
  int x_bf16;
  const float* att_src;
  const float* att_dst;
  int H, C;
  void* h;
  int h_bf16;
  int64_t ldh;
  float* asrc;
  float* adst;
};

__device__ __forceinline__ float load_elem(const void* base, int bf16, size_t idx) {
  if (bf16) {
    unsigned short v = __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    return __uint_as_float(uint32_t(v) << 16);
  }
  return __ldg(reinterpret_cast<const float*>(base) + idx);
}

__global__ void __launch_bounds__(kThreads) proj_simt_kernel(const ProjParams p) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  __shared__ float Cs[BM][BN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t row0 = int64_t(blockIdx.x) * BM;
  const bool att = p.att_src != nullptr;
  const int n_ct = int((p.F + BN - 1) / BN);

  for (int ct = 0; ct < n_ct; ++ct) {
    const int64_t col0 = int64_t(ct) * BN;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < p.K; k0 += BK) {
      // Stage x[row0:+BM, k0:+BK] and w[col0:+BN, k0:+BK] transposed (k-major).
      for (int i = threadIdx.x; i < BM * BK; i += kThreads) {
        const int r = i / BK, kk = i % BK;
        const int64_t gr = row0 + r, gk = k0 + kk;
        As[kk][r] = (gr < p.N && gk < p.K) ? load_elem(p.x, p.x_bf16, size_t(gr) * p.ldx + gk) : 0.f;
        const int64_t gc = col0 + r;
        Bs[kk][r] = (gc < p.F && gk < p.K) ? load_elem(p.w, p.x_bf16, size_t(gc) * p.ldw + gk) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
    // Store h and stage the fp32 tile for the attention sums.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty + 16 * i;
      const int64_t gr = row0 + r;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = tx + 16 * j;
        const int64_t gc = col0 + c;
        Cs[r][c] = acc[i][j];
        if (gr < p.N && gc < p.F) store_val(p.h, p.h_bf16 ? GNNC_BF16 : GNNC_F32, size_t(gr) * p.ldh + gc, acc[i][j]);
      }
    }
    if (att) {
      __syncthreads();
      // Heads overlapping this column tile: [hd0, hd1].
      const int tile_w = int(p.F - col0 < BN ? p.F - col0 : BN);
      const int hd0 = int(col0 / p.C), hd1 = int((col0 + tile_w - 1) / p.C);
      const int nh = hd1 - hd0 + 1;
      for (int i = threadIdx.x; i < BM * nh; i += kThreads) {
        const int r = i / nh, hh = i % nh, hd = hd0 + hh;
        const int c_lo = int((int64_t(hd) * p.C > col0 ? int64_t(hd) * p.C : col0) - col0);
        const int c_hi = int((int64_t(hd + 1) * p.C < col0 + tile_w ? int64_t(hd + 1) * p.C : col0 + tile_w) - col0);
        float ss = 0.f, sd = 0.f;
        for (int c = c_lo; c < c_hi; ++c) {
          ss = fmaf(Cs[r][c], __ldg(p.att_src + col0 + c), ss);
          sd = fmaf(Cs[r][c], __ldg(p.att_dst + col0 + c), sd);
        }
        const int64_t gr = row0 + r;
        if (gr < p.N) {
          // A head either starts in this tile (write) or continues from the
          // previous tile (accumulate); tiles are visited in column order.
          const bool starts_here = int64_t(hd) * p.C >= col0;
          float* ps = p.asrc + size_t(gr) * p.H + hd;
          float* pd = p.adst + size_t(gr) * p.H + hd;
          if (starts_here) {
            *ps = ss;
            *pd = sd;
          } else {
            *ps += ss;
            *pd += sd;
          }
        }
      }
    }
    __syncthreads();
  }
}

// fp32 operands on the tensor cores. Each value splits into three bf16 parts,
// v0 = bf16(v), v1 = bf16(v - v0), v2 = bf16(v - v0 - v1) (24 significant
// bits together), and x.w = x0.w0 + x0.w1 + x1.w0 + x0.w2 + x1.w1 + x2.w0 up
// to the dropped cross terms, which are below 2^-24 of |x||w|: one bf16 GEMM
// with fp32 accumulation over the six K-blocks [x0 x0 x1 x0 x1 x2] against
// [w0 w1 w0 w2 w1 w0]. This kernel writes the six blocks of one operand
// (pattern 0: x's, pattern 1: w's) for `rows` rows into out (row stride ldo).
__global__ void split3_kernel(const float* __restrict__ in, int64_t ldi, int64_t rows, int64_t K,
                              __nv_bfloat16* __restrict__ out, int64_t ldo, int pattern) {
  const int px[6] = {0, 0, 1, 0, 1, 2};
  const int pw[6] = {0, 1, 0, 2, 1, 0};
  const int64_t total = rows * K;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / K, k = i - r * K;
    const float v = in[r * ldi + k];
    __nv_bfloat16 part[3];
    part[0] = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(part[0]);
    part[1] = __float2bfloat16_rn(r1);
    part[2] = __float2bfloat16_rn(r1 - __bfloat162float(part[1]));
    __nv_bfloat16* o = out + r * ldo + k;
#pragma unroll
    for (int s = 0; s < 6; ++s) o[s * K] = part[pattern ? pw[s] : px[s]];
  }
}

// fp32 x and w through the tcgen05 kernel as a bf16 GEMM over 6K (see
// split3_kernel); kProjTcDeclined when the shapes or sizes do not suit it.
int proj_f32_split3(gnnc_ctx_t* ctx, const float* x, int64_t ldx, const float* w, int64_t ldw,
                    int64_t N, int64_t K, int64_t F, const float* att_src, const float* att_dst,
                    int64_t H, void* h, int h_dtype, int64_t ldh, float* asrc, float* adst) {
  // Worth it once the GEMM has some size; F beyond 256 is not a tcgen05 shape here.
  if (F > 256 || N < 1024 || double(N) * double(K) * double(F) < double(1 << 24))
    return gnnc::kProjTcDeclined;
  // shapes the tcgen05 kernel declines: decide before splitting
  const int hes = h_dtype == GNNC_BF16 ? 2 : 4;
  if (att_src && !(H == 1 || (F / H) % 16 == 0)) return gnnc::kProjTcDeclined;
  if (reinterpret_cast<uintptr_t>(h) % 16 || (ldh * hes) % 16 || F * hes < 16)
    return gnnc::kProjTcDeclined;
  const int64_t K6 = 6 * K;
  const int64_t ld6 = (K6 + 7) / 8 * 8;
  const size_t xb = size_t(N) * size_t(ld6) * 2, wb = size_t(F) * size_t(ld6) * 2;
  if (!ctx->ws_owned && ctx->ws_bytes < xb + wb) return gnnc::kProjTcDeclined;  // bound, too small
  int st = gnnc::ensure_workspace(ctx, xb + wb);
  if (st) return st;
  auto* x6 = reinterpret_cast<__nv_bfloat16*>(ctx->ws);
  auto* w6 = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(ctx->ws) + xb);
  const int threads = 256;
  auto grid_of = [&](int64_t n) {
    const int64_t g = (n + threads - 1) / threads;
    const int64_t cap = int64_t(ctx->num_sms) * 16;
    return unsigned(g < cap ? g : cap);
  };
  split3_kernel<<<grid_of(N * K), threads, 0, ctx->stream>>>(x, ldx, N, K, x6, ld6, 0);
  split3_kernel<<<grid_of(F * K), threads, 0, ctx->stream>>>(w, ldw, F, K, w6, ld6, 1);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return gnnc::proj_tc_try(ctx, x6, ld6, w6, ld6, N, K6, F, att_src, att_dst, H, h, h_dtype, ldh,
                           asrc, adst);
}

}  // namespace

extern "C" int gnnc_proj(gnnc_ctx_t* ctx, const void* x, int x_dtype, int64_t ldx,
                         const void* w, int64_t ldw, int64_t N, int64_t K, int64_t F,
                         const float* att_src, const float* att_dst, int64_t H, void* h,
                         int h_dtype, int64_t ldh, float* asrc, float* adst) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, N >= 0 && K > 0 && F > 0, "bad sizes N=%lld K=%lld F=%lld",
                 (long long)N, (long long)K, (long long)F);
  GNNC_CHECK_ARG(ctx, x_dtype == GNNC_F32 || x_dtype == GNNC_BF16, "bad x dtype");
  GNNC_CHECK_ARG(ctx, h_dtype == GNNC_F32 || h_dtype == GNNC_BF16, "bad h dtype");
  GNNC_CHECK_ARG(ctx, ldx >= K && ldw >= K && ldh >= F, "strides smaller than widths");
  GNNC_CHECK_ARG(ctx, N == 0 || (x && w && h), "null x/w/h");
  const bool att = att_src || att_dst || asrc || adst;
  if (att) {
    GNNC_CHECK_ARG(ctx, att_src && att_dst && asrc && adst,
                   "att_src, att_dst, asrc, adst must all be given or all be null");
    GNNC_CHECK_ARG(ctx, H >= 1 && F % H == 0, "F (%lld) not divisible by H (%lld)",
                   (long long)F, (long long)H);
  }
  if (N == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  // bf16 operands with tensor-core friendly shapes go to tcgen05.
  if (x_dtype == GNNC_BF16) {
    int st = gnnc::proj_tc_try(ctx, x, ldx, w, ldw, N, K, F, att ? att_src : nullptr,
                               att ? att_dst : nullptr, att ? H : 1, h, h_dtype, ldh,
                               att ? asrc : nullptr, att ? adst : nullptr);
    if (st != gnnc::kProjTcDeclined) return st;
  } else {
    int st = proj_f32_split3(ctx, static_cast<const float*>(x), ldx,
                             static_cast<const float*>(w), ldw, N, K, F, att ? att_src : nullptr,
                             att ? att_dst : nullptr, att ? H : 1, h, h_dtype, ldh,
                             att ? asrc : nullptr, att ? adst : nullptr);
    if (st != gnnc::kProjTcDeclined) return st;
  }
  ProjParams p{};
  p.x = x; p.ldx = ldx; p.w = w; p.ldw = ldw; p.N = N; p.K = K; p.F = F;
  p.x_bf16 = x_dtype == GNNC_BF16;
  p.att_src = att ? att_src : nullptr; p.att_dst = att ? att_dst : nullptr;
  p.H = att ? int(H) : 1; p.C = att ? int(F / H) : int(F);
  p.h = h; p.h_bf16 = h_dtype == GNNC_BF16; p.ldh = ldh; p.asrc = asrc; p.adst = adst;
  const unsigned grid = unsigned((N + BM - 1) / BM);
  proj_simt_kernel<<<grid, kThreads, 0, ctx->stream>>>(p);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}
