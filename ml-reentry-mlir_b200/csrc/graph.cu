// Graph preparation on the device: COO -> CSR by destination (the flip +
// coalesce + to_sparse_csr of gnnc/examples/util.py:16-41, and GATConv's
// remove_self_loops + add_self_loops), GCN normalisation (PyG gcn_norm as
// called at gnnc/examples/util.py:22) and CSR validation.
//
// CSR build: every edge becomes a packed key (dst << b) | src with
// b = bit_width(N); dropped self-loops become an all-ones sentinel that sorts
// last. A stable LSD radix sort (8-bit digits, 4096-key tiles) orders the keys
// by (dst, src) - exactly torch's coalesce() order - then duplicates are
// merged (coalesce) or kept (GATConv) and rowptr is filled from the row
// boundaries. All index work is integer and bit-exact.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;  // 4096

constexpr int kSortThreads = 256;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortThreads * kSortItems;  // 4096
constexpr int kRadix = 256;

// ---------------------------------------------------------------------------
// Exclusive scan of int32 (recursive three-phase: tile sums, scan of sums,
// tile scans with offsets). Totals fit in int32 (callers check).
// ---------------------------------------------------------------------------

__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kScanThreads / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kScanThreads / 32) s_warp[lane] = w;
  }
  __syncthreads();
  const int warp_off = warp > 0 ? s_warp[warp - 1] : 0;
  if (total) *total = s_warp[kScanThreads / 32 - 1];
  const int res = warp_off + x - v;
  __syncthreads();
  return res;
}

__global__ void __launch_bounds__(kScanThreads) tile_sum_kernel(const int* in, int64_t n, int* sums) {
  __shared__ int s_warp[32];
  const int64_t base = int64_t(blockIdx.x) * kScanTile;
  int v = 0;
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t idx = base + int64_t(i) * kScanThreads + threadIdx.x;
    if (idx < n) v += in[idx];
  }
  int total;
  block_exclusive_scan(v, s_warp, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Exclusive scan of one tile per block, items contiguous per thread.
__global__ void __launch_bounds__(kScanThreads) tile_scan_kernel(const int* in, int64_t n, int* out,
                                                                 const int* offsets) {
  __shared__ int s_warp[32];
  const int64_t base = int64_t(blockIdx.x) * kScanTile + int64_t(threadIdx.x) * kScanItems;
  int vals[kScanItems];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t idx = base + i;
    vals[i] = idx < n ? in[idx] : 0;
    sum += vals[i];
  }
  int run = block_exclusive_scan(sum, s_warp, nullptr) + (offsets ? offsets[blockIdx.x] : 0);
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t idx = base + i;
    if (idx < n) out[idx] = run;
    run += vals[i];
  }
}

int64_t scan_temp_ints(int64_t n) {
  int64_t t = 0;
  while (n > kScanTile) {
    n = (n + kScanTile - 1) / kScanTile;
    t += n + 1;
  }
  return t;
}

// out[i] = sum(in[0..i)); in and out may alias. temp: scan_temp_ints(n) ints.
void exclusive_scan(const int* in, int* out, int64_t n, int* temp, cudaStream_t st) {
  if (n <= 0) return;
  if (n <= kScanTile) {
    tile_scan_kernel<<<1, kScanThreads, 0, st>>>(in, n, out, nullptr);
    return;
  }
  const int64_t nb = (n + kScanTile - 1) / kScanTile;
  int* sums = temp;
  tile_sum_kernel<<<unsigned(nb), kScanThreads, 0, st>>>(in, n, sums);
  exclusive_scan(sums, sums, nb, temp + nb + 1, st);
  tile_scan_kernel<<<unsigned(nb), kScanThreads, 0, st>>>(in, n, out, sums);
}

// ---------------------------------------------------------------------------
// Key construction
// ---------------------------------------------------------------------------

__global__ void make_keys_kernel(const int64_t* src, const int64_t* dst, int64_t E, int64_t N,
                                 int bits, int self_loops, uint64_t* keys, int* bad) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const uint64_t sentinel = ~uint64_t(0);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < E + (self_loops ? N : 0);
       i += stride) {
    if (i < E) {
      const int64_t s = src[i], d = dst[i];
      if (s < 0 || s >= N || d < 0 || d >= N) {
        atomicAdd(bad, 1);
        atomicAdd(bad + 1, 1);
        keys[i] = sentinel;
      } else if (self_loops && s == d) {
        atomicAdd(bad + 1, 1);
        keys[i] = sentinel;
      } else {
        keys[i] = (uint64_t(d) << bits) | uint64_t(s);
      }
    } else {
      const uint64_t v = uint64_t(i - E);
      keys[i] = (v << bits) | v;
    }
  }
}

// ---------------------------------------------------------------------------
// Stable LSD radix sort pass (8-bit digit at `shift`)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kSortThreads) radix_hist_kernel(const uint64_t* keys, int64_t n,
                                                                  int shift, int num_tiles,
                                                                  int* counts) {
  __shared__ int s_hist[kRadix];
  s_hist[threadIdx.x] = 0;
  __syncthreads();
  const int64_t base = int64_t(blockIdx.x) * kSortTile;
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t idx = base + int64_t(r) * kSortThreads + threadIdx.x;
    if (idx < n) atomicAdd(&s_hist[int((keys[idx] >> shift) & 0xff)], 1);
  }
  __syncthreads();
  counts[int64_t(threadIdx.x) * num_tiles + blockIdx.x] = s_hist[threadIdx.x];
}

__global__ void __launch_bounds__(kSortThreads) radix_scatter_kernel(const uint64_t* keys_in,
                                                                     uint64_t* keys_out, int64_t n,
                                                                     int shift, int num_tiles,
                                                                     const int* offsets) {
  constexpr int kW = kSortThreads / 32;
  __shared__ int s_base[kRadix];       // global position of this tile's next key per digit
  __shared__ int s_wcnt[kW][kRadix];   // per-round, per-warp digit counts
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  s_base[threadIdx.x] = offsets[int64_t(threadIdx.x) * num_tiles + blockIdx.x];
  for (int w = 0; w < kW; ++w) s_wcnt[w][threadIdx.x] = 0;
  __syncthreads();
  const int64_t base = int64_t(blockIdx.x) * kSortTile;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t idx = base + int64_t(r) * kSortThreads + threadIdx.x;
    const bool ok = idx < n;
    const uint64_t key = ok ? keys_in[idx] : 0;
    const int digit = ok ? int((key >> shift) & 0xff) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, digit);
    const int rank = __popc(peers & lt_mask);
    if (ok && rank == 0) s_wcnt[warp][digit] = __popc(peers);
    __syncthreads();
    if (ok) {
      int pos = s_base[digit] + rank;
      for (int w = 0; w < warp; ++w) pos += s_wcnt[w][digit];
      keys_out[pos] = key;
    }
    __syncthreads();
    {
      int add = 0;
      for (int w = 0; w < kW; ++w) {
        add += s_wcnt[w][threadIdx.x];
        s_wcnt[w][threadIdx.x] = 0;
      }
      s_base[threadIdx.x] += add;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// CSR assembly from sorted keys
// ---------------------------------------------------------------------------

// flag[i] = 1 when key i starts a new (dst, src) run (always 1 without dedupe).
__global__ void run_flags_kernel(const uint64_t* keys, int64_t n, int dedupe, int* flag) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    flag[i] = (!dedupe || i == 0 || keys[i] != keys[i - 1]) ? 1 : 0;
}

// Writes col (and mult) of every run start at its compacted position.
__global__ void compact_kernel(const uint64_t* keys, int64_t n, int bits, const int* flag,
                               const int* pos, int total, int32_t* col, int32_t* mult) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const uint64_t smask = (uint64_t(1) << bits) - 1;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (!flag[i]) continue;
    const int j = pos[i];
    col[j] = int32_t(keys[i] & smask);
    if (mult) {
      // Run length = distance to the next run start (runs are the copies of
      // one duplicated edge, so the forward walk is short).
      int64_t e = i + 1;
      while (e < n && !flag[e]) ++e;
      mult[j] = int32_t(e - i);
    }
  }
}

// rowptr from the compacted entries: every row boundary fills the empty rows
// before it. dst of entry j is recovered from its key via pos/flag order.
__global__ void rowptr_kernel(const uint64_t* keys, int64_t n, int bits, const int* flag,
                              const int* pos, int total, int64_t N, int32_t* rowptr) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i <= n; i += stride) {
    // Consider run starts i (and the virtual end i == n).
    if (i < n && !flag[i]) continue;
    const int64_t d = i < n ? int64_t(keys[i] >> bits) : N;
    // previous run start's row
    int64_t dprev = -1;
    if (i > 0) dprev = int64_t(keys[i - 1] >> bits);
    if (d == dprev) continue;
    const int j = i < n ? pos[i] : total;
    for (int64_t r = dprev + 1; r <= d && r <= N; ++r) rowptr[r] = j;
  }
}

// ---------------------------------------------------------------------------
// GCN normalisation and validation
// ---------------------------------------------------------------------------

__global__ void gcn_deg_kernel(const int32_t* rowptr, const int32_t* mult, int64_t N,
                               float* deg, float* dinv) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; r < N; r += stride) {
    const int b = rowptr[r], e = rowptr[r + 1];
    int64_t d = 0;
    if (mult) {
      for (int k = b; k < e; ++k) d += mult[k];
    } else {
      d = e - b;
    }
    const float df = float(d);
    // torch: deg.pow_(-0.5) -> 1 / sqrt(deg) with IEEE rounding; inf -> 0.
    const float di = df > 0.f ? __fdiv_rn(1.0f, __fsqrt_rn(df)) : 0.f;
    if (deg) deg[r] = df;
    dinv[r] = di;
  }
}

__global__ void gcn_w_kernel(const int32_t* rowptr, const int32_t* col, const int32_t* mult,
                             int64_t N, const float* dinv, float* w) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < N; r += warps) {
    const float dd = dinv[r];
    const int b = rowptr[r], e = rowptr[r + 1];
    for (int k = b + lane; k < e; k += 32) {
      const int c = col[k];
      const float one = unsigned(c) < unsigned(N) ? __fmul_rn(dinv[c], dd) : 0.f;
      float v = one;
      if (mult)
        for (int m = 1; m < mult[k]; ++m) v = __fadd_rn(v, one);
      w[k] = v;
    }
  }
}

// SAGE mean weights: w_out[k] = w_in[k] / max(#{j in row : w_in[j] != 0}, 1)
// (w_in null: every stored edge counts, weight 1). One warp per row.
__global__ void mean_w_kernel(const int32_t* rowptr, int64_t n_rows, const float* w_in,
                              float* w_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < n_rows; r += warps) {
    const int b = rowptr[r], e = rowptr[r + 1];
    int nnz = 0;
    for (int k0 = b; k0 < e; k0 += 32) {
      const int k = k0 + lane;
      const bool nz = k < e && (w_in == nullptr || w_in[k] != 0.f);
      nnz += __popc(__ballot_sync(0xffffffffu, nz));
    }
    const float d = float(nnz > 1 ? nnz : 1);
    for (int k = b + lane; k < e; k += 32) w_out[k] = __fdiv_rn(w_in ? w_in[k] : 1.f, d);
  }
}

__global__ void validate_kernel(const int32_t* rowptr, const int32_t* col, int64_t n_rows,
                                int64_t E, int64_t n_src, int* words) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_rows; i += stride) {
    const int b = rowptr[i], e = rowptr[i + 1];
    if (b < 0 || e < b || e > E) {
      atomicAdd(words + 0, 1);
      atomicMin(words + 1, int(i));
    }
  }
  for (int64_t k = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; k < E; k += stride) {
    const int c = col[k];
    if (c < 0 || int64_t(c) >= n_src) {
      atomicAdd(words + 2, 1);
      atomicMin(words + 3, int(k));
    }
  }
}

unsigned grid_for(int64_t n, int threads, int num_sms) {
  int64_t g = (n + threads - 1) / threads;
  const int64_t cap = int64_t(num_sms) * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return unsigned(g);
}

int bit_width(int64_t v) {
  int b = 0;
  while ((int64_t(1) << b) <= v) ++b;
  return b;
}

}  // namespace

extern "C" int gnnc_csr_from_coo(gnnc_ctx_t* ctx, const int64_t* src, const int64_t* dst,
                                 int64_t E, int64_t N, int self_loops, int dedupe,
                                 int32_t* rowptr, int32_t* col, int32_t* mult, int64_t capacity,
                                 int64_t* E_out) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, E >= 0 && N >= 0, "negative sizes");
  GNNC_CHECK_ARG(ctx, E_out != nullptr && rowptr != nullptr, "null E_out/rowptr");
  GNNC_CHECK_ARG(ctx, E == 0 || (src && dst), "null src/dst");
  const int64_t n_keys = E + (self_loops ? N : 0);
  GNNC_CHECK_ARG(ctx, capacity >= n_keys, "capacity %lld < %lld", (long long)capacity,
                 (long long)n_keys);
  GNNC_CHECK_ARG(ctx, n_keys == 0 || col != nullptr, "null col");
  GNNC_CHECK_ARG(ctx, n_keys < (int64_t(1) << 31) - 1 && N < (int64_t(1) << 31) - 1,
                 "graph exceeds int32 CSR indexing");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  *E_out = 0;
  if (N == 0) {
    GNNC_CUDA_TRY(ctx, cudaMemsetAsync(rowptr, 0, sizeof(int32_t), st));
    return GNNC_OK;
  }
  const int bits = bit_width(N);  // N itself fits, so valid keys < all-ones sentinel
  const int key_bits = 2 * bits;
  const int passes = (key_bits + 7) / 8;
  const int64_t num_tiles = std::max<int64_t>(1, (n_keys + kSortTile - 1) / kSortTile);
  const int64_t n_counts = num_tiles * kRadix;
  GNNC_CHECK_ARG(ctx, n_counts < (int64_t(1) << 31), "too many sort tiles");

  // Workspace carve-up.
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    size_t o = off;
    off = gnnc::align_up(off + bytes, 256);
    return o;
  };
  const size_t o_ka = carve(sizeof(uint64_t) * std::max<int64_t>(n_keys, 1));
  const size_t o_kb = carve(sizeof(uint64_t) * std::max<int64_t>(n_keys, 1));
  const size_t o_cnt = carve(sizeof(int) * n_counts);
  const size_t o_flag = carve(sizeof(int) * std::max<int64_t>(n_keys, 1));
  const size_t o_pos = carve(sizeof(int) * std::max<int64_t>(n_keys, 1));
  const int64_t tmp_ints =
      std::max(scan_temp_ints(n_counts), scan_temp_ints(std::max<int64_t>(n_keys, 1))) + 64;
  const size_t o_tmp = carve(sizeof(int) * tmp_ints);
  int sts = gnnc::ensure_workspace(ctx, off);
  if (sts) return sts;
  char* ws = reinterpret_cast<char*>(ctx->ws);
  uint64_t* ka = reinterpret_cast<uint64_t*>(ws + o_ka);
  uint64_t* kb = reinterpret_cast<uint64_t*>(ws + o_kb);
  int* counts = reinterpret_cast<int*>(ws + o_cnt);
  int* flag = reinterpret_cast<int*>(ws + o_flag);
  int* pos = reinterpret_cast<int*>(ws + o_pos);
  int* tmp = reinterpret_cast<int*>(ws + o_tmp);
  int* words = ctx->dev_words + 8;  // [0] bad-index count

  GNNC_CUDA_TRY(ctx, cudaMemsetAsync(words, 0, 4 * sizeof(int), st));
  if (n_keys > 0) {
    make_keys_kernel<<<grid_for(n_keys, 256, ctx->num_sms), 256, 0, st>>>(src, dst, E, N, bits,
                                                                          self_loops, ka, words);
    GNNC_CUDA_TRY(ctx, cudaGetLastError());
    for (int ps = 0; ps < passes; ++ps) {
      const int shift = ps * 8;
      radix_hist_kernel<<<unsigned(num_tiles), kSortThreads, 0, st>>>(ka, n_keys, shift,
                                                                      int(num_tiles), counts);
      exclusive_scan(counts, counts, n_counts, tmp, st);
      radix_scatter_kernel<<<unsigned(num_tiles), kSortThreads, 0, st>>>(
          ka, kb, n_keys, shift, int(num_tiles), counts);
      std::swap(ka, kb);
    }
    GNNC_CUDA_TRY(ctx, cudaGetLastError());
  }
  // words[0] = endpoints outside [0, N), words[1] = keys turned into sentinels
  // (those plus dropped self-loops); sentinels sorted to the end.
  int hw[2] = {0, 0};
  GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(hw, words, sizeof(hw), cudaMemcpyDeviceToHost, st));
  GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(st));
  if (hw[0])
    return gnnc::set_error(ctx, GNNC_ERR_BOUNDS, "%d edge endpoints outside [0, %lld)", hw[0],
                           (long long)N);
  const int64_t n_valid = n_keys - hw[1];
  int total = 0;
  if (n_valid > 0) {
    run_flags_kernel<<<grid_for(n_valid, 256, ctx->num_sms), 256, 0, st>>>(ka, n_valid, dedupe,
                                                                           flag);
    exclusive_scan(flag, pos, n_valid, tmp, st);
    int last_pos = 0, last_flag = 0;
    GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(&last_pos, pos + n_valid - 1, sizeof(int),
                                       cudaMemcpyDeviceToHost, st));
    GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(&last_flag, flag + n_valid - 1, sizeof(int),
                                       cudaMemcpyDeviceToHost, st));
    GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(st));
    total = last_pos + last_flag;
    compact_kernel<<<grid_for(n_valid, 256, ctx->num_sms), 256, 0, st>>>(ka, n_valid, bits, flag,
                                                                         pos, total, col, mult);
    rowptr_kernel<<<grid_for(n_valid + 1, 256, ctx->num_sms), 256, 0, st>>>(
        ka, n_valid, bits, flag, pos, total, N, rowptr);
    GNNC_CUDA_TRY(ctx, cudaGetLastError());
  } else {
    GNNC_CUDA_TRY(ctx, cudaMemsetAsync(rowptr, 0, sizeof(int32_t) * (N + 1), st));
  }
  GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(st));
  *E_out = total;
  return GNNC_OK;
}

extern "C" int gnnc_gcn_norm(gnnc_ctx_t* ctx, const int32_t* rowptr, const int32_t* col,
                             const int32_t* mult, int64_t N, float* deg, float* dinv, float* w) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, N >= 0, "negative N");
  GNNC_CHECK_ARG(ctx, N == 0 || (rowptr && col && w), "null rowptr/col/w");
  if (N == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  float* di = dinv;
  if (!di) {
    int st = gnnc::ensure_workspace(ctx, sizeof(float) * N);
    if (st) return st;
    di = reinterpret_cast<float*>(ctx->ws);
  }
  gcn_deg_kernel<<<grid_for(N, 256, ctx->num_sms), 256, 0, ctx->stream>>>(rowptr, mult, N, deg,
                                                                          di);
  gcn_w_kernel<<<grid_for(N * 32, 256, ctx->num_sms), 256, 0, ctx->stream>>>(rowptr, col, mult,
                                                                             N, di, w);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}

extern "C" int gnnc_mean_norm(gnnc_ctx_t* ctx, const int32_t* rowptr, int64_t n_rows,
                              const float* w_in, float* w_out) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, n_rows >= 0, "negative n_rows");
  GNNC_CHECK_ARG(ctx, n_rows == 0 || (rowptr && w_out), "null rowptr/w_out");
  if (n_rows == 0) return GNNC_OK;
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  mean_w_kernel<<<grid_for(n_rows * 32, 256, ctx->num_sms), 256, 0, ctx->stream>>>(
      rowptr, n_rows, w_in, w_out);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}

extern "C" int gnnc_csr_validate(gnnc_ctx_t* ctx, const int32_t* rowptr, const int32_t* col,
                                 int64_t n_rows, int64_t E, int64_t n_src) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, n_rows >= 0 && E >= 0 && n_src >= 0, "negative sizes");
  GNNC_CHECK_ARG(ctx, rowptr != nullptr && (E == 0 || col != nullptr), "null rowptr/col");
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  int* words = ctx->dev_words + 16;
  int init[4] = {0, INT32_MAX, 0, INT32_MAX};
  GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(words, init, sizeof(init), cudaMemcpyHostToDevice,
                                     ctx->stream));
  const int64_t n = std::max(n_rows, E);
  if (n > 0)
    validate_kernel<<<grid_for(n, 256, ctx->num_sms), 256, 0, ctx->stream>>>(rowptr, col, n_rows,
                                                                             E, n_src, words);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  int res[4];
  GNNC_CUDA_TRY(ctx, cudaMemcpyAsync(res, words, sizeof(res), cudaMemcpyDeviceToHost,
                                     ctx->stream));
  GNNC_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  if (res[0])
    return gnnc::set_error(ctx, GNNC_ERR_BOUNDS, "%d bad rowptr entries, first at row %d", res[0],
                           res[1]);
  if (res[2])
    return gnnc::set_error(ctx, GNNC_ERR_BOUNDS,
                           "%d column indices outside [0, %lld), first at entry %d", res[2],
                           (long long)n_src, res[3]);
  return GNNC_OK;
}
