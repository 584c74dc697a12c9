// tcgen05 projection: h = x . w^T on the 5th-generation tensor cores, bf16
// operands, fp32 accumulation in tensor memory, with GATConv's attention
// coefficients (asrc = h_head . att_src, adst = h_head . att_dst) computed in
// the epilogue from the fp32 accumulator.
//
// One persistent CTA per SM walks 128-row tiles of x. Warp roles:
//   warp 0 (one lane): TMA producer. Each pipeline stage holds a 128 x 64
//     k-block of x and the matching F16 x 64 k-block of w, both in the
//     128-byte-swizzled K-major layout, loaded with cp.async.bulk.tensor into a
//     4-stage ring guarded by mbarriers (no multicast).
//   warp 1: allocates 512 TMEM columns (two 128 x 256 fp32 accumulators), and
//     one lane issues tcgen05.mma (M = 128, N = F16, K = 16 per instruction)
//     and tcgen05.commit to release stages and publish finished tiles.
//   warps 2-5: epilogue. Warp w reads TMEM lanes 32*(w%4) .. +31 (one tile row
//     per thread) with tcgen05.ld, folds the per-head dot products with
//     att_src / att_dst (sequential over columns: deterministic), converts the
//     row into a padded shared-memory staging tile, releases the accumulator,
//     then writes its 32 rows to h with one coalesced 512-byte store per row.
// The two accumulators let the MMAs of tile i+1 run under the epilogue of
// tile i. Every mbarrier wait is bounded by %globaltimer; a wait that gives up
// raises an abort flag the other roles see, records GNNC_ERR_TIMEOUT in the
// context's error word, drains outstanding copies / MMAs (again bounded) and
// frees TMEM before the kernel returns.
#include <cuda.h>  // CUtensorMap and the cuTensorMapEncodeTiled prototype (no libcuda link)

#include <mutex>

#include "proj_tc.cuh"

namespace {

constexpr int kBM = 128;  // tile rows = MMA M
constexpr int kBK = 64;   // k-block: 64 bf16 = one 128-byte swizzle row
constexpr int kStages = 3;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccStride = 256;  // TMEM columns per accumulator buffer
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait
constexpr int kMaxF = 256;
// Per epilogue warp: 32 output rows of up to 512 bytes, padded by 16 bytes so
// the per-thread row writes hit distinct banks.
constexpr int kStageRowBytes = 512 + 16;
// Bytes reserved for the 2*kStages + 5 mbarriers (a multiple of 16).
constexpr int kBarrierBytes = ((2 * kStages + 5) * 8 + 15) / 16 * 16;
static_assert(kStageRowBytes % 16 == 0 && kBarrierBytes % 16 == 0, "16-byte aligned regions");
static_assert((2 * kMaxF * 4) % 16 == 0, "staging must start 16-byte aligned");

struct TcParams {
  int N, K, F, N16, nkb, n_tiles;
  int H, C;
  const float* att_src;
  const float* att_dst;
  void* h;
  int h_bf16;
  int64_t ldh;
  float* asrc;
  float* adst;
  int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// One try_wait. The suspend hint lets the hardware park the thread until the
// phase completes (or ~10 ms pass) instead of spinning on issue slots that the
// epilogue warps sharing the scheduler need.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(10000000u)
      : "memory");
  return ok != 0;
}

// Waits for the phase `parity` of barrier b. Returns false when the wait gave
// up (time limit) or another role aborted; a time-out raises the abort flag.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort,
                                          bool watch_abort = true) {
  const unsigned long long t0 = now_ns();
  for (;;) {
    if (mbar_try_wait(b, parity)) return true;
    if (watch_abort && *abort) return false;
    if (now_ns() - t0 > kWaitNs) {
      *abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), tcgen05 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = uint64_t((saddr & 0x3FFFFu) >> 4);
  d |= uint64_t(1) << 16;            // LBO (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;    // SBO
  d |= uint64_t(1) << 46;            // version
  d |= uint64_t(2) << 61;            // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread
// (no wait: the caller batches loads before one tcgen05.wait::ld).
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// Instruction descriptor of kind::f16: fp32 accumulate, bf16 A and B, both
// K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
}

__global__ void __launch_bounds__(kThreads, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                   const TcParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_bytes = kBM * kBK * 2;
  const int b_bytes = p.N16 * kBK * 2;
  const int stage_bytes = a_bytes + b_bytes;  // multiple of 1024 (N16 % 16 == 0)
  // Carve-up (offsets from the 1024-byte aligned base; every region starts on
  // a multiple of 16 bytes whatever kStages is):
  //   [stages][kBarrierBytes: mbarriers][16: TMEM address, abort flag]
  //   [2*kMaxF floats: att_src, att_dst][kEpiWarps*32 rows: output staging]
  unsigned char* stages = smem;
  unsigned char* bar_base = smem + kStages * stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_base);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_base + kBarrierBytes);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_att = reinterpret_cast<float*>(bar_base + kBarrierBytes + 16);  // [2][kMaxF]
  unsigned char* s_stage = reinterpret_cast<unsigned char*>(s_att + 2 * kMaxF);  // [kEpiWarps][32][kStageRowBytes]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool att = p.att_src != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (att)
    for (int i = threadIdx.x; i < p.F; i += kThreads) {
      s_att[i] = p.att_src[i];
      s_att[kMaxF + i] = p.att_dst[i];
    }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x) {
        for (int kb = 0; kb < p.nkb; ++kb) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], uint32_t(stage_bytes));
          unsigned char* dst = stages + s * stage_bytes;
          tma_load_2d(dst, &map_x, &full[s], kb * kBK, tile * kBM);
          tma_load_2d(dst + a_bytes, &map_w, &full[s], kb * kBK, 0);
          ++it;
        }
      }
      if (!ok) {
        // Let the copies still in flight land before the CTA goes away.
        for (int j = it > kStages ? it - kStages : 0; j < it; ++j)
          mbar_wait(&full[j % kStages], (j / kStages) & 1, abort, false);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(p.N16);
      int it = 0, t_iter = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x, ++t_iter) {
        const int b = t_iter & 1;
        if (!mbar_wait(&tempty[b], ((t_iter >> 1) & 1) ^ 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b) * kAccStride;
        for (int kb = 0; kb < p.nkb; ++kb) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + s * stage_bytes);
          const uint64_t adesc = sw128_desc(a_addr);
          const uint64_t bdesc = sw128_desc(a_addr + uint32_t(a_bytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16(d, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                      (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
          ++it;
        }
        if (ok) umma_commit(&tfull[b]);
      }
      // Every MMA this thread issued is complete once `drain` flips.
      umma_commit(drain);
      mbar_wait(drain, 0, abort, false);
    }
  } else {
    // Epilogue: one tile row per thread.
    const int q = warp & 3;
    const int rloc = q * 32 + lane;
    const int esize = p.h_bf16 ? 2 : 4;
    const int pass_cols = 512 / esize;  // columns staged per pass
    unsigned char* stage = s_stage + (warp - 2) * 32 * kStageRowBytes;
    int t_iter = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++t_iter) {
      const int b = t_iter & 1;
      if (!mbar_wait(&tfull[b], (t_iter >> 1) & 1, abort)) break;
      tc_fence_after();
      const int64_t row = int64_t(tile) * kBM + rloc;
      const bool live = row < p.N;
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(b) * kAccStride;
      float run_s = 0.f, run_d = 0.f;
      int cur = 0;
      for (int p0 = 0; p0 < p.N16; p0 += pass_cols) {
        const int p1 = min(p.N16, p0 + pass_cols);
        int col0 = p0;
        for (; col0 < p1; col0 += 64) {
          // 64 columns per tcgen05.wait::ld when they fit, else 16 at a time.
          const int width = (col0 + 64 <= p1) ? 64 : 16;
          uint32_t r[64];
          if (width == 64) {
            tmem_ld32_async(taddr + uint32_t(col0), r);
            tmem_ld32_async(taddr + uint32_t(col0 + 32), r + 32);
            tmem_wait_ld();
          } else {
            uint32_t r16[16];
            tmem_ld16(taddr + uint32_t(col0), r16);
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = r16[e];
          }
          for (int sub = 0; sub < width; sub += 16) {
            const int c0 = col0 + sub;
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(r[sub + e]);
            if (att && live) {
              // Heads are contiguous column ranges; a 16-column chunk lies in
              // one head (C % 16 == 0 or H == 1), so the sums run per head.
              const int hd = p.H == 1 ? 0 : c0 / p.C;
              if (hd != cur) {
                p.asrc[size_t(row) * p.H + cur] = run_s;
                p.adst[size_t(row) * p.H + cur] = run_d;
                run_s = run_d = 0.f;
                cur = hd;
              }
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const float ws = c0 + e < p.F ? s_att[c0 + e] : 0.f;
                const float wd = c0 + e < p.F ? s_att[kMaxF + c0 + e] : 0.f;
                run_s = fmaf(v[e], ws, run_s);
                run_d = fmaf(v[e], wd, run_d);
              }
            }
            unsigned char* srow = stage + lane * kStageRowBytes + (c0 - p0) * esize;
            if (p.h_bf16) {
              uint4* o4 = reinterpret_cast<uint4*>(srow);
              o4[0] = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]),
                                 pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
              o4[1] = make_uint4(pack_bf16(v[8], v[9]), pack_bf16(v[10], v[11]),
                                 pack_bf16(v[12], v[13]), pack_bf16(v[14], v[15]));
            } else {
              float4* o4 = reinterpret_cast<float4*>(srow);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                o4[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
            }
          }
          if (width == 16) col0 -= 48;  // advance by 16 for the tail chunks
        }
        if (p1 >= p.N16) {
          // Accumulator fully read: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
        }
        __syncwarp();
        // Coalesced write-out of this warp's 32 rows, columns [p0, min(F, p1)).
        const int cols = min(p.F, p1) - p0;
        if (cols > 0) {
          const int bytes = cols * esize;
          const int n16 = bytes / 16;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const int64_t grow = int64_t(tile) * kBM + q * 32 + rr;
            if (grow >= p.N) continue;
            unsigned char* g = reinterpret_cast<unsigned char*>(p.h) +
                               (size_t(grow) * size_t(p.ldh) + size_t(p0)) * esize;
            const unsigned char* sr = stage + rr * kStageRowBytes;
            for (int j = lane; j < n16; j += 32)
              *reinterpret_cast<uint4*>(g + j * 16) = *reinterpret_cast<const uint4*>(sr + j * 16);
            for (int j = n16 * 16 + lane * esize; j < bytes; j += 32 * esize) {
              if (esize == 2)
                *reinterpret_cast<uint16_t*>(g + j) = *reinterpret_cast<const uint16_t*>(sr + j);
              else
                *reinterpret_cast<uint32_t*>(g + j) = *reinterpret_cast<const uint32_t*>(sr + j);
            }
          }
        }
        __syncwarp();
      }
      if (att && live) {
        p.asrc[size_t(row) * p.H + cur] = run_s;
        p.adst[size_t(row) * p.H + cur] = run_d;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && *abort) atomicExch(p.err, GNNC_ERR_TIMEOUT);
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);

std::mutex g_encode_mu;
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn(gnnc_ctx_t* ctx) {
  std::lock_guard<std::mutex> lock(g_encode_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    else
      gnnc::set_error(ctx, GNNC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  }
  return g_encode;
}

// 2-D bf16 tensor map: inner dim `inner` (elements), `rows` rows of `ld`
// elements, box kBK x box_rows, 128-byte swizzle, zero fill out of bounds.
bool make_map(EncodeTiledFn enc, CUtensorMap* map, const void* base, int64_t inner,
              int64_t rows, int64_t ld, int box_rows) {
  const cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace gnnc {

int proj_tc_try(gnnc_ctx_t* ctx, const void* x, int64_t ldx, const void* w, int64_t ldw,
                int64_t N, int64_t K, int64_t F, const float* att_src, const float* att_dst,
                int64_t H, void* h, int h_dtype, int64_t ldh, float* asrc, float* adst) {
  const bool att = att_src != nullptr;
  const int64_t C = att ? F / H : F;
  // Shapes and alignment the tensor-core kernel handles; anything else goes
  // to the CUDA-core kernel.
  if (F > kMaxF || N < 1 || N > (int64_t(1) << 31) - 1 || K < 1 || K > (1 << 20)) return kProjTcDeclined;
  if (ldx % 8 || ldw % 8) return kProjTcDeclined;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16) return kProjTcDeclined;
  if (reinterpret_cast<uintptr_t>(h) % 16) return kProjTcDeclined;
  if (h_dtype == GNNC_BF16 ? (ldh % 8 != 0) : (ldh % 4 != 0)) return kProjTcDeclined;
  if (att && !(H == 1 || C % 16 == 0)) return kProjTcDeclined;
  EncodeTiledFn enc = encode_fn(ctx);
  if (!enc) return kProjTcDeclined;

  const int N16 = int((F + 15) / 16 * 16);
  CUtensorMap map_x, map_w;
  if (!make_map(enc, &map_x, x, K, N, ldx, kBM) || !make_map(enc, &map_w, w, K, F, ldw, N16))
    return kProjTcDeclined;

  TcParams p{};
  p.N = int(N);
  p.K = int(K);
  p.F = int(F);
  p.N16 = N16;
  p.nkb = int((K + kBK - 1) / kBK);
  p.n_tiles = int((N + kBM - 1) / kBM);
  p.H = att ? int(H) : 1;
  p.C = int(C);
  p.att_src = att_src;
  p.att_dst = att_dst;
  p.h = h;
  p.h_bf16 = h_dtype == GNNC_BF16;
  p.ldh = ldh;
  p.asrc = asrc;
  p.adst = adst;
  p.err = ctx->dev_words + 3;

  const size_t stage_bytes = size_t(kBM) * kBK * 2 + size_t(N16) * kBK * 2;
  static_assert((kBM * kBK * 2) % 1024 == 0, "stage base alignment");
  if (stage_bytes % 1024 != 0) return kProjTcDeclined;  // keeps every stage 1024-byte aligned
  size_t smem = 1024 + kStages * stage_bytes + kBarrierBytes + 16 + 2 * kMaxF * sizeof(float) +
                size_t(kEpiWarps) * 32 * kStageRowBytes;
  // At least 120 KB, so two CTAs never share an SM (each takes all 512 TMEM columns).
  if (smem < 120 * 1024) smem = 120 * 1024;
  GNNC_CUDA_TRY(ctx, cudaFuncSetAttribute(proj_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int grid = p.n_tiles < ctx->num_sms ? p.n_tiles : ctx->num_sms;
  proj_tc_kernel<<<grid, kThreads, smem, ctx->stream>>>(map_x, map_w, p);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}

}  // namespace gnnc
