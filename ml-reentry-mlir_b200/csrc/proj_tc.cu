// tcgen05 projection: h = x . w^T on the 5th-generation tensor cores, bf16
// operands, fp32 accumulation in tensor memory, with GATConv's attention
// coefficients (asrc = h_head . att_src, adst = h_head . att_dst) computed in
// the epilogue from the fp32 accumulator.
//
// One persistent CTA per SM walks 128-row tiles of x. Warp roles:
//   warp 0 (one lane): TMA producer (cp.async.bulk.tensor, no multicast). When
//     all k-blocks of w fit in 64 KB they are loaded once and stay resident,
//     and the ring of stages carries only 128 x 64 k-blocks of x; otherwise
//     each stage carries the x k-block and the matching w k-block. Operands are
//     in the 128-byte-swizzled K-major layout.
//   warp 1: allocates 512 TMEM columns (two 128 x 256 fp32 accumulators); one
//     lane issues tcgen05.mma (M = 128, N = F16, K = 16 per instruction) and
//     tcgen05.commit to release stages and publish finished tiles.
//   warps 2-17: epilogue, four warps per scheduler (the epilogue is a chain
//     of dependent TMEM loads, FMAs and conversions: it needs the warps to
//     hide that latency). Warp w reads TMEM lanes 32*(w%4) .. +31 (one tile
//     row per thread) and the column group (w-2)/4 of the accumulator (four
//     groups, split at multiples of 128 bytes of output and, for GAT, at head
//     boundaries). Per 128-byte pass of its columns it folds the per-head dot
//     products with att_src / att_dst (fixed summation order: deterministic),
//     converts, writes the values into a 128-byte-swizzled staging box and
//     hands the box to a TMA bulk-tensor store (one box per warp: at F = 256
//     bf16 a warp makes one pass per tile, so the box it reuses was handed
//     off a whole tile earlier). The store clips rows >= N and columns >= F.
// The two accumulators let the MMAs of tile i+1 run under the epilogue of
// tile i. Every mbarrier wait is bounded by %globaltimer; a wait that gives up
// raises an abort flag the other roles see, records GNNC_ERR_TIMEOUT in the
// context's error word, drains outstanding copies / MMAs (again bounded) and
// frees TMEM before the kernel returns.
#include <cuda.h>  // CUtensorMap and the cuTensorMapEncodeTiled prototype (no libcuda link)

#include <climits>
#include <mutex>

#include "proj_tc.cuh"

namespace {

constexpr int kBM = 128;  // tile rows = MMA M
constexpr int kBK = 64;   // k-block: 64 bf16 = one 128-byte swizzle row
constexpr int kStagesResident = 5;  // x-only stages when w stays resident
constexpr int kStagesStream = 3;    // x + w stages otherwise
constexpr int kMaxStages = 5;
constexpr int kEpiWarps = 16;
constexpr int kEpiGroups = kEpiWarps / 4;  // column groups (4 TMEM lane quarters each)
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccStride = 256;  // TMEM columns per accumulator buffer
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait
constexpr int kMaxF = 256;
constexpr int kResidentWBytes = 64 * 1024;
// Output staging: one TMA store box = 32 rows x 128 bytes per epilogue warp
// (1024-byte aligned: the 128-byte swizzle repeats every 8 rows).
constexpr int kBoxRows = 32;
constexpr int kBoxBytes = kBoxRows * 128;
constexpr int kStagingBytes = kEpiWarps * kBoxBytes;
// Bytes reserved for the 2*kMaxStages + 6 mbarriers (a multiple of 16).
constexpr int kBarrierBytes = ((2 * kMaxStages + 6) * 8 + 15) / 16 * 16;
static_assert(kBarrierBytes % 16 == 0 && kBoxBytes % 1024 == 0, "aligned regions");

struct TcParams {
  int N, K, F, N16, nkb, n_tiles;
  int cs;  // accumulator columns per epilogue column group
  int Fs;  // columns the bulk stores cover: F rounded down to 16 bytes of output
  int w_resident;  // all w k-blocks live in shared memory for the whole kernel
  int stages;
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
                                          bool watch_abort = true,
                                          unsigned long long limit_ns = kWaitNs) {
  const unsigned long long t0 = now_ns();
  for (;;) {
    if (mbar_try_wait(b, parity)) return true;
    if (watch_abort && *abort) return false;
    if (now_ns() - t0 > limit_ns) {
      *abort = 1;
      return false;
    }
  }
}

// Self-test of the bounded wait and of its error report: thread 0 waits, with
// the projection's mbar_wait, on an mbarrier that nothing ever arrives on.
// The wait gives up after limit_ns and the kernel records GNNC_ERR_TIMEOUT in
// the context's error word exactly as a projection whose wait gave up does.
// Nothing is in flight (no copy, no MMA, no TMEM), so giving up is harmless.
__global__ void wait_selftest_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile int* abort = &abort_flag;
    if (!mbar_wait(&bar, 0, abort, true, limit_ns) && *abort) atomicExch(err, GNNC_ERR_TIMEOUT);
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

// Shared -> global bulk-tensor store of one box (rows / columns outside the
// tensor map's extent are not written).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until no committed store group still reads shared memory.
__device__ __forceinline__ void bulk_wait_read_0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
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

// (c0, c1) += (a0 * b0, a1 * b1) as one packed fp32x2 FMA: each lane rounds
// exactly as fmaf does.
__device__ __forceinline__ void ffma2(float& c0, float& c1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Flushes the attention sums of head `hd` for this thread's row.
__device__ __forceinline__ void att_flush(const TcParams& p, int64_t row, int hd, const float (&ps)[4],
                                          const float (&pd)[4]) {
  if (row < p.N) {
    p.asrc[size_t(row) * p.H + hd] = (ps[0] + ps[1]) + (ps[2] + ps[3]);
    p.adst[size_t(row) * p.H + hd] = (pd[0] + pd[1]) + (pd[2] + pd[3]);
  }
}

// One block of WB (32 or 16) accumulator columns from column c of this
// thread's row (TMEM lane): attention partial sums of the heads the columns
// belong to, then conversion into the row's slot of the swizzled staging box
// (16-byte chunk j of row r at chunk slot j ^ (r % 8); jbase = the block's
// first chunk within the 128-byte row). Blocks are loaded and retired one at a
// time so a thread holds at most 32 accumulator columns. `cur` is the head
// whose sums ps / pd hold and `head_end` its first column past the head;
// columns arrive in increasing order, so crossing head_end moves to the next
// head (a 16-column chunk never straddles two: C % 16 == 0 or H == 1).
template <int WB, bool kBf16>
__device__ __forceinline__ void epi_block(const TcParams& p, uint32_t taddr, int c, int jbase,
                                          unsigned char* srow, const float* s_att, bool att,
                                          int64_t row, float (&ps)[4], float (&pd)[4], int& cur,
                                          int& head_end, int lane) {
  static_assert(WB == 32 || WB == 16, "block width");
  uint32_t r[WB];
  if constexpr (WB == 32)
    tmem_ld32_async(taddr + uint32_t(c), r);
  else
    tmem_ld16_async(taddr + uint32_t(c), r);
  tmem_wait_ld();
  if (att) {
#pragma unroll
    for (int sub = 0; sub < WB; sub += 16) {
      const int cc = c + sub;
      if (cc >= head_end) {
        att_flush(p, row, cur, ps, pd);
#pragma unroll
        for (int j = 0; j < 4; ++j) ps[j] = pd[j] = 0.f;
        ++cur;
        head_end += p.C;
      }
      const float4* ws = reinterpret_cast<const float4*>(s_att + cc);
      const float4* wd = reinterpret_cast<const float4*>(s_att + kMaxF + cc);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 a = ws[j], d = wd[j];
        const float v0 = __uint_as_float(r[sub + 4 * j]), v1 = __uint_as_float(r[sub + 4 * j + 1]);
        const float v2 = __uint_as_float(r[sub + 4 * j + 2]), v3 = __uint_as_float(r[sub + 4 * j + 3]);
        ffma2(ps[0], ps[1], v0, v1, a.x, a.y);
        ffma2(ps[2], ps[3], v2, v3, a.z, a.w);
        ffma2(pd[0], pd[1], v0, v1, d.x, d.y);
        ffma2(pd[2], pd[3], v2, v3, d.z, d.w);
      }
    }
  }
  constexpr int kChunks = kBf16 ? WB / 8 : WB / 4;
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    uint4 v;
    if constexpr (kBf16) {
      const uint32_t* q = r + 8 * j;
      v = make_uint4(pack_bf16(__uint_as_float(q[0]), __uint_as_float(q[1])),
                     pack_bf16(__uint_as_float(q[2]), __uint_as_float(q[3])),
                     pack_bf16(__uint_as_float(q[4]), __uint_as_float(q[5])),
                     pack_bf16(__uint_as_float(q[6]), __uint_as_float(q[7])));
    } else {
      v = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    }
    *reinterpret_cast<uint4*>(srow + (((jbase + j) ^ (lane & 7)) << 4)) = v;
  }
}

// One 128-byte pass of an epilogue warp over W accumulator columns from c0 of
// this thread's row: the blocks of epi_block, the partial last chunk, and the
// TMA store of the staging box.
template <int W, bool kBf16>
__device__ __forceinline__ void epi_pass(const TcParams& p, const CUtensorMap* map_h,
                                         uint32_t taddr, int c0, int64_t row, int row0,
                                         unsigned char* box, const float* s_att, bool att,
                                         float (&ps)[4], float (&pd)[4], int& cur, int& head_end,
                                         int lane) {
  static_assert(W % 16 == 0 && W <= (kBf16 ? 64 : 32), "one 128-byte pass");
  constexpr int kColsPerChunk = kBf16 ? 8 : 4;
  unsigned char* srow = box + lane * 128;
#pragma unroll
  for (int b = 0; b + 32 <= W; b += 32)
    epi_block<32, kBf16>(p, taddr, c0 + b, b / kColsPerChunk, srow, s_att, att, row, ps, pd, cur,
                         head_end, lane);
  if constexpr (W % 32 != 0)
    epi_block<16, kBf16>(p, taddr, c0 + W - 16, (W - 16) / kColsPerChunk, srow, s_att, att, row,
                         ps, pd, cur, head_end, lane);
  // Columns [Fs, F) end in a partial 16-byte chunk, which a bulk store would
  // write whole: this thread stores them from its staged chunk instead.
  if (p.Fs < p.F && p.Fs >= c0 && p.Fs < c0 + W && row < p.N) {
    constexpr int kEsize = kBf16 ? 2 : 4;
    const int jt = (p.Fs - c0) * kEsize / 16;
    const unsigned char* chunk = srow + ((jt ^ (lane & 7)) << 4);
    unsigned char* g = reinterpret_cast<unsigned char*>(p.h) + (size_t(row) * size_t(p.ldh) + size_t(p.Fs)) * kEsize;
    for (int e = 0; e < p.F - p.Fs; ++e) {
      if constexpr (kBf16)
        reinterpret_cast<uint16_t*>(g)[e] = reinterpret_cast<const uint16_t*>(chunk)[e];
      else
        reinterpret_cast<uint32_t*>(g)[e] = reinterpret_cast<const uint32_t*>(chunk)[e];
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && row0 < p.N && c0 < p.Fs) {  // a box wholly below the last row has nothing to store
    tma_store_2d(map_h, box, c0, row0);
    bulk_commit();
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                   const __grid_constant__ CUtensorMap map_h, const TcParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_bytes = kBM * kBK * 2;                // 16 KB
  const int b_bytes = p.N16 * kBK * 2;              // one w k-block
  const int stage_bytes = p.w_resident ? a_bytes : a_bytes + b_bytes;  // multiple of 1024
  const int S = p.stages;
  // Carve-up (offsets from the 1024-byte aligned base; the first three regions
  // are multiples of 1024 bytes long, the rest start on 16-byte multiples):
  //   [resident w: nkb * b_bytes][S stages][output staging: kStagingBytes]
  //   [kBarrierBytes: mbarriers][16: TMEM address, abort flag]
  //   [2*kMaxF floats: att_src, att_dst]
  unsigned char* w_res = smem;
  unsigned char* stages = smem + (p.w_resident ? p.nkb * b_bytes : 0);
  unsigned char* s_stage = stages + S * stage_bytes;
  unsigned char* bar_base = s_stage + kStagingBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_base);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* wfull = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_base + kBarrierBytes);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_att = reinterpret_cast<float*>(bar_base + kBarrierBytes + 16);  // [2][kMaxF]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool att = p.att_src != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    mbar_init(wfull, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Attention vectors, zero beyond F so the epilogue needs no column test.
  for (int i = threadIdx.x; i < kMaxF; i += kThreads) {
    s_att[i] = (att && i < p.F) ? p.att_src[i] : 0.f;
    s_att[kMaxF + i] = (att && i < p.F) ? p.att_dst[i] : 0.f;
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
      if (p.w_resident) {
        mbar_expect_tx(wfull, uint32_t(p.nkb * b_bytes));
        for (int kb = 0; kb < p.nkb; ++kb) tma_load_2d(w_res + kb * b_bytes, &map_w, wfull, kb * kBK, 0);
      }
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x) {
        for (int kb = 0; kb < p.nkb; ++kb) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], uint32_t(stage_bytes));
          unsigned char* dst = stages + s * stage_bytes;
          tma_load_2d(dst, &map_x, &full[s], kb * kBK, tile * kBM);
          if (!p.w_resident) tma_load_2d(dst + a_bytes, &map_w, &full[s], kb * kBK, 0);
          ++it;
        }
      }
      if (!ok) {
        // Let the copies still in flight land before the CTA goes away.
        for (int j = it > S ? it - S : 0; j < it; ++j)
          mbar_wait(&full[j % S], (j / S) & 1, abort, false);
        if (p.w_resident) mbar_wait(wfull, 0, abort, false);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(p.N16);
      int it = 0, t_iter = 0;
      bool ok = !p.w_resident || mbar_wait(wfull, 0, abort);
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x, ++t_iter) {
        const int b = t_iter & 1;
        if (!mbar_wait(&tempty[b], ((t_iter >> 1) & 1) ^ 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b) * kAccStride;
        for (int kb = 0; kb < p.nkb; ++kb) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + s * stage_bytes);
          const uint32_t b_addr =
              p.w_resident ? smem_u32(w_res + kb * b_bytes) : a_addr + uint32_t(a_bytes);
          const uint64_t adesc = sw128_desc(a_addr);
          const uint64_t bdesc = sw128_desc(b_addr);
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
    // Epilogue: TMEM lanes 32*(warp%4) .. +31, column group (warp-2)/4.
    const int q = warp & 3;
    const int group = (warp - 2) >> 2;
    const int c_begin = group * p.cs;
    const int c_end = min(p.N16, c_begin + p.cs);
    const int pass_cols = p.h_bf16 ? 64 : 32;  // 128 bytes of output per row
    unsigned char* box = s_stage + (warp - 2) * kBoxBytes;
    // The group starts on a head boundary (the host splits at whole heads).
    const bool multi_head = att && p.H > 1;
    const int hd0 = multi_head ? c_begin / p.C : 0;
    const int head_end0 = multi_head ? (hd0 + 1) * p.C : INT_MAX;
    int t_iter = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++t_iter) {
      const int b = t_iter & 1;
      if (!mbar_wait(&tfull[b], (t_iter >> 1) & 1, abort)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(b) * kAccStride;
      const int row0 = tile * kBM + q * 32;
      const int64_t row = int64_t(row0) + lane;
      float ps[4] = {0.f, 0.f, 0.f, 0.f}, pd[4] = {0.f, 0.f, 0.f, 0.f};
      int cur = hd0, head_end = head_end0;
      for (int c0 = c_begin; c0 < c_end; c0 += pass_cols) {
        const int width = min(pass_cols, c_end - c0);
        // the store that last read this box (the previous pass) is done reading
        if (lane == 0) bulk_wait_read_0();
        __syncwarp();
        if (p.h_bf16) {
          switch (width) {
            case 64: epi_pass<64, true>(p, &map_h, taddr, c0, row, row0, box, s_att, att, ps, pd, cur, head_end, lane); break;
            case 48: epi_pass<48, true>(p, &map_h, taddr, c0, row, row0, box, s_att, att, ps, pd, cur, head_end, lane); break;
            case 32: epi_pass<32, true>(p, &map_h, taddr, c0, row, row0, box, s_att, att, ps, pd, cur, head_end, lane); break;
            default: epi_pass<16, true>(p, &map_h, taddr, c0, row, row0, box, s_att, att, ps, pd, cur, head_end, lane); break;
          }
        } else {
          if (width == 32)
            epi_pass<32, false>(p, &map_h, taddr, c0, row, row0, box, s_att, att, ps, pd, cur, head_end, lane);
          else
            epi_pass<16, false>(p, &map_h, taddr, c0, row, row0, box, s_att, att, ps, pd, cur, head_end, lane);
        }
      }
      if (att && c_begin < c_end) att_flush(p, row, cur, ps, pd);
      // Accumulator fully read: hand it back to the MMA warp.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    // Every store has finished with shared memory (and global memory) before
    // the CTA can go away.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
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

// 2-D tensor map: inner dim `inner` (elements), `rows` rows of `ld`
// elements, box box_inner x box_rows, 128-byte swizzle, zero fill out of
// bounds on loads, clipping on stores.
bool make_map(EncodeTiledFn enc, CUtensorMap* map, const void* base, int64_t inner,
              int64_t rows, int64_t ld, int box_rows, int box_inner = kBK,
              CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, int esize = 2) {
  const cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * cuuint64_t(esize)};
  const cuuint32_t box[2] = {cuuint32_t(box_inner), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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
  const bool h_bf16 = h_dtype == GNNC_BF16;
  const int h_esize = h_bf16 ? 2 : 4;
  const int pass_cols = 128 / h_esize;
  // Bulk stores cover whole 16-byte chunks of a row: columns [0, Fs); the
  // epilogue writes the few columns of a partial last chunk itself.
  const int Fs = int(F * h_esize / 16 * 16 / h_esize);
  if (Fs == 0) return kProjTcDeclined;
  CUtensorMap map_x, map_w, map_h;
  if (att && H > kMaxF / 16) return kProjTcDeclined;
  if (!make_map(enc, &map_x, x, K, N, ldx, kBM) || !make_map(enc, &map_w, w, K, F, ldw, N16) ||
      !make_map(enc, &map_h, h, Fs, N, ldh, kBoxRows, pass_cols,
                h_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                h_esize))
    return kProjTcDeclined;
  // Column split between the epilogue's column groups: about a quarter of the
  // columns each, rounded up to whole 128-byte passes and, with attention, to
  // whole heads (a head's dot products stay in one warp).
  int unit = pass_cols;
  if (att && H > 1) {
    const int c = int(C);
    int l = unit;
    while (l % c) l += unit;  // lcm(pass_cols, C)
    unit = l;
  } else if (att) {
    unit = N16;
  }
  int cs = ((N16 + kEpiGroups - 1) / kEpiGroups + unit - 1) / unit * unit;
  if (cs < unit) cs = unit;

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
  p.cs = cs;
  p.Fs = Fs;
  p.h = h;
  p.h_bf16 = h_bf16;
  p.ldh = ldh;
  p.asrc = asrc;
  p.adst = adst;
  p.err = ctx->dev_words + 3;

  const size_t a_bytes = size_t(kBM) * kBK * 2;
  const size_t b_bytes = size_t(N16) * kBK * 2;
  if (a_bytes % 1024 || b_bytes % 1024) return kProjTcDeclined;  // stage alignment
  p.w_resident = size_t(p.nkb) * b_bytes <= size_t(kResidentWBytes) ? 1 : 0;
  p.stages = p.w_resident ? kStagesResident : kStagesStream;
  const size_t stage_bytes = p.w_resident ? a_bytes : a_bytes + b_bytes;
  size_t smem = 1024 + (p.w_resident ? size_t(p.nkb) * b_bytes : 0) + size_t(p.stages) * stage_bytes +
                kStagingBytes + kBarrierBytes + 16 + 2 * kMaxF * sizeof(float);
  // At least 120 KB, so two CTAs never share an SM (each takes all 512 TMEM columns).
  if (smem < 120 * 1024) smem = 120 * 1024;
  int max_smem = 0;
  GNNC_CUDA_TRY(ctx, cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                            ctx->device));
  if (smem > size_t(max_smem)) return kProjTcDeclined;
  GNNC_CUDA_TRY(ctx, cudaFuncSetAttribute(proj_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int grid = p.n_tiles < ctx->num_sms ? p.n_tiles : ctx->num_sms;
  proj_tc_kernel<<<grid, kThreads, smem, ctx->stream>>>(map_x, map_w, map_h, p);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}

}  // namespace gnnc

extern "C" int gnnc_wait_selftest(gnnc_ctx_t* ctx, int64_t limit_ns) {
  if (!ctx) return GNNC_ERR_INVALID;
  GNNC_CHECK_ARG(ctx, limit_ns > 0 && limit_ns <= int64_t(kWaitNs),
                 "gnnc_wait_selftest: limit must be in (0, %llu] ns", kWaitNs);
  GNNC_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  wait_selftest_kernel<<<1, 32, 0, ctx->stream>>>(ctx->dev_words + 3,
                                                  (unsigned long long)limit_ns);
  GNNC_CUDA_TRY(ctx, cudaGetLastError());
  return GNNC_OK;
}
