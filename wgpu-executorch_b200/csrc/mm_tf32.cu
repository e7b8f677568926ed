// fp32 aten.mm on the tcgen05 tensor cores: 3xTF32 (sm_100a).
//
// Replaces src/shaders/mm/mm-64x64.wgsl.ts:8-115 (fp32 64x64 tiles, FMA
// chain) for fp32 matrices whose sizes fit the tiling below; other shapes
// keep the FFMA kernel (conv_simt.cu). C = A B, A [M,K], B [K,N], C [M,N],
// row-major, fp32 accumulation.
//
// Each fp32 operand is split into a TF32 head and a tail: hi = x with the
// 13 low mantissa bits cleared (exactly what a TF32 multiply reads), lo =
// x - hi (exact in fp32). C += A_hi B_hi + A_hi B_lo + A_lo B_hi in fp32 on
// tcgen05.mma kind::tf32; only the A_lo B_lo term (2^-22 of |a b| at most)
// and the TF32 reading of the tails (2^-11 of them) are dropped, so the
// result stays close to the FFMA product (tested at 1e-4 against both
// oracles; measured 5e-6 at 1024^3, 2e-5 at 2048^3, against 1e-6 / 2e-6
// for FFMA).
//
// Tiling: one 128 x 128 output tile per cluster of S CTAs (S = 1..8, all
// clusters resident at once); CTA r of the cluster multiplies K slice r
// into its own TMEM accumulator (128 lanes x 128 fp32 columns), 32 K at a
// time through two operand buffers:
// all 256 threads load the A and B slices with 16-byte loads, split them and
// store the four operands in the K-major no-swizzle layout (rows of 4 fp32 =
// 16 bytes, one plane per 4 K columns; B is transposed on the way), one
// thread issues the 4 K steps x 3 MMAs (M 128, N 128, K 8); the next
// round's loads are in flight meanwhile. The partial tiles then go to
// shared memory and CTA r sums rows r*128/S.. of all S partials in rank order
// through distributed shared memory (deterministic, no atomics) and stores
// them. The MMA completion wait is bounded (device error word on expiry).
#include <cstdlib>
#include <mutex>

#include "internal.h"
#include "tcgen05.h"

namespace wgx {

namespace {

constexpr int kTile = 128;
constexpr int kKB = 32;                        // K per round
constexpr int kThreads = 256;
constexpr uint32_t kOpBytes = kTile * kKB * 4;  // one operand of one round: 16 KB
constexpr uint32_t kBufBytes = 4 * kOpBytes;    // A_hi, A_lo, B_hi, B_lo of one round
constexpr int kPitch = kTile + 4;              // partial tile row pitch (floats)
constexpr uint32_t kSmem = 2 * kBufBytes + 1024 + 64;

// WGX_MM_TF32: 0 = never, 1 (default) = products of at least 2^29
// multiply-adds, 2 = every size the tiling takes
int tf32_mode() {
  static const int mode = [] {
    const char *e = std::getenv("WGX_MM_TF32");
    return (e && e[0] >= '0' && e[0] <= '2') ? e[0] - '0' : 1;
  }();
  return mode;
}

__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ float4 tf32_head(float4 v) {
  const uint32_t m = 0xffffe000u;
  return make_float4(__uint_as_float(__float_as_uint(v.x) & m),
                     __uint_as_float(__float_as_uint(v.y) & m),
                     __uint_as_float(__float_as_uint(v.z) & m),
                     __uint_as_float(__float_as_uint(v.w) & m));
}

__device__ __forceinline__ float f4_get(const float4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    mm_tf32_kernel(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C,
                   int M, int N, int K, int kslice, uint32_t *err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // operands: A_hi, A_lo, B_hi, B_lo; each 16 planes (4 K columns) of 128
  // rows x 16 bytes
  uint8_t *ops = smem;
  float *part = reinterpret_cast<float *>(smem);  // partial tile, after the MMAs
  // done[b]: the MMAs of the last round staged in buffer b completed
  uint64_t *done = reinterpret_cast<uint64_t *>(smem + 2 * kBufBytes);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 2);

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int S = gridDim.z, rank = blockIdx.z;
  const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
  const int kb = rank * kslice, ke = min(K, kb + kslice);

  if (tid == 0) {
    mbar_init(smem_u32(&done[0]), 1);
    mbar_init(smem_u32(&done[1]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(128)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint32_t idesc = (1u << 4)                  // D = f32
                         | (2u << 7) | (2u << 10)   // A, B = tf32
                         | (uint32_t(kTile >> 3) << 17) | (uint32_t(kTile >> 4) << 24);
  const uint32_t plane = kTile * 16;  // 2 KB: one plane of 4 K columns
  // Rounds of 32 K, two operand buffers: the global loads of round r + 1
  // go into registers right after round r is staged, so their latency
  // overlaps round r's MMAs (and round r - 1's, still in flight).
  constexpr int kATasks = (kTile / 8) * (kKB / 16) / (kThreads / 32);  // 4 per warp
  constexpr int kBTasks = (kKB / 4) * (kTile / 4) / kThreads;          // 1 per thread
  float4 av[kATasks], bv[kBTasks][4];
  auto load_round = [&](int k0) {
#pragma unroll
    for (int i = 0; i < kATasks; ++i) {
      const int t = warp + i * (kThreads / 32);
      const int r = (t % (kTile / 8)) * 8 + (lane & 7), q = (t / (kTile / 8)) * 4 + (lane >> 3);
      av[i] = *reinterpret_cast<const float4 *>(A + size_t(m0 + r) * K + k0 + 4 * q);
    }
#pragma unroll
    for (int i = 0; i < kBTasks; ++i) {
      const int t = tid + i * kThreads;
      const int nq = t % (kTile / 4), q = t / (kTile / 4);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        bv[i][j] = *reinterpret_cast<const float4 *>(B + size_t(k0 + 4 * q + j) * N + n0 + 4 * nq);
    }
  };
  // A: a warp task = 8 rows x 16 columns (lane = quad * 8 + row: 8 lanes
  // store 8 consecutive 16-byte rows of one plane); B: a thread task = 4 K
  // rows x 4 columns, transposed to rows of 4 K
  auto stage_round = [&](uint8_t *ops) {
#pragma unroll
    for (int i = 0; i < kATasks; ++i) {
      const int t = warp + i * (kThreads / 32);
      const int r = (t % (kTile / 8)) * 8 + (lane & 7), q = (t / (kTile / 8)) * 4 + (lane >> 3);
      const float4 v = av[i], h = tf32_head(v);
      const float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      *reinterpret_cast<float4 *>(ops + 0 * kOpBytes + q * plane + r * 16) = h;
      *reinterpret_cast<float4 *>(ops + 1 * kOpBytes + q * plane + r * 16) = l;
    }
#pragma unroll
    for (int i = 0; i < kBTasks; ++i) {
      const int t = tid + i * kThreads;
      const int nq = t % (kTile / 4), q = t / (kTile / 4);
      const float4 *v = bv[i];
      // column c of the 4x4 block goes to row 4 nq + c; lanes take the
      // columns in an order rotated by (nq / 2) % 4, so the rows that the 8
      // lanes of one store wavefront write differ mod 8 (distinct banks)
      const int rot = (nq >> 1) & 3;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int cc = (c + rot) & 3;
        const float4 c4 = make_float4(f4_get(v[0], cc), f4_get(v[1], cc), f4_get(v[2], cc),
                                      f4_get(v[3], cc));
        const float4 h = tf32_head(c4);
        const float4 l = make_float4(c4.x - h.x, c4.y - h.y, c4.z - h.z, c4.w - h.w);
        const int n = 4 * nq + cc;
        *reinterpret_cast<float4 *>(ops + 2 * kOpBytes + q * plane + n * 16) = h;
        *reinterpret_cast<float4 *>(ops + 3 * kOpBytes + q * plane + n * 16) = l;
      }
    }
  };
  const int rounds = (ke - kb) / kKB;
  if (rounds > 0) load_round(kb);
  for (int rd = 0; rd < rounds; ++rd) {
    const int buf = rd & 1;
    uint8_t *ops = smem + size_t(buf) * kBufBytes;
    if (rd >= 2) {
      // the MMAs of round rd - 2 have read this buffer
      if (!mbar_wait(smem_u32(&done[buf]), uint32_t((rd - 2) >> 1) & 1))
        atomicOr(err, kErrMmaTimeout);
      tc_fence_after();
    }
    stage_round(ops);
    if (rd + 1 < rounds) load_round(kb + (rd + 1) * kKB);
    // generic-proxy stores -> visible to the tensor cores
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t base = smem_u32(ops);
#pragma unroll
      for (int ks = 0; ks < kKB / 8; ++ks) {
        // K step ks: planes 2ks, 2ks+1 (LBO = one plane), rows 16 B apart
        const uint32_t off = uint32_t(ks) * 2u * plane;
        const uint64_t ah = kmajor_desc(base + 0 * kOpBytes + off, plane);
        const uint64_t al = kmajor_desc(base + 1 * kOpBytes + off, plane);
        const uint64_t bh = kmajor_desc(base + 2 * kOpBytes + off, plane);
        const uint64_t bl = kmajor_desc(base + 3 * kOpBytes + off, plane);
        mma_tf32(tmem, al, bh, idesc, (rd > 0 || ks > 0) ? 1u : 0u);
        mma_tf32(tmem, ah, bl, idesc, 1u);
        mma_tf32(tmem, ah, bh, idesc, 1u);
      }
      mma_commit(smem_u32(&done[buf]));
    }
  }
  // all MMAs complete before the partial tile leaves TMEM (the last commit
  // covers every MMA issued before it)
  const int round = rounds;
  if (rounds > 0 &&
      !mbar_wait(smem_u32(&done[(rounds - 1) & 1]), uint32_t((rounds - 1) >> 1) & 1))
    atomicOr(err, kErrMmaTimeout);
  tc_fence_after();
  __syncthreads();
  if (warp < 4) {
    // lane quadrant warp: rows 32*warp + lane, 128 columns
    const int row = warp * 32 + lane;
    for (int c0 = 0; c0 < kTile; c0 += 32) {
      float v[32];
      if (round > 0) {
        tmem_ld32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c0), v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4 *>(part + row * kPitch + c0 + j) =
            make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128)
                 : "memory");
  cluster_sync();
  // CTA `rank` sums rows [rows_per * rank, ...) of the S partials
  const int rows_per = kTile / S;
  const uint32_t part_base = smem_u32(part);
  for (int e = tid; e < rows_per * (kTile / 4); e += kThreads) {
    const int r = rank * rows_per + e / (kTile / 4), c = (e % (kTile / 4)) * 4;
    const uint32_t local = part_base + uint32_t(r * kPitch + c) * 4u;
    // all S partials requested before the first add (rank order kept)
    float4 x[8];
#pragma unroll
    for (int src = 0; src < 8; ++src) {
      x[src] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (src < S) {
        uint32_t addr;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(local), "r"(src));
        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(x[src].x), "=f"(x[src].y), "=f"(x[src].z), "=f"(x[src].w)
                     : "r"(addr));
      }
    }
    float4 sum = x[0];
#pragma unroll
    for (int src = 1; src < 8; ++src) {
      sum.x += x[src].x;
      sum.y += x[src].y;
      sum.z += x[src].z;
      sum.w += x[src].w;
    }
    *reinterpret_cast<float4 *>(C + size_t(m0 + r) * N + n0 + c) = sum;
  }
  // no CTA leaves while another may still read its partial
  cluster_sync();
}

}  // namespace

// Sizes the tiling takes: M, N multiples of 128, K a multiple of 32, every
// 16-byte aligned; and products of at least 2^29 multiply-adds (B200, L2
// flushed: 512^3 17.4 us here, 18.0 us FFMA, which also rounds less;
// 1024^3 34 against 73 us; 2048^3 191 against 447 us).
bool mm_tf32_supported(const void *a, const void *b, const void *c, int64_t M, int64_t N,
                       int64_t K) {
  if (tf32_mode() == 0) return false;
  if (tf32_mode() == 1 && double(M) * double(N) * double(K) < double(1ll << 29)) return false;
  if (M < kTile || N < kTile || K < kKB || M % kTile || N % kTile || K % kKB) return false;
  if (M > (1 << 20) || N > (1 << 20) || K > (1 << 20)) return false;
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
           reinterpret_cast<uintptr_t>(c)) &
          15) == 0;
}

void mm_tf32_run(const float *a, const float *b, float *c, int64_t M, int64_t N, int64_t K,
                 int n_sm, cudaStream_t stream) {
  const int64_t gx = N / kTile, gy = M / kTile, tiles = gx * gy;
  if (gy > 65535) fail("aten.mm.default: matrix too large");
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  static_assert(kTile * kPitch * 4 <= 2 * kBufBytes, "partial tile fits the operand space");
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(gx), unsigned(gy), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // clusters of S CTAs that can be resident at once (per device and S; a
  // cluster needs S SMs of one GPC, so on B200 only 15 clusters of 8 fit)
  static std::mutex mu;
  static bool attr_set[64] = {};
  static int max_clusters[64][4] = {};
  {
    // (before any launch or occupancy query on this device)
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 64 || !attr_set[dev]) {
      check_cuda(cudaFuncSetAttribute(mm_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(kSmem)),
                 "mm tf32 smem attr");
      if (dev < 64) attr_set[dev] = true;
    }
  }
  auto resident_clusters = [&](int S) {
    std::lock_guard<std::mutex> lock(mu);
    const int si = S == 1 ? 0 : S == 2 ? 1 : S == 4 ? 2 : 3;
    if (dev < 64 && max_clusters[dev][si]) return max_clusters[dev][si];
    cudaLaunchConfig_t q = cfg;
    q.gridDim.z = unsigned(S);
    attr[0].val.clusterDim.z = unsigned(S);
    int n = 0;
    check_cuda(cudaOccupancyMaxActiveClusters(&n, mm_tf32_kernel, &q), "mm tf32 cluster occupancy");
    if (dev < 64) max_clusters[dev][si] = n;
    return n;
  };
  // split K over a cluster of S CTAs while the grid stays within the SMs,
  // every cluster is resident at once (one wave) and every slice keeps
  // whole 64-column rounds
  int S = 1;
  while (S < 8 && tiles * S * 2 <= n_sm && K % (2 * S * kKB) == 0 &&
         tiles <= resident_clusters(2 * S))
    S *= 2;
  const int kslice = int(K / S);
  cfg.gridDim.z = unsigned(S);
  attr[0].val.clusterDim.z = unsigned(S);
  int th = timer_begin("mm_tf32_kernel", stream);
  check_cuda(cudaLaunchKernelEx(&cfg, mm_tf32_kernel, a, b, c, int(M), int(N), int(K), kslice,
                                device_error_word(dev)),
             "mm tf32 launch");
  timer_end(th, stream);
}

}  // namespace wgx
