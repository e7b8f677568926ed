// Fused attention of the YOLO26-N PSA block on tcgen05 / TMEM.
//
// The exported program spells one attention head as
//   S  = bmm(Q, K^T)                    Q [n, L, dq], K^T [n, dq, L]
//   P  = softmax(S, dim = -1)           (view_copy / _softmax)
//   O^T = bmm(V^T, P^T)                 V^T [n, dv, L], P^T via permute_copy
// (src/shaders/bmm, softmax, permute). This kernel computes O^T without
// materialising S, P or P^T. One CTA per head:
//   1. all of K and V are staged once in shared memory in the canonical
//      K-major no-swizzle operand layout (zero padded to Lp, a multiple of
//      16 keys): V^T rows are already K-major over keys (16-byte copies), K^T
//      is transposed 8x8 in registers from 16-byte loads;
//   2. per block of 128 queries: the Q block is staged, S[128 x Lp] = Q K^T
//      goes into TMEM (M = 128, N <= 256 per MMA, K = 16);
//   3. eight warps (two per TMEM lane quadrant, each half of the key
//      columns, one query row per thread) take the row maximum (halves
//      combined through shared memory), write p = exp(s - max) as fp16 into
//      shared memory (the A operand of the second product) and sum the row;
//   4. O[128 x dv] = P V into TMEM;
//   5. the same warps divide by the row sums and store O^T (each warp store
//      is 32 consecutive queries of one channel), half the channels each.
// Softmax runs in fp32 on fp32 scores, both products accumulate in fp32;
// the reference computes all three steps in f16 (bmm-64x64-f16,
// softmax-last-dim-f16.wgsl.ts).
#include <mutex>

#include "internal.h"
#include "tcgen05.h"

namespace wgx {

namespace {

constexpr int AT_SWARPS = 8;                        // softmax / epilogue warps
constexpr int AT_THREADS = 32 * (AT_SWARPS + 1);    // + the TMEM / MMA warp
constexpr int AT_MMA_WARP = AT_SWARPS;
constexpr int AT_QB = 128;        // queries per block (MMA M)
constexpr uint32_t AT_TMEM_COLS = 512;
// dynamic shared memory limit (the 227 KB per-block maximum less the
// kernel's static barriers and slack)
constexpr uint32_t kAttnSmemMax = 226 * 1024;

struct AttnGeom {
  int n, L, Lp, dq, dv, vec;            // vec: L % 8 == 0 and aligned rows
  uint32_t q_off, k_off, p_off, v_off, red_off;  // shared-memory offsets (bytes)
  uint32_t *err;
};

__device__ __forceinline__ void mma_commit_arrive(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// barrier among the softmax / epilogue warps only
__device__ __forceinline__ void softmax_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(AT_SWARPS * 32) : "memory");
}
// transpose helper: position k of 8 rows of 8 fp16 (one uint4 per row)
__device__ __forceinline__ uint4 column8(const uint4 *rows, int k) {
  const uint32_t sel = (k & 1) ? 0x7632u : 0x5410u;
  uint32_t w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint4 &v = rows[e];
    w[e] = (k >> 1) == 0 ? v.x : (k >> 1) == 1 ? v.y : (k >> 1) == 2 ? v.z : v.w;
  }
  return make_uint4(__byte_perm(w[0], w[1], sel), __byte_perm(w[2], w[3], sel),
                    __byte_perm(w[4], w[5], sel), __byte_perm(w[6], w[7], sel));
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    attention_kernel(const AttnGeom g, const __half *__restrict__ Q, const __half *__restrict__ KT,
                     const __half *__restrict__ VT, __half *__restrict__ OT) {
  extern __shared__ __align__(128) uint8_t at_smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(at_smem_raw) + 127) & ~uintptr_t(127));
  uint8_t *sQ = smem + g.q_off, *sK = smem + g.k_off, *sP = smem + g.p_off, *sV = smem + g.v_off;
  float *red = reinterpret_cast<float *>(smem + g.red_off);  // [2 halves][128 rows] x {max, sum}
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int head = blockIdx.x;
  const __half *q = Q + size_t(head) * g.L * g.dq;
  const __half *kt = KT + size_t(head) * g.dq * g.L;
  const __half *vt = VT + size_t(head) * g.dv * g.L;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == AT_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(AT_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // ---- K and V once (K-major: [8-element chunk][row][8], 16 B per row)
  const int qc = g.dq / 8, kg = g.Lp / 8;
  for (int i = threadIdx.x; i < qc * kg; i += AT_THREADS) {
    const int c = i / kg, j0 = (i % kg) * 8;  // dq chunk c, keys j0 .. j0 + 7
    uint4 rows[8];
    if (g.vec) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        rows[e] = j0 < g.L ? *reinterpret_cast<const uint4 *>(kt + size_t(c * 8 + e) * g.L + j0)
                           : make_uint4(0u, 0u, 0u, 0u);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        __align__(16) __half h[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          h[k] = j0 + k < g.L ? kt[size_t(c * 8 + e) * g.L + j0 + k] : __float2half_rn(0.f);
        rows[e] = *reinterpret_cast<const uint4 *>(h);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
      *reinterpret_cast<uint4 *>(sK + (size_t(c) * g.Lp + j0 + k) * 16) = column8(rows, k);
  }
  for (int i = threadIdx.x; i < kg * g.dv; i += AT_THREADS) {
    const int c = i / g.dv, ch = i % g.dv;
    uint4 v;
    if (g.vec) {
      v = c * 8 < g.L ? *reinterpret_cast<const uint4 *>(vt + size_t(ch) * g.L + c * 8)
                      : make_uint4(0u, 0u, 0u, 0u);
    } else {
      __align__(16) __half h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = c * 8 + e;
        h[e] = j < g.L ? vt[size_t(ch) * g.L + j] : __float2half_rn(0.f);
      }
      v = *reinterpret_cast<const uint4 *>(h);
    }
    *reinterpret_cast<uint4 *>(sV + (size_t(c) * g.dv + ch) * 16) = v;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t o_col = uint32_t(g.Lp);  // O after the Lp score columns
  bool ok = true;
  // softmax / epilogue roles: rows of lane quadrant qd, column half hf
  const int qd = warp & 3, hf = warp >> 2;
  const int r = qd * 32 + lane;
  const int nsc = (g.Lp + 31) / 32, sc0 = hf ? (nsc + 1) / 2 : 0, sc1 = hf ? nsc : (nsc + 1) / 2;
  const int noc = g.dv / 32, oc0 = hf ? (noc + 1) / 2 : 0, oc1 = hf ? noc : (noc + 1) / 2;
  const uint32_t lane_base = tmem + (uint32_t(qd * 32) << 16);
  const int nqb = (g.L + AT_QB - 1) / AT_QB;

  for (int qb = 0; qb < nqb; ++qb) {
    const int q0 = qb * AT_QB;
    // ---- Q block
    for (int i = threadIdx.x; i < qc * AT_QB; i += AT_THREADS) {
      const int c = i / AT_QB, rr = i % AT_QB;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (q0 + rr < g.L) v = *reinterpret_cast<const uint4 *>(q + size_t(q0 + rr) * g.dq + c * 8);
      *reinterpret_cast<uint4 *>(sQ + (size_t(c) * AT_QB + rr) * 16) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- S = Q K^T
    if (warp == AT_MMA_WARP && lane == 0) {
      for (int n0 = 0; n0 < g.Lp; n0 += 256) {
        const int nn = min(256, g.Lp - n0);
        const uint32_t idesc = (1u << 4) | (uint32_t(nn >> 3) << 17) | (uint32_t(AT_QB >> 4) << 24);
        for (int ks = 0; ks < g.dq / 16; ++ks) {
          const uint64_t a = kmajor_desc(smem_u32(sQ) + uint32_t(ks * 2 * AT_QB * 16), AT_QB * 16);
          const uint64_t b =
              kmajor_desc(smem_u32(sK) + uint32_t((ks * 2 * g.Lp + n0) * 16), uint32_t(g.Lp) * 16);
          mma_f16(tmem + uint32_t(n0), a, b, idesc, ks > 0);
        }
      }
      mma_commit_arrive(smem_u32(&bars[0]));
    }
    // ---- softmax rows -> P (fp16, K-major over keys)
    float row_sum = 1.f;
    if (warp < AT_SWARPS) {
      if (!mbar_wait(smem_u32(&bars[0]), qb & 1)) {
        if (lane == 0) atomicOr(g.err, kErrMmaTimeout);
        ok = false;
      }
      tc_fence_after();
      float s[32];
      float mx = -INFINITY;
      for (int sc = sc0; sc < sc1; ++sc) {
        const int c0 = sc * 32;
        tmem_ld32(lane_base + uint32_t(c0), s);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < g.L) mx = fmaxf(mx, s[j]);
      }
      red[hf * AT_QB + r] = mx;
      softmax_bar();
      mx = fmaxf(mx, red[(1 - hf) * AT_QB + r]);
      float sum = 0.f;
      for (int sc = sc0; sc < sc1; ++sc) {
        const int c0 = sc * 32;
        tmem_ld32(lane_base + uint32_t(c0), s);
        uint32_t pw[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = c0 + j < g.L ? __expf(s[j] - mx) : 0.f;
          const float p1 = c0 + j + 1 < g.L ? __expf(s[j + 1] - mx) : 0.f;
          sum += p0 + p1;
          const __half2 h = __floats2half2_rn(p0, p1);
          pw[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (c0 + 8 * k < g.Lp)
            *reinterpret_cast<uint4 *>(sP + (size_t((c0 >> 3) + k) * AT_QB + r) * 16) =
                make_uint4(pw[4 * k], pw[4 * k + 1], pw[4 * k + 2], pw[4 * k + 3]);
      }
      red[2 * AT_QB + hf * AT_QB + r] = sum;
      softmax_bar();
      row_sum = sum + red[2 * AT_QB + (1 - hf) * AT_QB + r];
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- O = P V
    if (warp == AT_MMA_WARP && lane == 0) {
      const uint32_t idesc = (1u << 4) | (uint32_t(g.dv >> 3) << 17) | (uint32_t(AT_QB >> 4) << 24);
      for (int ks = 0; ks < g.Lp / 16; ++ks) {
        const uint64_t a = kmajor_desc(smem_u32(sP) + uint32_t(ks * 2 * AT_QB * 16), AT_QB * 16);
        const uint64_t b =
            kmajor_desc(smem_u32(sV) + uint32_t(ks * 2 * g.dv * 16), uint32_t(g.dv) * 16);
        mma_f16(tmem + o_col, a, b, idesc, ks > 0);
      }
      mma_commit_arrive(smem_u32(&bars[1]));
    }
    // ---- epilogue: O / sum -> O^T, half the channel chunks per warp
    if (warp < AT_SWARPS) {
      if (!mbar_wait(smem_u32(&bars[1]), qb & 1)) {
        if (lane == 0) atomicOr(g.err, kErrEpilogueTimeout);
        ok = false;
      }
      tc_fence_after();
      const float inv = 1.f / row_sum;
      __half *ot = OT + size_t(head) * g.dv * g.L + q0 + r;
      float o[32];
      for (int oc = oc0; oc < oc1; ++oc) {
        const int c0 = oc * 32;
        tmem_ld32(lane_base + o_col + uint32_t(c0), o);
        if (ok && q0 + r < g.L) {
#pragma unroll
          for (int j = 0; j < 32; ++j) ot[size_t(c0 + j) * g.L] = __float2half_rn(o[j] * inv);
        }
      }
    }
    // every thread leaves together (the softmax barriers count all 8 warps)
    if (__syncthreads_or(!ok)) break;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == AT_MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(AT_TMEM_COLS)
                 : "memory");
  }
}

}  // namespace

bool attention_supported(int64_t n, int64_t L, int64_t dq, int64_t dv) {
  if (n < 1 || L < 1 || dq % 16 || dv % 32 || dq < 16 || dv < 32 || dv > 256) return false;
  const int64_t Lp = (L + 15) / 16 * 16;
  if (Lp + dv > AT_TMEM_COLS) return false;
  const int64_t bytes = (AT_QB * dq + Lp * dq + AT_QB * Lp + Lp * dv) * 2 + 4 * AT_QB * 4 + 128;
  return bytes <= int64_t(kAttnSmemMax) && n < (1ll << 31);
}

void launch_attention(const __half *Q, const __half *KT, const __half *VT, __half *OT, int64_t n,
                      int64_t L, int64_t dq, int64_t dv, cudaStream_t stream) {
  if (!attention_supported(n, L, dq, dv)) fail("attention: shape not supported");
  AttnGeom g{};
  g.n = int(n);
  g.L = int(L);
  g.Lp = int((L + 15) / 16 * 16);
  g.dq = int(dq);
  g.dv = int(dv);
  g.q_off = 0;
  g.k_off = g.q_off + uint32_t(AT_QB * dq * 2);
  g.p_off = g.k_off + uint32_t(g.Lp * dq * 2);
  g.v_off = g.p_off + uint32_t(AT_QB * g.Lp * 2);
  g.red_off = g.v_off + uint32_t(g.Lp * dv * 2);
  // 16-byte row loads of K^T and V^T need L % 8 == 0 and aligned heads
  g.vec = L % 8 == 0 && ((reinterpret_cast<uintptr_t>(KT) | reinterpret_cast<uintptr_t>(VT)) & 15) == 0;
  if ((reinterpret_cast<uintptr_t>(Q) & 15) != 0) fail("attention: Q must be 16-byte aligned");
  // at least 120 KB so that one CTA is resident per SM and its 512-column
  // TMEM allocation never waits on another CTA's
  const uint32_t smem = max(g.red_off + uint32_t(4 * AT_QB * 4) + 128, 120u * 1024u);
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  g.err = device_error_word(dev);
  {
    // once per device; host threads share the table, so under a lock
    static std::mutex setup_mu;
    static bool attr_set[64] = {};
    std::lock_guard<std::mutex> lock(setup_mu);
    if (dev >= 64 || !attr_set[dev]) {
      check_cuda(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(kAttnSmemMax)),
                 "attention smem attr");
      if (dev < 64) attr_set[dev] = true;
    }
  }
  const unsigned grid = unsigned(n);  // one CTA per head, looping over query blocks
  int th = timer_begin("attention_kernel", stream);
  attention_kernel<<<grid, AT_THREADS, smem, stream>>>(g, Q, KT, VT, OT);
  check_cuda(cudaGetLastError(), "attention launch");
  timer_end(th, stream);
}

}  // namespace wgx
