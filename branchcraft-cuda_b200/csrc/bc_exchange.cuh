// The context-split merge fused with its exchange over peer memory: one
// kernel per rank reduces the rank's key splits of each row to one partial
// state (M, L, unnormalised accumulator), writes that state straight into
// every rank's exchange buffer over NVLink (plain peer stores through CUDA
// IPC mappings; no multicast, no TMA on peer memory), raises a flag per row
// block in every rank's buffer, waits (bounded) for the other ranks' flags of
// the same row block in its own buffer, and merges the world's states into
// the output. It replaces merge_to_partial + an NCCL all-gather +
// merge_gathered: the exchange costs one NVLink store round trip instead of a
// collective launch.
//
// Exchange buffer of a rank (bc_exchange_bytes): for each step parity p (the
// epoch's low bit: a rank writes step e + 1's states while a slower peer may
// still read step e's), states [p][world][rows][Exch<D>::kStride floats: M, L,
// -, -, accumulator[D]], then flags [p][world][blocks] holding the epoch whose
// states are complete. A rank can only reach step e + 2 after every peer has
// published step e + 1, which each does after finishing step e: the parity's
// slots are free again by then.
#pragma once

#include "bc_device.cuh"

namespace bc {

constexpr int kExchRowsPerBlock = 4;  // one warp per row, 4 warps per CTA

template <int D>
struct Exch {
  static constexpr int kStride = D + 4;  // floats per row state (16-byte rows)
  __host__ __device__ static size_t states_floats(int world, int rows) {
    return size_t(2) * world * rows * kStride;
  }
  __host__ __device__ static size_t flags_offset_bytes(int world, int rows) {
    return (states_floats(world, rows) * 4 + 255) & ~size_t(255);
  }
  static size_t bytes(int world, int rows) {
    const int blocks = (rows + kExchRowsPerBlock - 1) / kExchRowsPerBlock;
    return flags_offset_bytes(world, rows) + size_t(2) * world * blocks * 4;
  }
};

__device__ __forceinline__ void st_release_sys(unsigned* flag, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* flag) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
  return v;
}

// Local splits: partial s of row `row` at pml[(s * rows + row) * 2] (m in
// natural-log units, l) and pa[(s * rows + row) * D] (the reference's
// scratch layout). peers[w]: rank w's exchange buffer, mapped here.
template <int D>
__global__ void __launch_bounds__(32 * kExchRowsPerBlock)
    exchange_merge_kernel(int world, int rank, unsigned epoch, int splits, int rows,
                          const float* __restrict__ pml, const float* __restrict__ pa,
                          float* const* __restrict__ peers, float* __restrict__ out,
                          unsigned token, unsigned* err) {
  using X = Exch<D>;
  constexpr int R = D / 32;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kExchRowsPerBlock + (threadIdx.x >> 5);
  const int blocks = gridDim.x;
  const int par = int(epoch & 1u);
  if (threadIdx.x == 0) s_launch_token = token;
  grid_dependency_wait();  // the local partials of the preceding kernel are visible

  // 1. This rank's splits of the row -> one state (as merge_kernel TO_PARTIAL).
  float M = -INFINITY, L = 0.f, acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  if (row < rows) {
    for (int s = 0; s < splits; ++s) M = fmaxf(M, pml[(size_t(s) * rows + row) * 2]);
    if (M != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const size_t ml = (size_t(s) * rows + row) * 2;
        const float w = __expf(pml[ml] - M);
        L += w * pml[ml + 1];
        const float* a = pa + (size_t(s) * rows + row) * D;
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += w * a[r * 32 + lane];
      }
    }
    // 2. ... into slot `rank` of every rank's buffer (its own included).
    for (int w = 0; w < world; ++w) {
      float* st = peers[w] + ((size_t(par) * world + rank) * rows + row) * X::kStride;
      if (lane == 0) *reinterpret_cast<float2*>(st) = make_float2(M, L);
#pragma unroll
      for (int r = 0; r < R; ++r) st[4 + r * 32 + lane] = acc[r];
    }
  }
  // 3. This row block is published to every rank once all its rows are.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) {
    unsigned* flags = reinterpret_cast<unsigned*>(
        reinterpret_cast<uint8_t*>(peers[threadIdx.x]) + X::flags_offset_bytes(world, rows));
    st_release_sys(flags + (size_t(par) * world + rank) * blocks + blockIdx.x, epoch);
  }
  // 4. Wait (bounded) for every rank's states of this row block.
  __shared__ unsigned s_ok;
  if (threadIdx.x == 0) s_ok = 1u;
  __syncthreads();
  if (threadIdx.x < world) {
    const unsigned* flags = reinterpret_cast<const unsigned*>(
        reinterpret_cast<const uint8_t*>(peers[rank]) + X::flags_offset_bytes(world, rows));
    const unsigned* f = flags + (size_t(par) * world + threadIdx.x) * blocks + blockIdx.x;
    bool seen = ld_acquire_sys(f) == epoch;
    if (!seen) {
      const unsigned long long start = globaltimer_ns();
      for (;;) {
        __nanosleep(64);
        if (ld_acquire_sys(f) == epoch) {
          seen = true;
          break;
        }
        if (*reinterpret_cast<volatile unsigned*>(&g_abort_token) == token) break;
        if (globaltimer_ns() - start > kWaitLimitNs) {
          atomicExch(&g_abort_token, token);
          break;
        }
      }
    }
    if (!seen) {
      atomicAnd(&s_ok, 0u);
      atomicOr(err, kErrTimeout);
    }
  }
  __syncthreads();
  if (row >= rows) return;
  // 5. The world's states of the row -> the output (rank order: every rank
  // computes the same bits). Loads through L2: other GPUs wrote the states,
  // and this SM's L1 may still hold older copies of these lines.
  const float* own = peers[rank];
  float* o = out + size_t(row) * D;
  if (!s_ok) {
#pragma unroll
    for (int r = 0; r < R; ++r) o[r * 32 + lane] = 0.f;
    return;
  }
  float MM = -INFINITY;
  for (int w = 0; w < world; ++w)
    MM = fmaxf(MM, __ldcg(own + ((size_t(par) * world + w) * rows + row) * X::kStride));
  float LL = 0.f, tot[R];
#pragma unroll
  for (int r = 0; r < R; ++r) tot[r] = 0.f;
  if (MM != -INFINITY) {
    for (int w = 0; w < world; ++w) {
      const float* st = own + ((size_t(par) * world + w) * rows + row) * X::kStride;
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(st));
      const float wt = ml.x != -INFINITY ? __expf(ml.x - MM) : 0.f;
      LL += wt * ml.y;
#pragma unroll
      for (int r = 0; r < R; ++r) tot[r] += wt * __ldcg(st + 4 + r * 32 + lane);
    }
  }
  const float inv = LL > 0.f ? 1.f / LL : 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) o[r * 32 + lane] = tot[r] * inv;
}

}  // namespace bc
