// On-device token sampling: SwiftletSession.sample (SwiftletSession.swift:
// 226-273) for a batch of logit rows, one CTA of 1024 threads per row.
//
// Per row: suppressed ids and (when the row bans EOS) the EOS ids become
// -inf; every token seen n > 0 times loses presence + frequency * n; then
// temperature <= 0 takes the first maximum, otherwise the k = clamp(top_k, 1,
// V) largest logits are selected (radix select over order-preserving 32-bit
// keys: four 8-bit histogram passes find the k-th largest key, over the row
// until the keys at or above the chosen bin fit SMP_CAP and then over a
// shared-memory copy of those; the larger keys and the lowest-id ties needed
// are gathered), sorted by
// logit (ties: lower id first), weighted by exp((l - l_max) / temperature),
// cut at the first cumulative share >= top_p, and sampled by walking
// u * sum down the weights, as the reference does, in its sequential order.
#include "common.h"
#include "kernels.h"
#include "launch.h"

namespace swl {

namespace {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_CAP = 8192;  // keys the top-k select keeps in shared memory

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float fval(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key ^ 0x80000000u) : ~key);
}

__device__ __forceinline__ float adjusted(const SampleArgs& a, const float* lg, const int* cnt,
                                          const uint32_t* ban, int v) {
  float x = lg[v];
  if (ban[v >> 5] & (1u << (v & 31))) x = -INFINITY;
  if (cnt && (a.presence != 0.f || a.frequency != 0.f)) {
    const int n = cnt[v];
    if (n > 0) x = __fsub_rn(x, __fadd_rn(a.presence, __fmul_rn(a.frequency, float(n))));
  }
  return x;
}

// exclusive block scan of one int per thread; returns the total
__device__ int block_scan(int v, int* ex, int* warp_sums) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane], wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  *ex = warp_sums[warp] + inc - v;
  const int total = warp_sums[32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(const SampleArgs a) {
  extern __shared__ uint32_t ban[];  // ceil(V / 32) words, then SMP_CAP keys and SMP_CAP ids
  __shared__ unsigned hist[256];
  __shared__ float cval[SMP_KMAX], prob[SMP_KMAX];
  __shared__ int cidx[SMP_KMAX];
  __shared__ int warp_sums[33];
  __shared__ float bval[32];
  __shared__ int bidx[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining, s_bin, s_n;
  const int s = blockIdx.x, tid = threadIdx.x, V = a.vocab;
  const float* lg = a.logits + int64_t(s) * a.row_stride;
  int* cnt = a.counts ? a.counts + int64_t(s) * V : nullptr;
  const int nw = (V + 31) >> 5;
  for (int w = tid; w < nw; w += SMP_THREADS) ban[w] = 0u;
  __syncthreads();
  for (int i = tid; i < a.n_suppress; i += SMP_THREADS) {
    const int t = a.suppress[i];
    if (t >= 0 && t < V) atomicOr(&ban[t >> 5], 1u << (t & 31));
  }
  if (a.eos && (!a.ban_eos || a.ban_eos[s]))
    for (int i = tid; i < a.n_eos; i += SMP_THREADS) {
      const int t = a.eos[i];
      if (t >= 0 && t < V) atomicOr(&ban[t >> 5], 1u << (t & 31));
    }
  __syncthreads();

  int token = 0;
  if (a.temperature <= 0.f) {
    // first maximum (strict >, ids ascending)
    float best = -INFINITY;
    int bi = -1;
    for (int v = tid; v < V; v += SMP_THREADS) {
      const float x = adjusted(a, lg, cnt, ban, v);
      if (bi < 0 || x > best) { best = x; bi = v; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_down_sync(0xffffffffu, best, o);
      const int oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ob > best || (ob == best && oi < bi))) { best = ob; bi = oi; }
    }
    if ((tid & 31) == 0) { bval[tid >> 5] = best; bidx[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
      best = bval[0]; bi = bidx[0];
      for (int w = 1; w < SMP_THREADS / 32; ++w)
        if (bidx[w] >= 0 && (bi < 0 || bval[w] > best || (bval[w] == best && bidx[w] < bi))) {
          best = bval[w]; bi = bidx[w];
        }
      token = bi < 0 ? 0 : bi;
    }
  } else {
    const int k = max(1, min(a.top_k, V));
    // k-th largest key, 8 bits at a time from the top. The passes read the
    // row until the keys at or above the chosen bin fit SMP_CAP; then one
    // more pass copies them to shared memory and the remaining passes and
    // the gather run there.
    uint32_t* lkey = ban + ((V + 31) >> 5);
    int* lidx = reinterpret_cast<int*>(lkey + SMP_CAP);
    if (tid == 0) { s_prefix = 0u; s_remaining = k; s_n = 0; }
    uint32_t mask = 0u;
    bool local = false;
    int n_local = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += SMP_THREADS) hist[b] = 0u;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      if (local) {
        for (int i = tid; i < n_local; i += SMP_THREADS) {
          const uint32_t key = lkey[i];
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
      } else {
        for (int v = tid; v < V; v += SMP_THREADS) {
          const uint32_t key = fkey(adjusted(a, lg, cnt, ban, v));
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
      }
      __syncthreads();
      if (tid == 0) {
        int rem = s_remaining, b = 255;
        for (; b > 0; --b) {
          if (int(hist[b]) >= rem) break;
          rem -= int(hist[b]);
        }
        s_prefix = prefix | (uint32_t(b) << shift);
        s_bin = int(hist[b]);
        s_remaining = rem;
      }
      mask |= 255u << shift;
      __syncthreads();
      if (!local && shift > 0 && (k - s_remaining) + s_bin <= SMP_CAP) {
        // keys whose leading bits are at or above the chosen bin's
        const uint32_t top = s_prefix >> shift;
        for (int v = tid; v < V; v += SMP_THREADS) {
          const uint32_t key = fkey(adjusted(a, lg, cnt, ban, v));
          if ((key >> shift) >= top) {
            const int at = atomicAdd(&s_n, 1);
            lkey[at] = key;
            lidx[at] = v;
          }
        }
        __syncthreads();
        local = true;
        n_local = s_n;
      }
    }
    const uint32_t thr = s_prefix;
    const int need_eq = s_remaining, tot_gt = k - need_eq;
    if (local) {
      // larger keys in any order (the sort below fixes it); of the keys equal
      // to the threshold, the need_eq lowest ids
      if (tid == 0) s_n = 0;
      __syncthreads();
      for (int i = tid; i < n_local; i += SMP_THREADS) {
        const uint32_t key = lkey[i];
        if (key > thr) {
          const int at = atomicAdd(&s_n, 1);
          cval[at] = fval(key); cidx[at] = lidx[i];
        } else if (key == thr) {
          int rank = 0;
          for (int j = 0; j < n_local; ++j) rank += lkey[j] == thr && lidx[j] < lidx[i];
          if (rank < need_eq) { cval[tot_gt + rank] = fval(key); cidx[tot_gt + rank] = lidx[i]; }
        }
      }
    } else {
      // gather: thread t scans ids [t * C, (t + 1) * C) in order
      const int C = (V + SMP_THREADS - 1) / SMP_THREADS;
      const int v0 = min(V, tid * C), v1 = min(V, v0 + C);
      int n_gt = 0, n_eq = 0;
      for (int v = v0; v < v1; ++v) {
        const uint32_t key = fkey(adjusted(a, lg, cnt, ban, v));
        n_gt += key > thr;
        n_eq += key == thr;
      }
      int gt_off, eq_off;
      block_scan(n_gt, &gt_off, warp_sums);
      block_scan(n_eq, &eq_off, warp_sums);
      for (int v = v0; v < v1; ++v) {
        const float x = adjusted(a, lg, cnt, ban, v);
        const uint32_t key = fkey(x);
        if (key > thr) {
          cval[gt_off] = x; cidx[gt_off] = v; ++gt_off;
        } else if (key == thr) {
          if (eq_off < need_eq) { cval[tot_gt + eq_off] = x; cidx[tot_gt + eq_off] = v; }
          ++eq_off;
        }
      }
    }
    // bitonic sort of the k candidates: logit descending, id ascending
    int P = 1;
    while (P < k) P <<= 1;
    for (int i = k + tid; i < P; i += SMP_THREADS) { cval[i] = -INFINITY; cidx[i] = 0x7fffffff; }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1)
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < P; i += SMP_THREADS) {
          const int j = i ^ stride;
          if (j > i) {
            const bool desc = (i & size) == 0;
            const float vi = cval[i], vj = cval[j];
            const int ii = cidx[i], ij = cidx[j];
            const bool i_first = vi > vj || (vi == vj && ii < ij);
            if (i_first != desc) { cval[i] = vj; cval[j] = vi; cidx[i] = ij; cidx[j] = ii; }
          }
        }
        __syncthreads();
      }
    const float l0 = cval[0];
    for (int i = tid; i < k; i += SMP_THREADS) prob[i] = expf((cval[i] - l0) / a.temperature);
    __syncthreads();
    if (tid == 0) {
      float sum = 0.f;
      for (int i = 0; i < k; ++i) sum += prob[i];
      int cut = k;
      if (a.top_p < 1.f) {
        float cum = 0.f;
        for (int i = 0; i < k; ++i) {
          cum += prob[i] / sum;
          if (cum >= a.top_p) { cut = i + 1; break; }
        }
        sum = 0.f;
        for (int i = 0; i < cut; ++i) sum += prob[i];
      }
      float r = a.uniform[s] * sum;
      token = cidx[0];
      for (int i = 0; i < cut; ++i) {
        r -= prob[i];
        if (r <= 0.f) { token = cidx[i]; break; }
      }
    }
  }
  if (tid == 0) {
    a.out[s] = token;
    if (cnt && a.update_counts) cnt[token] += 1;
  }
}

}  // namespace

void launch_sample(const SampleArgs& a, cudaStream_t st) {
  if (a.nseq < 1 || a.vocab < 1 || a.row_stride < a.vocab) throw Error(ERR_INVALID, "sampling: bad shape");
  if (a.temperature > 0.f && a.top_k > SMP_KMAX && a.vocab > SMP_KMAX)
    throw Error(ERR_UNSUPPORTED, "sampling: top_k above " + std::to_string(SMP_KMAX));
  const size_t smem = size_t((a.vocab + 31) / 32) * 4 + size_t(SMP_CAP) * 8;
  if (smem > 200 * 1024) throw Error(ERR_UNSUPPORTED, "sampling: vocabulary above 1.1M tokens");
  SWL_CUDA(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  k_sample<<<a.nseq, SMP_THREADS, smem, st>>>(a);
  SWL_CUDA(cudaGetLastError());
}

}  // namespace swl
