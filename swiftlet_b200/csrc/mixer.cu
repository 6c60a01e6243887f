// Token-mixer kernels of the decode step: the gated-DeltaNet step
// (conv + norms + gating + delta-rule recurrence) and gated GQA attention,
// plus the embedding row and the bit-exact dequant helper.
#include <algorithm>

#include "kcommon.cuh"
#include "kernels.h"
#include "launch.h"

namespace swl {

// ------------------------------------------------------------ DeltaNet ----
// One decode step of a gated-DeltaNet layer after its in-projections:
// causal conv (ring of conv_k rows, slot = pos % conv_k) + SiLU, q/k
// RMSNorm (no weight, eps 1e-6) scaled 1/dk and 1/sqrt(dk),
// g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b), and the
// recurrence S <- gS; d = (v - S k) beta; S <- S + k d^T; y = S q
// (QwenCPUModel.swift:423-488). Block = (v-head, slice of RB dv rows); a
// warp owns rows r = warp, warp + 4, ...; the state rows are loaded into
// registers before the dependency wait (they were written one token ago).
constexpr int DELTA_THREADS = 128;     // single-sequence launches
constexpr int DELTA_MAX_THREADS = 512; // batched launches: one CTA per (v-head, sequence), 8 rows per warp
constexpr int DELTA_RPW = 8;  // rows per warp (RB <= 32)
constexpr int DELTA_EPL = 4;  // state elements per lane (dk <= 128)

// RPW rows of state per warp: 8 for single-sequence launches (128 threads per
// 32-row slice); 16 for batched launches, whose 256-thread CTAs hold a whole
// 128-row head and fit two per SM, so one CTA's state loads overlap another's
// update.
template <int RPW>
__global__ void __launch_bounds__(RPW == 8 ? DELTA_MAX_THREADS : 256, RPW == 8 ? 1 : 2) k_delta(const DeltaArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int dk = a.dk, dv = a.dv, K = a.conv_k, RB = a.rows_per_block;
  const int hv = blockIdx.x, slice = blockIdx.y, rep = a.nv / a.nk, hk = hv / rep;
  const int keyDim = a.nk * dk;
  const int nch = 2 * dk + RB;
  float* q = sm;                  // [dk]
  float* k = q + dk;              // [dk]
  float* v = k + dk;              // [RB]
  float* taps = v + RB;           // [nch][K-1] older conv inputs
  float* cw = taps + nch * (K - 1);  // [nch][K] conv weights
  __shared__ float gb[2], nrm[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  // sequence blockIdx.z of a batched step (0 for one sequence)
  const StateDev* sd = a.sd + blockIdx.z;
  const float* proj = a.proj + blockIdx.z * a.proj_stride;
  float* yout = a.y + int64_t(blockIdx.z) * a.nv * dv;
  float* zout = a.z + int64_t(blockIdx.z) * a.nv * dv;
  TraceRec trc;
  trc.start(a.trace);
  // ---- before the wait: everything written by earlier tokens ----
  const int pos = *sd->pos;
  const float* ring = sd->conv[a.layer];
  float* S = sd->dstate[a.layer];
  auto chan = [&](int t) {
    if (t < dk) return hk * dk + t;
    if (t < 2 * dk) return keyDim + hk * dk + (t - dk);
    return 2 * keyDim + hv * dv + slice * RB + (t - 2 * dk);
  };
  for (int t = threadIdx.x; t < nch; t += blockDim.x) {
    const int c = chan(t);
    for (int j = 0; j < K - 1; ++j) {
      const int rs = ((pos - (K - 1) + j) % K + K) % K;
      taps[t * (K - 1) + j] = ring[int64_t(rs) * a.conv_dim + c];
    }
    for (int j = 0; j < K; ++j) cw[t * K + j] = a.conv_w[c * K + j];
  }
  float st[RPW][DELTA_EPL];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const int r = warp + j * nw;
    const float* Sr = S + (int64_t(hv) * dv + slice * RB + r) * dk;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) {
      const int i = lane + 32 * e;
      st[j][e] = (r < RB && i < dk) ? Sr[i] : 0.f;
    }
  }
  const float alog = a.a_log[hv], dtb = a.dt_bias[hv];
  pdl_wait();
  trc.waited(a.trace);
  // ---- the current token's projections ----
  float* ring_w = sd->conv[a.layer];
  const int slot = pos % K;
  const bool own_qk = (hv % rep) == 0 && slice == 0;
  for (int t = threadIdx.x; t < nch; t += blockDim.x) {
    const int c = chan(t);
    const float xn = proj[delta_src(a, c)];
    float acc = 0.f;
    for (int j = 0; j < K - 1; ++j) acc += cw[t * K + j] * taps[t * (K - 1) + j];
    acc += cw[t * K + K - 1] * xn;
    const float o = silu_ref(acc);
    if (t < dk) q[t] = o; else if (t < 2 * dk) k[t - dk] = o; else v[t - 2 * dk] = o;
    if (t >= 2 * dk || own_qk) ring_w[int64_t(slot) * a.conv_dim + c] = xn;
  }
  if (threadIdx.x == 0) {
    int bi, ai;
    delta_ba(a, hv, bi, ai);
    gb[0] = expf(-expf(alog) * softplus_ref(proj[ai] + dtb));
    gb[1] = sigmoid_ref(proj[bi]);
  }
  for (int i = threadIdx.x; i < RB; i += blockDim.x) {
    const int d = slice * RB + i;
    zout[hv * dv + d] = silu_ref(proj[delta_z(a, hv, d)]);  // the output gate's activation
  }
  __syncthreads();
  pdl_launch();
  // q/k RMSNorm: warp 0 reduces q, warp 1 reduces k
  if (warp < 2) {
    const float* x = warp == 0 ? q : k;
    float ss = 0.f;
    for (int i = lane; i < dk; i += 32) ss += x[i] * x[i];
    ss = warp_sum(ss);
    if (lane == 0) nrm[warp] = 1.f / sqrtf(ss / float(dk) + 1e-6f);
  }
  __syncthreads();
  const float inv = 1.f / sqrtf(float(dk));
  float qr[DELTA_EPL], kr[DELTA_EPL];
#pragma unroll
  for (int e = 0; e < DELTA_EPL; ++e) {
    const int i = lane + 32 * e;
    qr[e] = i < dk ? (q[i] * nrm[0]) * (inv * inv) : 0.f;
    kr[e] = i < dk ? (k[i] * nrm[1]) * inv : 0.f;
  }
  const float g = gb[0], beta = gb[1];
  float kv[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    float p = 0.f;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) { st[j][e] *= g; p += st[j][e] * kr[e]; }
    kv[j] = p;
  }
#pragma unroll
  for (int j = 0; j < RPW; ++j) kv[j] = warp_sum(kv[j]);
  float y[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const int r = warp + j * nw;
    const float delta = ((r < RB ? v[r] : 0.f) - kv[j]) * beta;
    float p = 0.f;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) { st[j][e] += kr[e] * delta; p += st[j][e] * qr[e]; }
    y[j] = p;
  }
#pragma unroll
  for (int j = 0; j < RPW; ++j) y[j] = warp_sum(y[j]);
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const int r = warp + j * nw;
    if (r >= RB) continue;
    float* Sr = S + (int64_t(hv) * dv + slice * RB + r) * dk;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) {
      const int i = lane + 32 * e;
      if (i < dk) Sr[i] = st[j][e];
    }
    if (lane == 0) yout[hv * dv + slice * RB + r] = y[j];
  }
  trc.end(a.trace);
}

// The same step for 128-dim key heads, spread over many small CTAs so that
// every SM streams state: CTA = (v-head, slice of RB = NW * RPW rows[, sequence
// of a batched step]); warp w owns rows w * RPW .. w * RPW + RPW - 1 of the
// slice and each lane holds four consecutive elements of a row, so a row is
// one 16-byte load (and store) per lane. The rows are loaded, and the conv
// history and weights staged, before the dependency wait.
constexpr int DELTA4_DK = 128;
template <int RPW, int NW>
__global__ void __launch_bounds__(NW * 32) k_delta4(const DeltaArgs a) {
  constexpr int RB = RPW * NW, DK = DELTA4_DK;
  extern __shared__ __align__(16) float sm[];
  __shared__ __align__(16) float q[DK];
  __shared__ __align__(16) float k[DK];
  __shared__ float v[RB], gb[2], nrm[2];
  const int K = a.conv_k;
  const int hv = blockIdx.x, slice = blockIdx.y, rep = a.nv / a.nk, hk = hv / rep;
  const int keyDim = a.nk * DK, dv = a.dv;
  constexpr int nch = 2 * DK + RB;
  float* taps = sm;                  // [nch][K-1] older conv inputs
  float* cw = taps + nch * (K - 1);  // [nch][K] conv weights
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const StateDev* sd = a.sd + blockIdx.z;
  const float* proj = a.proj + blockIdx.z * a.proj_stride;
  float* yout = a.y + int64_t(blockIdx.z) * a.nv * dv;
  float* zout = a.z + int64_t(blockIdx.z) * a.nv * dv;
  TraceRec trc;
  trc.start(a.trace);
  // ---- before the wait: everything written by earlier tokens ----
  const int pos = *sd->pos;
  const float* ring = sd->conv[a.layer];
  float* S = sd->dstate[a.layer];
  const int row0 = slice * RB + warp * RPW;  // first row of this warp within the head
  float4* S4 = reinterpret_cast<float4*>(S + (int64_t(hv) * dv + row0) * DK) + lane;
  float4 st[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j) st[j] = S4[j * (DK / 4)];
  auto chan = [&](int t) {
    if (t < DK) return hk * DK + t;
    if (t < 2 * DK) return keyDim + hk * DK + (t - DK);
    return 2 * keyDim + hv * dv + slice * RB + (t - 2 * DK);
  };
  for (int t = threadIdx.x; t < nch; t += blockDim.x) {
    const int c = chan(t);
    for (int j = 0; j < K - 1; ++j) {
      const int rs = ((pos - (K - 1) + j) % K + K) % K;
      taps[t * (K - 1) + j] = ring[int64_t(rs) * a.conv_dim + c];
    }
    for (int j = 0; j < K; ++j) cw[t * K + j] = a.conv_w[c * K + j];
  }
  const float alog = a.a_log[hv], dtb = a.dt_bias[hv];
  pdl_wait();
  trc.waited(a.trace);
  // ---- the current token's projections ----
  float* ring_w = sd->conv[a.layer];
  const int slot = pos % K;
  const bool own_qk = (hv % rep) == 0 && slice == 0;
  for (int t = threadIdx.x; t < nch; t += blockDim.x) {
    const int c = chan(t);
    const float xn = proj[delta_src(a, c)];
    float acc = 0.f;
    for (int j = 0; j < K - 1; ++j) acc += cw[t * K + j] * taps[t * (K - 1) + j];
    acc += cw[t * K + K - 1] * xn;
    const float o = silu_ref(acc);
    if (t < DK) q[t] = o; else if (t < 2 * DK) k[t - DK] = o; else v[t - 2 * DK] = o;
    if (t >= 2 * DK || own_qk) ring_w[int64_t(slot) * a.conv_dim + c] = xn;
  }
  if (threadIdx.x == 0) {
    int bi, ai;
    delta_ba(a, hv, bi, ai);
    gb[0] = expf(-expf(alog) * softplus_ref(proj[ai] + dtb));
    gb[1] = sigmoid_ref(proj[bi]);
  }
  for (int i = threadIdx.x; i < RB; i += blockDim.x) {
    const int d = slice * RB + i;
    zout[hv * dv + d] = silu_ref(proj[delta_z(a, hv, d)]);  // the output gate's activation
  }
  __syncthreads();
  pdl_launch();
  // q/k RMSNorm: warp 0 reduces q, warp 1 reduces k
  if (warp < 2) {
    const float4 x4 = reinterpret_cast<const float4*>(warp == 0 ? q : k)[lane];
    float ss = x4.x * x4.x + x4.y * x4.y + x4.z * x4.z + x4.w * x4.w;
    ss = warp_sum(ss);
    if (lane == 0) nrm[warp] = 1.f / sqrtf(ss / float(DK) + 1e-6f);
  }
  __syncthreads();
  const float inv = 1.f / sqrtf(float(DK));
  const float qs = nrm[0] * (inv * inv), ks = nrm[1] * inv;
  float4 qr = reinterpret_cast<const float4*>(q)[lane], kr = reinterpret_cast<const float4*>(k)[lane];
  qr.x *= qs; qr.y *= qs; qr.z *= qs; qr.w *= qs;
  kr.x *= ks; kr.y *= ks; kr.z *= ks; kr.w *= ks;
  const float g = gb[0], beta = gb[1];
  float kv[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    st[j].x *= g; st[j].y *= g; st[j].z *= g; st[j].w *= g;
    kv[j] = st[j].x * kr.x + st[j].y * kr.y + st[j].z * kr.z + st[j].w * kr.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int j = 0; j < RPW; ++j) kv[j] += __shfl_xor_sync(0xffffffffu, kv[j], o);
  float y[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const float delta = (v[warp * RPW + j] - kv[j]) * beta;
    st[j].x += kr.x * delta; st[j].y += kr.y * delta; st[j].z += kr.z * delta; st[j].w += kr.w * delta;
    y[j] = st[j].x * qr.x + st[j].y * qr.y + st[j].z * qr.z + st[j].w * qr.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int j = 0; j < RPW; ++j) y[j] += __shfl_xor_sync(0xffffffffu, y[j], o);
#pragma unroll
  for (int j = 0; j < RPW; ++j) S4[j * (DK / 4)] = st[j];
  if (lane < RPW) {
    float yl = y[0];
#pragma unroll
    for (int j = 1; j < RPW; ++j) if (lane == j) yl = y[j];
    yout[hv * dv + row0 + lane] = yl;
  }
  trc.end(a.trace);
}

// Chunked step: the recurrence of k_delta over a sequence's consecutive
// tokens in order, the state rows in registers throughout (one CTA per
// (v-head, sequence), the whole head's dv rows). The conv window of each
// channel starts from the ring (positions pos - 3 .. pos - 1) and slides over
// the chunk's inputs; the ring itself is updated afterwards by k_conv_ring
// (other CTAs of the launch still read the old positions).
__global__ void __launch_bounds__(DELTA_MAX_THREADS) k_delta_seq(const DeltaArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int dk = a.dk, dv = a.dv, K = a.conv_k, RB = dv;
  const int hv = blockIdx.x, s = blockIdx.y, rep = a.nv / a.nk, hk = hv / rep;
  const int keyDim = a.nk * dk;
  const int nch = 2 * dk + RB;
  float* q = sm;                     // [dk]
  float* k = q + dk;                 // [dk]
  float* v = k + dk;                 // [RB]
  float* win = v + RB;               // [nch][K-1] the channel's previous conv inputs, oldest first
  float* cw = win + nch * (K - 1);   // [nch][K] conv weights
  __shared__ float gb[2], nrm[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const StateDev* sd = a.sd + s;
  const int pos = *sd->pos;
  const float* ring = sd->conv[a.layer];
  float* S = sd->dstate[a.layer];
  auto chan = [&](int t) {
    if (t < dk) return hk * dk + t;
    if (t < 2 * dk) return keyDim + hk * dk + (t - dk);
    return 2 * keyDim + hv * dv + (t - 2 * dk);
  };
  for (int t = threadIdx.x; t < nch; t += blockDim.x) {
    const int c = chan(t);
    for (int j = 0; j < K - 1; ++j) {
      const int rs = ((pos - (K - 1) + j) % K + K) % K;
      win[t * (K - 1) + j] = ring[int64_t(rs) * a.conv_dim + c];
    }
    for (int j = 0; j < K; ++j) cw[t * K + j] = a.conv_w[c * K + j];
  }
  float st[DELTA_RPW][DELTA_EPL];
#pragma unroll
  for (int j = 0; j < DELTA_RPW; ++j) {
    const int r = warp + j * nw;
    const float* Sr = S + (int64_t(hv) * dv + r) * dk;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) {
      const int i = lane + 32 * e;
      st[j][e] = (r < RB && i < dk) ? Sr[i] : 0.f;
    }
  }
  const float alog = a.a_log[hv], dtb = a.dt_bias[hv];
  pdl_wait();
  const int t0 = a.seq_first[s], n = a.seq_n[s];
  const float inv = 1.f / sqrtf(float(dk));
  for (int i = 0; i < n; ++i) {
    const int tok = t0 + i;
    const float* proj = a.proj + tok * a.proj_stride;
    float* yout = a.y + int64_t(tok) * a.nv * dv;
    float* zout = a.z + int64_t(tok) * a.nv * dv;
    for (int t = threadIdx.x; t < nch; t += blockDim.x) {
      const int c = chan(t);
      const float xn = proj[delta_src(a, c)];
      float* w = win + t * (K - 1);
      float acc = 0.f;
      for (int j = 0; j < K - 1; ++j) acc += cw[t * K + j] * w[j];
      acc += cw[t * K + K - 1] * xn;
      for (int j = 0; j + 1 < K - 1; ++j) w[j] = w[j + 1];
      if (K > 1) w[K - 2] = xn;
      const float o = silu_ref(acc);
      if (t < dk) q[t] = o; else if (t < 2 * dk) k[t - dk] = o; else v[t - 2 * dk] = o;
    }
    if (threadIdx.x == 0) {
      int bi, ai;
      delta_ba(a, hv, bi, ai);
      gb[0] = expf(-expf(alog) * softplus_ref(proj[ai] + dtb));
      gb[1] = sigmoid_ref(proj[bi]);
    }
    for (int d = threadIdx.x; d < RB; d += blockDim.x) zout[hv * dv + d] = silu_ref(proj[delta_z(a, hv, d)]);
    __syncthreads();
    if (warp < 2) {
      const float* x = warp == 0 ? q : k;
      float ss = 0.f;
      for (int j = lane; j < dk; j += 32) ss += x[j] * x[j];
      ss = warp_sum(ss);
      if (lane == 0) nrm[warp] = 1.f / sqrtf(ss / float(dk) + 1e-6f);
    }
    __syncthreads();
    float qr[DELTA_EPL], kr[DELTA_EPL];
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) {
      const int j = lane + 32 * e;
      qr[e] = j < dk ? (q[j] * nrm[0]) * (inv * inv) : 0.f;
      kr[e] = j < dk ? (k[j] * nrm[1]) * inv : 0.f;
    }
    const float g = gb[0], beta = gb[1];
    float kv[DELTA_RPW];
#pragma unroll
    for (int j = 0; j < DELTA_RPW; ++j) {
      float p = 0.f;
#pragma unroll
      for (int e = 0; e < DELTA_EPL; ++e) { st[j][e] *= g; p += st[j][e] * kr[e]; }
      kv[j] = p;
    }
#pragma unroll
    for (int j = 0; j < DELTA_RPW; ++j) kv[j] = warp_sum(kv[j]);
    float y[DELTA_RPW];
#pragma unroll
    for (int j = 0; j < DELTA_RPW; ++j) {
      const int r = warp + j * nw;
      const float delta = ((r < RB ? v[r] : 0.f) - kv[j]) * beta;
      float p = 0.f;
#pragma unroll
      for (int e = 0; e < DELTA_EPL; ++e) { st[j][e] += kr[e] * delta; p += st[j][e] * qr[e]; }
      y[j] = p;
    }
#pragma unroll
    for (int j = 0; j < DELTA_RPW; ++j) y[j] = warp_sum(y[j]);
#pragma unroll
    for (int j = 0; j < DELTA_RPW; ++j) {
      const int r = warp + j * nw;
      if (r < RB && lane == 0) yout[hv * dv + r] = y[j];
    }
    __syncthreads();  // q / k / v / gates of the next token overwrite shared memory
  }
  pdl_launch();
#pragma unroll
  for (int j = 0; j < DELTA_RPW; ++j) {
    const int r = warp + j * nw;
    if (r >= RB) continue;
    float* Sr = S + (int64_t(hv) * dv + r) * dk;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) {
      const int i2 = lane + 32 * e;
      if (i2 < dk) Sr[i2] = st[j][e];
    }
  }
}

// The conv ring after a chunk: slot p % conv_k of every channel takes the
// input of position p for the chunk's last min(n, conv_k) positions.
__global__ void k_conv_ring(const DeltaArgs a) {
  pdl_wait();
  const int s = blockIdx.x, c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= a.conv_dim) return;
  const StateDev* sd = a.sd + s;
  const int pos = *sd->pos, n = a.seq_n[s], t0 = a.seq_first[s], K = a.conv_k;
  float* ring = sd->conv[a.layer];
  const int src = delta_src(a, c);
  for (int i = max(0, n - K); i < n; ++i)
    ring[int64_t((pos + i) % K) * a.conv_dim + c] = a.proj[(t0 + i) * a.proj_stride + src];
}

// Chunked step: token z's key (RMSNorm with weight, partial NeoX RoPE at its
// position, as in k_attn) and value into the cache of its sequence.
__global__ void k_kv_append(const AttnArgs a) {
  pdl_wait();
  const int z = blockIdx.x, kvh = blockIdx.y, HD = a.hd, tid = threadIdx.x;
  const StateDev* sd = a.sd + a.tok_seq[z];
  const int pos = *sd->pos + a.tok_off[z];
  const float* kin = a.knew + z * a.proj_stride + kvh * HD;
  const float* vin = a.vnew + z * a.proj_stride + kvh * HD;
  float* Kr = sd->kc[a.layer] + (int64_t(kvh) * sd->max_ctx + pos) * HD;
  float* Vr = sd->vc[a.layer] + (int64_t(kvh) * sd->max_ctx + pos) * HD;
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  for (int i = tid; i < HD; i += blockDim.x) { xs[i] = kin[i]; Vr[i] = vin[i]; }
  float ss = 0.f;
  for (int i = tid; i < HD; i += blockDim.x) ss += xs[i] * xs[i];
  ss = block_sum(ss, red);
  const float sc0 = 1.f / sqrtf(ss / float(HD) + a.eps);
  __syncthreads();
  for (int i = tid; i < HD; i += blockDim.x) xs[i] *= sc0 * a.kn[i];
  __syncthreads();
  const int half = a.rot / 2;
  for (int j = tid; j < half; j += blockDim.x) {
    const float invf = powf(a.rope_theta, -float(2 * j) / float(a.rot));
    const float ang = float(pos) * invf;
    const float cs = cosf(ang), sn = sinf(ang);
    const float xa = xs[j], xb = xs[half + j];
    xs[j] = xa * cs - xb * sn;
    xs[half + j] = xb * cs + xa * sn;
  }
  __syncthreads();
  for (int i = tid; i < HD; i += blockDim.x) Kr[i] = xs[i];
}

// ----------------------------------------------------------- attention ----
// Gated GQA decode for one token: q/k RMSNorm with weight, partial NeoX
// RoPE, KV append, causal softmax(q k^T / sqrt(hd)) v, times sigmoid(gate)
// (QwenCPUModel.swift:285-367). KV layout: [kv_head][max_ctx][head_dim].
//
// Grid (kv heads, chunks); the context is cut into chunks of at least
// ATTN_MINP positions, one per CTA, and clusters of ATTN_CL consecutive
// chunks of one kv head combine their partial results through distributed
// shared memory. A CTA walks its chunk in sub-tiles of ATTN_TP positions held
// in a ring of shared-memory slots, each filled by two bulk copies (the keys
// and the values of consecutive positions are contiguous); the first slots
// are filled before the dependency wait, since the cached positions were
// written by earlier tokens. Scores take one warp per position with the G
// heads reduced together; an online softmax carries (max, sum, output) across
// sub-tiles; in P.V each thread owns one head-dimension column and reads each
// value once for all its heads. Every inner loop has a compile-time trip
// count (head size HD, sub-tile ATTN_TP; the value rows past the chunk are
// zero). Each CTA of a cluster then combines one slice of the G x HD outputs
// over the cluster's CTAs; with one busy cluster per kv head it writes the
// gated output, otherwise the slice's cluster partial goes to global memory
// and, per slice, the CTA of that rank in the last cluster to finish it
// combines the (at most eight) cluster partials.
//
// Output gate sigmoid with the fast exponential and divide (within a few
// ulp of 1 / (1 + exp(-v)); one per output element).
__device__ __forceinline__ float fast_sigmoid(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }

constexpr int ATTN_THREADS = 256;
constexpr int ATTN_MINP = 16;  // minimum positions per chunk
constexpr int ATTN_TP = 16;    // positions per staged sub-tile
constexpr int ATTN_MAXO = 16;  // heads per thread in P.V: G * hd <= ATTN_MAXO * ATTN_THREADS
constexpr int ATTN_CL = 8;     // CTAs (chunks) per cluster
constexpr int ATTN_KO = ATTN_MAXO / ATTN_CL;  // combine outputs per thread
// ring slots: about 64 KiB of keys and values, at least two sub-tiles
template <int HD>
constexpr int attn_ring() {
  return 65536 / (8 * ATTN_TP * HD) < 2 ? 2 : (65536 / (8 * ATTN_TP * HD) > 8 ? 8 : 65536 / (8 * ATTN_TP * HD));
}
template <int HD>
size_t attn_smem_bytes(int G, int rot) {
  return size_t(G * HD + 2 * HD + attn_ring<HD>() * 2 * ATTN_TP * HD + G * ATTN_TP + rot) * 4;
}

constexpr int ATTN_JW = ATTN_TP / (ATTN_THREADS / 32);  // positions per warp in the scores
static_assert(ATTN_JW * 8 <= 32, "the score reduction spreads 8 * ATTN_JW rows over a warp");
// The E = max(HD / 32, 1) elements of a row that lane l holds in the scores:
// float4 chunks l + 32u (HD >= 128), a float2 (HD = 64) or one element
// (elements past HD are zero).
template <int HD>
__device__ __forceinline__ void attn_row_ld(const float* row, int lane, float (&v)[HD >= 32 ? HD / 32 : 1]) {
  constexpr int E = HD >= 32 ? HD / 32 : 1;
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int u = 0; u < E / 4; ++u) {
      const float4 t = reinterpret_cast<const float4*>(row)[lane + 32 * u];
      v[4 * u] = t.x, v[4 * u + 1] = t.y, v[4 * u + 2] = t.z, v[4 * u + 3] = t.w;
    }
  } else if constexpr (E == 2) {
    const float2 t = reinterpret_cast<const float2*>(row)[lane];
    v[0] = t.x, v[1] = t.y;
  } else {
    v[0] = lane < HD ? row[lane] : 0.f;
  }
}

template <int HD>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn(const AttnArgs a) {
  constexpr int E = HD >= 32 ? HD / 32 : 1;      // row elements per lane (l + 32e)
  constexpr int RING = attn_ring<HD>();
  constexpr int SLOT = 2 * ATTN_TP * HD;         // floats per slot: keys, then values
  constexpr int HSTEP = ATTN_THREADS / HD;       // heads per pass of the block in P.V
  extern __shared__ __align__(16) float sm[];
  const int G = a.H / a.Hkv, kvh = blockIdx.x, chunk = blockIdx.y;
  const int half = a.rot / 2;
  float* q = sm;                      // [G][HD] rotated queries; after the loop this CTA's partial
  float* kn = q + G * HD;             // [HD] the new key (normalised, rotated)
  float* vn = kn + HD;                // [HD] the new value
  float* ring = vn + HD;              // RING x SLOT
  float* sc = ring + RING * SLOT;     // [G][TP] scores, then weights
  float* cs = sc + G * ATTN_TP;       // [half] cos
  float* sn = cs + half;              // [half] sin
  __shared__ float hm[64], hl[64], hal[64], hn[72];
  __shared__ __align__(8) uint64_t full[RING];
  __shared__ unsigned last_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = ATTN_THREADS / 32;
  // sequence blockIdx.z of a batched step (0 for one sequence); in a chunked
  // step blockIdx.z is a token of sequence tok_seq[z] whose keys and values
  // are all in the cache already
  const int seq = blockIdx.z;
  const bool cached = a.tok_seq != nullptr;
  const StateDev* sd = a.sd + (cached ? a.tok_seq[seq] : seq);
  const float* qout = a.qout + seq * a.proj_stride;
  const float* knew = a.knew + seq * a.proj_stride;
  const float* vnew = a.vnew + seq * a.proj_stride;
  float* aout = a.out + int64_t(seq) * a.H * HD;
  const int NCL = a.nchunks / ATTN_CL;
  float* apart = a.part + int64_t(seq) * a.Hkv * NCL * G * (HD + 2);
  unsigned* actr = a.counters + seq * a.Hkv * ATTN_CL;
  TraceRec trc;
  trc.start(a.trace);
  const int pos = *sd->pos + (cached ? a.tok_off[seq] : 0);  // written by an earlier step: complete
  const int ctx = pos + 1;
  const int per = max(ATTN_MINP, (ctx + a.nchunks - 1) / a.nchunks);
  const int nvalid = (ctx + per - 1) / per;               // busy chunks (<= nchunks)
  const int ncl = (nvalid + ATTN_CL - 1) / ATTN_CL;       // busy clusters
  const int cl = chunk / ATTN_CL;
  if (cl >= ncl) {  // the whole cluster is idle: no cluster barrier is reached
    trc.end(a.trace);
    return;
  }
  const unsigned rank = cluster_rank();
  const int p0 = chunk * per;
  const int n = chunk < nvalid ? min(ctx, p0 + per) - p0 : 0;
  const int ntiles = (n + ATTN_TP - 1) / ATTN_TP;
  const float* Kc = sd->kc[a.layer] + int64_t(kvh) * sd->max_ctx * HD;
  const float* Vc = sd->vc[a.layer] + int64_t(kvh) * sd->max_ctx * HD;
  uint64_t* fb = full;
  // sub-tile t into slot t % RING: the cached rows (every row but the new
  // position, which is always the chunk's last) by two bulk copies
  auto issue = [=](int t) {
    const int t0 = p0 + t * ATTN_TP, nt = min(ATTN_TP, p0 + n - t0);
    const int nc = !cached && pos < t0 + nt ? nt - 1 : nt;
    float* kt = ring + (t % RING) * SLOT;
    uint64_t* bar = fb + t % RING;
    const unsigned bytes = unsigned(nc) * HD * 4;
    mbar_expect_tx(bar, 2 * bytes);
    if (bytes) {
      bulk_g2s_keep(kt, Kc + int64_t(t0) * HD, bytes, bar);
      bulk_g2s_keep(kt + ATTN_TP * HD, Vc + int64_t(t0) * HD, bytes, bar);
    }
  };
  if (tid == 0) {
    for (int s = 0; s < RING; ++s) mbar_init(&full[s], 1);
    mbar_init_fence();
    // the chunk's own rows were written by the previous kernel: in a chunked
    // step the first copies wait for it
    if (!cached)
      for (int t = 0; t < min(RING, ntiles); ++t) issue(t);
  }
  // before the wait: RoPE table, norm weights, softmax state
  for (int j = tid; j < half; j += ATTN_THREADS) {
    const float invf = powf(a.rope_theta, -float(2 * j) / float(a.rot));
    const float ang = float(pos) * invf;
    cs[j] = cosf(ang);
    sn[j] = sinf(ang);
  }
  for (int h = tid; h < G; h += ATTN_THREADS) { hm[h] = -INFINITY; hl[h] = 0.f; }
  float wq[E], wk[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = lane + 32 * e;
    wq[e] = d < HD ? a.qn[d] : 0.f;
    wk[e] = d < HD ? a.kn[d] : 0.f;
  }
  const int SL = G * HD / ATTN_CL;  // combine slice of this CTA: outputs [rank * SL, (rank + 1) * SL)
  __syncthreads();  // RoPE table and barrier initialisation visible to all
  pdl_wait();
  trc.waited(a.trace);
  if (cached && tid == 0)
    for (int t = 0; t < min(RING, ntiles); ++t) issue(t);
  for (int i = tid; i < HD; i += ATTN_THREADS) vn[i] = __ldcg(vnew + kvh * HD + i);
  // gate values of the combine slice (used if this CTA writes the output)
  float gate[ATTN_KO];
#pragma unroll
  for (int k = 0; k < ATTN_KO; ++k) {
    const int li = tid + k * ATTN_THREADS, i = int(rank) * SL + li;
    gate[k] = li < SL ? __ldcg(qout + (kvh * G + i / HD) * 2 * HD + HD + i % HD) : 0.f;
  }
  if constexpr (HD >= 32) {
    // one warp per head (G q heads and the new k head): RMSNorm in
    // registers (lane l holds elements l + 32e), then RoPE in place
    for (int h = warp; h <= G; h += nw) {
      const float* src = h < G ? qout + (kvh * G + h) * 2 * HD : knew + kvh * HD;
      float v[E];
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = __ldcg(src + lane + 32 * e);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += v[e] * v[e];
      ss = warp_sum(ss);
      const float sc0 = 1.f / sqrtf(ss / float(HD) + a.eps);
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] *= sc0 * (h < G ? wq[e] : wk[e]);
      float* x = h < G ? q + h * HD : kn;
#pragma unroll
      for (int e = 0; e < E; ++e) x[lane + 32 * e] = v[e];
      __syncwarp();
      for (int j = lane; j < half; j += 32) {  // RoPE pairs (j, j + half)
        const float xa = x[j], xb = x[half + j];
        x[j] = xa * cs[j] - xb * sn[j];
        x[half + j] = xb * cs[j] + xa * sn[j];
      }
    }
  } else {
    for (int h = 0; h < G; ++h) copy_async(q + h * HD, qout + (kvh * G + h) * 2 * HD, HD);
    copy_async(kn, knew + kvh * HD, HD);
    cp_async_wait_all();
    __syncthreads();
    // RMSNorm of G q heads and the new k head, one warp per head
    for (int h = warp; h <= G; h += nw) {
      float* x = h < G ? q + h * HD : kn;
      float ss = 0.f;
      for (int i = lane; i < HD; i += 32) ss += x[i] * x[i];
      ss = warp_sum(ss);
      if (lane == 0) hn[h] = 1.f / sqrtf(ss / float(HD) + a.eps);
    }
    __syncthreads();
    for (int i = tid; i < (G + 1) * HD; i += ATTN_THREADS) {
      const int h = i / HD, d = i % HD;
      float* x = h < G ? q + h * HD : kn;
      const float* w = h < G ? a.qn : a.kn;
      x[d] *= hn[h] * w[d];
    }
    __syncthreads();
    for (int i = tid; i < (G + 1) * half; i += ATTN_THREADS) {
      const int h = i / half, j = i % half;
      float* x = h < G ? q + h * HD : kn;
      const float xa = x[j], xb = x[half + j];
      x[j] = xa * cs[j] - xb * sn[j];
      x[half + j] = xb * cs[j] + xa * sn[j];
    }
  }
  __syncthreads();
  pdl_launch();
  if (chunk == 0 && !cached)
    for (int i = tid; i < HD; i += ATTN_THREADS) {
      const_cast<float*>(Kc)[int64_t(pos) * HD + i] = kn[i];
      const_cast<float*>(Vc)[int64_t(pos) * HD + i] = vn[i];
    }
  trc.staged(a.trace);
  const float scale = 1.f / sqrtf(float(HD));
  const int dcol = tid % HD, hb = tid / HD;
  float acc[ATTN_MAXO];
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) acc[o] = 0.f;
  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    float* kt = ring + (t % RING) * SLOT;
    float* vt = kt + ATTN_TP * HD;
    const int t0 = p0 + t * ATTN_TP, nt = min(ATTN_TP, p0 + n - t0);
    if (!mbar_wait(&full[t % RING], unsigned(t / RING) & 1u)) ok = false;
    if (!cached && pos < t0 + nt)  // the new position (the last row): its key and value
      for (int i = tid; i < HD; i += ATTN_THREADS) {
        kt[(pos - t0) * HD + i] = kn[i];
        vt[(pos - t0) * HD + i] = vn[i];
      }
    for (int i = nt * HD + tid; i < ATTN_TP * HD; i += ATTN_THREADS) vt[i] = 0.f;
    __syncthreads();
    // scores: warp w takes positions w and w + 8 for all heads, eight heads
    // at a time; the 16 partial dot products of a lane are reduced together
    for (int h0 = 0; h0 < G; h0 += 8) {
      float qr[8][E];
#pragma unroll
      for (int r = 0; r < 8; ++r) attn_row_ld<HD>(q + min(h0 + r, G - 1) * HD, lane, qr[r]);
      float kv[ATTN_JW][E];
#pragma unroll
      for (int jj = 0; jj < ATTN_JW; ++jj) attn_row_ld<HD>(kt + (warp + jj * nw) * HD, lane, kv[jj]);
      float pr[8 * ATTN_JW];
#pragma unroll
      for (int jj = 0; jj < ATTN_JW; ++jj)
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) d += qr[r][e] * kv[jj][e];
          pr[jj * 8 + r] = d;
        }
      int rr;
      const float d = reduce_rows<8 * ATTN_JW>(pr, 32, lane, rr);
      const int jj = rr >> 3, h = h0 + (rr & 7), j = warp + jj * nw;
      if ((lane & (32 / (8 * ATTN_JW) - 1)) == 0 && h < G) sc[h * ATTN_TP + j] = j < nt ? d * scale : -INFINITY;
    }
    __syncthreads();
    // online softmax: per head the new max, the rescale of what came before,
    // the weights of this sub-tile (0 for rows past the chunk)
    for (int h = warp; h < G; h += nw) {
      const float v = lane < ATTN_TP ? sc[h * ATTN_TP + lane] : -INFINITY;
      const float mt = warp_max(v);
      const float mo = hm[h], mn = fmaxf(mo, mt);
      const float e = lane < ATTN_TP && v != -INFINITY ? expf(v - mn) : 0.f;
      const float s = warp_sum(e);
      if (lane < ATTN_TP) sc[h * ATTN_TP + lane] = e;
      if (lane == 0) {
        const float al = mo == -INFINITY ? 0.f : expf(mo - mn);
        hal[h] = al;
        hl[h] = hl[h] * al + s;
        hm[h] = mn;
      }
    }
    __syncthreads();
    // P.V: column dcol of heads hb, hb + HSTEP, ...: each value read once
    {
      float v[ATTN_TP];
#pragma unroll
      for (int j = 0; j < ATTN_TP; ++j) v[j] = vt[j * HD + dcol];
#pragma unroll
      for (int o = 0; o < ATTN_MAXO; ++o) {
        const int h = hb + o * HSTEP;
        if (h < G) {
          const float4* p4 = reinterpret_cast<const float4*>(sc + h * ATTN_TP);
          float r = acc[o] * hal[h];
#pragma unroll
          for (int j4 = 0; j4 < ATTN_TP / 4; ++j4) {
            const float4 p = p4[j4];
            r += p.x * v[4 * j4] + p.y * v[4 * j4 + 1] + p.z * v[4 * j4 + 2] + p.w * v[4 * j4 + 3];
          }
          acc[o] = r;
        }
      }
    }
    __syncthreads();
    if (tid == 0 && t + RING < ntiles) {
      fence_proxy_async();
      issue(t + RING);
    }
  }
  if (!ok && a.status) atomicOr(a.status, 1);
  trc.looped(a.trace);
  // this CTA's partial: unnormalised outputs (against its running max hm)
  // in the query buffer, max and sum in hm / hl (-inf / 0 for an idle chunk)
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int h = hb + o * HSTEP;
    if (h < G) q[h * HD + dcol] = acc[o];
  }
  cluster_sync();
  // slice `rank` of the outputs, combined over the cluster's CTAs
  float res[ATTN_KO], rm[ATTN_KO], rl[ATTN_KO];
#pragma unroll
  for (int k = 0; k < ATTN_KO; ++k) {
    const int li = tid + k * ATTN_THREADS, i = int(rank) * SL + li, h = i / HD;
    res[k] = 0.f, rm[k] = -INFINITY, rl[k] = 0.f;
    if (li < SL) {
      float mc[ATTN_CL], lc[ATTN_CL], ac[ATTN_CL];
#pragma unroll
      for (int c = 0; c < ATTN_CL; ++c) {
        mc[c] = dsmem_ld(dsmem_map(&hm[h], c));
        lc[c] = dsmem_ld(dsmem_map(&hl[h], c));
        ac[c] = dsmem_ld(dsmem_map(&q[i], c));
      }
      float m = mc[0];
#pragma unroll
      for (int c = 1; c < ATTN_CL; ++c) m = fmaxf(m, mc[c]);
      float l = 0.f, r = 0.f;
#pragma unroll
      for (int c = 0; c < ATTN_CL; ++c) {
        const float f = mc[c] == -INFINITY ? 0.f : expf(mc[c] - m);
        l += lc[c] * f;
        r += ac[c] * f;
      }
      res[k] = r, rm[k] = m, rl[k] = l;
    }
  }
  // done with the other CTAs' shared memory; the matching wait before the
  // exit keeps this CTA's alive until every CTA has read it
  cluster_arrive();
  if (ncl == 1) {
#pragma unroll
    for (int k = 0; k < ATTN_KO; ++k) {
      const int li = tid + k * ATTN_THREADS;
      if (li < SL) aout[kvh * G * HD + int(rank) * SL + li] = (res[k] / rl[k]) * fast_sigmoid(gate[k]);
    }
    cluster_wait();
    trc.end(a.trace);
    return;
  }
  // several busy clusters: the slice's partial to global memory; the CTA of
  // this rank in the last cluster to finish combines the slice over them
  float* pcl = apart + (int64_t(kvh) * NCL + cl) * G * (HD + 2);
#pragma unroll
  for (int k = 0; k < ATTN_KO; ++k) {
    const int li = tid + k * ATTN_THREADS, i = int(rank) * SL + li, h = i / HD, d = i % HD;
    if (li < SL) {
      pcl[h * (HD + 2) + 2 + d] = res[k];
      if (d == 0) {
        pcl[h * (HD + 2)] = rm[k];
        pcl[h * (HD + 2) + 1] = rl[k];
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    unsigned* ctr = actr + kvh * ATTN_CL + rank;
    __threadfence();
    const bool lst = atomicAdd(ctr, 1u) == unsigned(ncl) - 1;
    if (lst) {
      __threadfence();
      *ctr = 0u;
    }
    last_flag = lst ? 1u : 0u;
  }
  __syncthreads();
  if (last_flag) {
    __threadfence();
#pragma unroll
    for (int k = 0; k < ATTN_KO; ++k) {
      const int li = tid + k * ATTN_THREADS, i = int(rank) * SL + li, h = i / HD, d = i % HD;
      if (li < SL) {
        float mc[ATTN_CL], lc[ATTN_CL], ac[ATTN_CL];
#pragma unroll
        for (int c = 0; c < ATTN_CL; ++c) {
          const float* pc = apart + ((int64_t(kvh) * NCL + c) * G + h) * (HD + 2);
          mc[c] = c < ncl ? __ldcg(pc) : -INFINITY;
          lc[c] = c < ncl ? __ldcg(pc + 1) : 0.f;
          ac[c] = c < ncl ? __ldcg(pc + 2 + d) : 0.f;
        }
        float m = mc[0];
#pragma unroll
        for (int c = 1; c < ATTN_CL; ++c) m = fmaxf(m, mc[c]);
        float l = 0.f, r = 0.f;
#pragma unroll
        for (int c = 0; c < ATTN_CL; ++c) {
          const float f = mc[c] == -INFINITY ? 0.f : expf(mc[c] - m);
          l += lc[c] * f;
          r += ac[c] * f;
        }
        aout[kvh * G * HD + i] = (r / l) * fast_sigmoid(gate[k]);
      }
    }
  }
  cluster_wait();
  trc.end(a.trace);
}

// --------------------------------------------------------------- embed ----
__global__ void k_embed(const EmbedArgs a, int D) {
  TraceRec trc;
  trc.start(a.trace);
  pdl_wait();
  trc.waited(a.trace);
  const int tok = a.cursor ? a.tokens[*a.cursor] : a.tokens[blockIdx.y];
  pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float* h = a.h + int64_t(blockIdx.y) * D;
  if (tok < 0 || tok >= a.vocab) {
    if (i == 0) *a.err = 1;
    if (i < D) h[i] = 0.f;
    trc.end(a.trace);
    return;
  }
  trc.end(a.trace);
  if (i >= D) return;
  const QLin& L = a.table;
  float v;
  if (L.bits) {
    const int per = 32 / L.bits;
    const uint32_t word = reinterpret_cast<const uint32_t*>(L.w + int64_t(tok) * L.row_bytes)[i / per];
    const uint32_t qv = (word >> (L.bits * (i % per))) & ((1u << L.bits) - 1u);
    const int64_t g = int64_t(tok) * L.srow + i / L.gs;
    v = __fadd_rn(__fmul_rn(load_scalar(L.s, L.dt, g), float(qv)), load_scalar(L.b, L.dt, g));
  } else {
    v = load_scalar(L.w, L.dt, int64_t(tok) * D + i);
  }
  h[i] = v;
}

// Dequantised rows (bit-exact w = fl(fl(scale * q) + bias), two roundings).
__global__ void k_dequant(const QLin L, int64_t r0, int64_t r1, float* out) {
  const int64_t cols = L.in, n = (r1 - r0) * cols;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < n; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = r0 + t / cols, i = t % cols;
    float v;
    if (L.bits) {
      const int per = 32 / L.bits;
      const uint32_t word = reinterpret_cast<const uint32_t*>(L.w + r * L.row_bytes)[i / per];
      const uint32_t qv = (word >> (L.bits * (i % per))) & ((1u << L.bits) - 1u);
      const int64_t g = r * L.srow + i / L.gs;
      v = __fadd_rn(__fmul_rn(load_scalar(L.s, L.dt, g), float(qv)), load_scalar(L.b, L.dt, g));
    } else {
      v = load_scalar(L.w, L.dt, r * cols + i);
    }
    out[t] = v;
  }
}

// ------------------------------------------------------------- launches --
// 128-dim key heads: RB = NW * RPW rows per CTA.
template <int RPW, int NW>
static bool launch_delta4(const DeltaArgs& a, int T, cudaStream_t st, bool pdl) {
  constexpr int RB = RPW * NW;
  if (a.dk != DELTA4_DK || a.dv % RB || a.conv_k < 1 || a.conv_k > 8) return false;
  const size_t smem = size_t(2 * DELTA4_DK + RB) * (2 * a.conv_k - 1) * 4;
  launch(k_delta4<RPW, NW>, dim3(a.nv, a.dv / RB, T), dim3(NW * 32), smem, st, pdl, a);
  return true;
}

void launch_delta(const DeltaArgs& a, cudaStream_t st, bool pdl) {
  // one token: 8 rows per CTA (512 CTAs of 128 threads at 32 heads x 128 rows)
  if (launch_delta4<2, 4>(a, 1, st, pdl)) { path_note("delta"); return; }
  if (a.dk > 32 * DELTA_EPL || a.rows_per_block > DELTA_RPW * (DELTA_THREADS / 32) || a.dv % a.rows_per_block)
    throw Error(ERR_UNSUPPORTED, "DeltaNet head dims outside the decode kernel's range");
  const int nch = 2 * a.dk + a.rows_per_block;
  const size_t smem = size_t(2 * a.dk + a.rows_per_block + nch * (2 * a.conv_k - 1)) * 4;
  launch(k_delta<DELTA_RPW>, dim3(a.nv, a.dv / a.rows_per_block), dim3(DELTA_THREADS), smem, st, pdl, a);
  path_note("delta");
}

// Batched: up to 128 rows per CTA (a whole 128-row value head), so the q/k
// convolution and norms of a key head are computed by fewer CTAs.
void launch_delta_batch(const DeltaArgs& a, int T, cudaStream_t st, bool pdl) {
  // 32 rows per CTA: 4 CTAs per head and sequence
  if (launch_delta4<4, 8>(a, T, st, pdl)) return;
  constexpr int RPW = 2 * DELTA_RPW;
  const int threads = std::max(DELTA_THREADS, 32 * ((a.rows_per_block + RPW - 1) / RPW));
  if (a.dk > 32 * DELTA_EPL || threads > 256 || a.dv % a.rows_per_block)
    throw Error(ERR_UNSUPPORTED, "DeltaNet head dims outside the decode kernel's range");
  const int nch = 2 * a.dk + a.rows_per_block;
  const size_t smem = size_t(2 * a.dk + a.rows_per_block + nch * (2 * a.conv_k - 1)) * 4;
  launch(k_delta<RPW>, dim3(a.nv, a.dv / a.rows_per_block, T), dim3(threads), smem, st, pdl, a);
}

void launch_delta_seq(const DeltaArgs& a, int S, cudaStream_t st, bool pdl) {
  const int threads = std::max(DELTA_THREADS, 32 * ((a.dv + DELTA_RPW - 1) / DELTA_RPW));
  if (a.dk > 32 * DELTA_EPL || threads > DELTA_MAX_THREADS || !a.seq_first || !a.seq_n)
    throw Error(ERR_UNSUPPORTED, "DeltaNet head dims outside the chunked kernel's range");
  const int nch = 2 * a.dk + a.dv;
  const size_t smem = size_t(2 * a.dk + a.dv + nch * (2 * a.conv_k - 1)) * 4;
  launch(k_delta_seq, dim3(a.nv, S), dim3(threads), smem, st, pdl, a);
}

void launch_conv_ring(const DeltaArgs& a, int S, cudaStream_t st, bool pdl) {
  launch(k_conv_ring, dim3(S, (a.conv_dim + 255) / 256), dim3(256), 0, st, pdl, a);
}

void launch_kv_append(const AttnArgs& a, int T, cudaStream_t st, bool pdl) {
  if (!a.tok_seq || !a.tok_off) throw Error(ERR_INVALID, "kv append needs the token map");
  launch(k_kv_append, dim3(T, a.Hkv), dim3(128), size_t(a.hd) * 4, st, pdl, a);
}

void launch_attn(const AttnArgs& a, cudaStream_t st, bool pdl, int T) {
  const int G = a.H / a.Hkv;
  if (G > 63 || a.hd > 256 || a.rot > a.hd || a.rot % 2) throw Error(ERR_UNSUPPORTED, "attention geometry outside the decode kernel's range");
  if (G * a.hd > ATTN_MAXO * ATTN_THREADS || a.nchunks > ATTN_CL * ATTN_CL || a.nchunks % ATTN_CL)
    throw Error(ERR_UNSUPPORTED, "attention shape outside the decode kernel's limits");
  const dim3 grid(a.Hkv, a.nchunks, T), block(ATTN_THREADS), cluster(1, ATTN_CL, 1);
  switch (a.hd) {
    case 16: launch_cluster(k_attn<16>, grid, block, cluster, attn_smem_bytes<16>(G, a.rot), st, pdl, a); break;
    case 32: launch_cluster(k_attn<32>, grid, block, cluster, attn_smem_bytes<32>(G, a.rot), st, pdl, a); break;
    case 64: launch_cluster(k_attn<64>, grid, block, cluster, attn_smem_bytes<64>(G, a.rot), st, pdl, a); break;
    case 128: launch_cluster(k_attn<128>, grid, block, cluster, attn_smem_bytes<128>(G, a.rot), st, pdl, a); break;
    case 256: launch_cluster(k_attn<256>, grid, block, cluster, attn_smem_bytes<256>(G, a.rot), st, pdl, a); break;
    default: throw Error(ERR_UNSUPPORTED, "attention head size must be 16, 32, 64, 128 or 256");
  }
  path_note("attn");
}

void launch_embed(const EmbedArgs& a, int hidden, cudaStream_t st, bool pdl) {
  launch(k_embed, dim3((hidden + 255) / 256), dim3(256), 0, st, pdl, a, hidden);
  path_note("embed");
}

// A wait that nothing completes: one mbarrier expecting an arrival that never
// comes, waited on with the streaming kernels' bounded wait and a short
// limit. Giving up sets bit 0 of the status word exactly as those kernels do;
// no copy is in flight, so nothing is left behind.
__global__ void k_wait_probe(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait_for(&bar, 0, limit_ns)) atomicOr(status, 1);
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&bar)) : "memory");
  }
}

void launch_wait_probe(int* status, unsigned long long limit_ns, cudaStream_t st) {
  launch(k_wait_probe, dim3(1), dim3(32), 0, st, false, status, limit_ns);
}

void launch_bembed(const EmbedArgs& a, int hidden, int T, cudaStream_t st, bool pdl) {
  EmbedArgs b = a;
  b.cursor = nullptr;
  launch(k_embed, dim3((hidden + 255) / 256, T), dim3(256), 0, st, pdl, b, hidden);
}

void launch_dequant(const QLin& l, int64_t r0, int64_t r1, float* out, cudaStream_t st) {
  const int64_t n = (r1 - r0) * int64_t(l.in);
  const int grid = int(std::min<int64_t>((n + 255) / 256, 4096));
  launch(k_dequant, dim3(std::max(grid, 1)), dim3(256), 0, st, false, l, r0, r1, out);
}

}  // namespace swl
