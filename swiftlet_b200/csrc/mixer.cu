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
__device__ __forceinline__ int delta_src(const DeltaArgs& a, int c) {
  // Index into `proj` of mixed-qkv channel c.
  if (a.split) return c;
  const int keyDim = a.nk * a.dk, rep = a.nv / a.nk, chunk = 2 * a.dk + 2 * rep * a.dv;
  if (c < keyDim) { const int hk = c / a.dk; return hk * chunk + (c - hk * a.dk); }
  if (c < 2 * keyDim) { const int cc = c - keyDim, hk = cc / a.dk; return hk * chunk + a.dk + (cc - hk * a.dk); }
  const int cv = c - 2 * keyDim, hv = cv / a.dv, i = cv - hv * a.dv, hk = hv / rep, ri = hv - hk * rep;
  return hk * chunk + 2 * a.dk + ri * a.dv + i;
}
__device__ __forceinline__ int delta_z(const DeltaArgs& a, int hv, int i) {
  if (a.split) return a.conv_dim + hv * a.dv + i;
  const int rep = a.nv / a.nk, chunk = 2 * a.dk + 2 * rep * a.dv, hk = hv / rep, ri = hv - hk * rep;
  return hk * chunk + 2 * a.dk + rep * a.dv + ri * a.dv + i;
}
__device__ __forceinline__ void delta_ba(const DeltaArgs& a, int hv, int& bi, int& ai) {
  const int valueDim = a.nv * a.dv;
  if (a.split) { bi = a.conv_dim + valueDim + hv; ai = a.conv_dim + valueDim + a.nv + hv; return; }
  const int keyDim = a.nk * a.dk, rep = a.nv / a.nk, hk = hv / rep, ri = hv - hk * rep;
  const int base = 2 * keyDim + 2 * valueDim + hk * 2 * rep;
  bi = base + ri; ai = base + rep + ri;
}

constexpr int DELTA_THREADS = 128;
constexpr int DELTA_RPW = 8;  // rows per warp (RB <= 32)
constexpr int DELTA_EPL = 4;  // state elements per lane (dk <= 128)

__global__ void __launch_bounds__(DELTA_THREADS) k_delta(const DeltaArgs a) {
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
  const StateDev* sd = a.sd;
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
  float st[DELTA_RPW][DELTA_EPL];
#pragma unroll
  for (int j = 0; j < DELTA_RPW; ++j) {
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
    const float xn = a.proj[delta_src(a, c)];
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
    gb[0] = expf(-expf(alog) * softplus_ref(a.proj[ai] + dtb));
    gb[1] = sigmoid_ref(a.proj[bi]);
  }
  for (int i = threadIdx.x; i < RB; i += blockDim.x) {
    const int d = slice * RB + i;
    a.z[hv * dv + d] = silu_ref(a.proj[delta_z(a, hv, d)]);  // the output gate's activation
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
    if (r >= RB) continue;
    float* Sr = S + (int64_t(hv) * dv + slice * RB + r) * dk;
#pragma unroll
    for (int e = 0; e < DELTA_EPL; ++e) {
      const int i = lane + 32 * e;
      if (i < dk) Sr[i] = st[j][e];
    }
    if (lane == 0) a.y[hv * dv + slice * RB + r] = y[j];
  }
  trc.end(a.trace);
}

// ----------------------------------------------------------- attention ----
// Gated GQA decode for one token: q/k RMSNorm with weight, partial NeoX
// RoPE, KV append, causal softmax(q k^T / sqrt(hd)) v split over context
// chunks of at least ATTN_MINP positions, times sigmoid(gate)
// (QwenCPUModel.swift:285-367). KV layout: [kv_head][max_ctx][head_dim].
// A CTA walks its chunk in sub-tiles of ATTN_TP positions, double-buffered:
// the K and V rows of the next sub-tile are copied to shared memory
// (asynchronously; the first sub-tile's cached rows before the dependency
// wait) while the current one is scored. Scores take one warp per position
// with the G heads reduced together; an online softmax carries (max, sum,
// output) across sub-tiles. Every inner loop has a compile-time trip count
// (head size HD, sub-tile ATTN_TP; the rows of a short sub-tile are zero), so
// its loads issue together rather than one dependent round trip at a time.
// With one chunk the CTA writes the output; otherwise the last CTA of each kv
// head combines the chunks' partials.
//
// Output gate sigmoid with the fast exponential and divide (within a few
// ulp of 1 / (1 + exp(-v)); one per output element).
__device__ __forceinline__ float fast_sigmoid(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }

constexpr int ATTN_THREADS = 256;
constexpr int ATTN_MINP = 64;  // minimum positions per chunk
constexpr int ATTN_TP = 16;    // positions per staged sub-tile
constexpr int ATTN_MAXO = 16;  // output values per thread: G * hd <= ATTN_MAXO * ATTN_THREADS

template <int HD>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn(const AttnArgs a) {
  constexpr int E = HD >= 32 ? HD / 32 : 1;  // row elements per lane (l + 32e)
  constexpr int HQ = HD / 4;                 // float4 per row
  extern __shared__ __align__(16) float sm[];
  const int G = a.H / a.Hkv, kvh = blockIdx.x, chunk = blockIdx.y;
  const int half = a.rot / 2;
  float* q = sm;                      // [G][HD]
  float* kn = q + G * HD;             // [HD]
  float* vn = kn + HD;                // [HD]
  float* kvb = vn + HD;               // 2 x ([TP][HD] keys, [TP][HD] values)
  float* sc = kvb + 4 * ATTN_TP * HD; // [G][TP]
  float* fw = sc + G * ATTN_TP;       // [G][nchunks] combine weights
  float* cs = fw + G * a.nchunks;     // [half] cos
  float* sn = cs + half;              // [half] sin
  __shared__ float hm[64], hl[64], hal[64], hn[72];
  __shared__ bool last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  const StateDev* sd = a.sd;
  TraceRec trc;
  trc.start(a.trace);
  const int pos = *sd->pos;  // written by the previous token: complete
  const int ctx = pos + 1;
  const int nvalid = min(a.nchunks, (ctx + ATTN_MINP - 1) / ATTN_MINP);
  const int per = (ctx + nvalid - 1) / nvalid;
  const int p0 = chunk * per, p1 = min(ctx, p0 + per), n = chunk < nvalid ? max(0, p1 - p0) : 0;
  const int ntiles = (n + ATTN_TP - 1) / ATTN_TP;
  float* Kc = sd->kc[a.layer] + int64_t(kvh) * sd->max_ctx * HD;
  float* Vc = sd->vc[a.layer] + int64_t(kvh) * sd->max_ctx * HD;
  // copies of sub-tile t into buffer t & 1: cached rows asynchronously, the
  // rows past the chunk's end zeroed (the new position's row is written from
  // kn / vn once they are ready)
  auto stage = [&](int t) {
    float* kt = kvb + (t & 1) * 2 * ATTN_TP * HD;
    float* vt = kt + ATTN_TP * HD;
    const int t0 = p0 + t * ATTN_TP, nt = min(ATTN_TP, p0 + n - t0);
    for (int i = tid; i < ATTN_TP * HQ; i += ATTN_THREADS) {
      const int j = i / HQ, c = i - j * HQ, p = t0 + j;
      if (j < nt && p != pos) {
        cp_async16(kt + j * HD + 4 * c, Kc + int64_t(p) * HD + 4 * c);
        cp_async16(vt + j * HD + 4 * c, Vc + int64_t(p) * HD + 4 * c);
      } else if (j >= nt) {
        reinterpret_cast<float4*>(vt + j * HD)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
  };
  // before the wait: the first sub-tile's cached rows, RoPE table, norm weights
  if (ntiles > 0) stage(0);
  for (int j = tid; j < half; j += blockDim.x) {
    const float invf = powf(a.rope_theta, -float(2 * j) / float(a.rot));
    const float ang = float(pos) * invf;
    cs[j] = cosf(ang);
    sn[j] = sinf(ang);
  }
  for (int h = tid; h < G; h += blockDim.x) { hm[h] = -INFINITY; hl[h] = 0.f; }
  float wq[E], wk[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = lane + 32 * e;
    wq[e] = d < HD ? a.qn[d] : 0.f;
    wk[e] = d < HD ? a.kn[d] : 0.f;
  }
  pdl_wait();
  trc.waited(a.trace);
  for (int h = 0; h < G; ++h) copy_async(q + h * HD, a.qout + (kvh * G + h) * 2 * HD, HD);
  copy_async(kn, a.knew + kvh * HD, HD);
  copy_async(vn, a.vnew + kvh * HD, HD);
  cp_async_commit();
  cp_async_wait_group<0>();
  __syncthreads();
  pdl_launch();
  if (HD >= 32 && half % 32 == 0) {
    // one warp per head (G q heads and the new k head), in registers: lane l
    // holds elements l + 32e, so RoPE partners (j, j + half) share a lane
    const int hs = half >> 5;
    for (int h = warp; h <= G; h += nw) {
      float* x = h < G ? q + h * HD : kn;
      float v[E];
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        v[e] = x[lane + 32 * e];
        ss += v[e] * v[e];
      }
      ss = warp_sum(ss);
      const float sc0 = 1.f / sqrtf(ss / float(HD) + a.eps);
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] *= sc0 * (h < G ? wq[e] : wk[e]);
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (e < hs) {
          const int j = lane + 32 * e;
          float xb = 0.f;
#pragma unroll
          for (int f = 0; f < E; ++f)
            if (f == e + hs) xb = v[f];
          const float xa = v[e];
          v[e] = xa * cs[j] - xb * sn[j];
#pragma unroll
          for (int f = 0; f < E; ++f)
            if (f == e + hs) v[f] = xb * cs[j] + xa * sn[j];
        }
#pragma unroll
      for (int e = 0; e < E; ++e) x[lane + 32 * e] = v[e];
    }
  } else {
    // RMSNorm of G q heads and the new k head, one warp per head
    for (int h = warp; h <= G; h += nw) {
      float* x = h < G ? q + h * HD : kn;
      float ss = 0.f;
      for (int i = lane; i < HD; i += 32) ss += x[i] * x[i];
      ss = warp_sum(ss);
      if (lane == 0) hn[h] = 1.f / sqrtf(ss / float(HD) + a.eps);
    }
    __syncthreads();
    for (int i = tid; i < (G + 1) * HD; i += blockDim.x) {
      const int h = i / HD, d = i % HD;
      float* x = h < G ? q + h * HD : kn;
      const float* w = h < G ? a.qn : a.kn;
      x[d] *= hn[h] * w[d];
    }
    __syncthreads();
    for (int i = tid; i < (G + 1) * half; i += blockDim.x) {
      const int h = i / half, j = i % half;
      float* x = h < G ? q + h * HD : kn;
      const float xa = x[j], xb = x[half + j];
      x[j] = xa * cs[j] - xb * sn[j];
      x[half + j] = xb * cs[j] + xa * sn[j];
    }
  }
  __syncthreads();
  if (chunk == 0)
    for (int i = tid; i < HD; i += blockDim.x) {
      Kc[int64_t(pos) * HD + i] = kn[i];
      Vc[int64_t(pos) * HD + i] = vn[i];
    }
  trc.staged(a.trace);
  const float scale = 1.f / sqrtf(float(HD));
  const int nout = G * HD;
  float acc[ATTN_MAXO];
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) acc[o] = 0.f;
  for (int t = 0; t < ntiles; ++t) {
    float* kt = kvb + (t & 1) * 2 * ATTN_TP * HD;
    float* vt = kt + ATTN_TP * HD;
    const int t0 = p0 + t * ATTN_TP, nt = min(ATTN_TP, p0 + n - t0);
    if (t + 1 < ntiles) {
      stage(t + 1);
      cp_async_wait_group<1>();  // sub-tile t landed, t + 1 may still fly
    } else {
      cp_async_wait_group<0>();
    }
    if (pos >= t0 && pos < t0 + nt)  // the new position: its normalised, rotated key and its value
      for (int i = tid; i < HD; i += blockDim.x) {
        kt[(pos - t0) * HD + i] = kn[i];
        vt[(pos - t0) * HD + i] = vn[i];
      }
    __syncthreads();
    // scores: one warp per position; lane l covers elements l + 32e of the
    // row, and the head partials are reduced eight heads at a time
    for (int j = warp; j < ATTN_TP; j += nw) {
      const bool live = j < nt;
      float kv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) kv[e] = live && lane + 32 * e < HD ? kt[j * HD + lane + 32 * e] : 0.f;
      for (int h0 = 0; h0 < G; h0 += 8) {
        float pr[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const bool ok = h0 + r < G && lane + 32 * e < HD;
            d += (ok ? q[(h0 + r) * HD + lane + 32 * e] : 0.f) * kv[e];
          }
          pr[r] = d;
        }
        int rr;
        const float d = reduce_rows<8>(pr, 32, lane, rr);
        if ((lane & 3) == 0 && h0 + rr < G) sc[(h0 + rr) * ATTN_TP + j] = live ? d * scale : -INFINITY;
      }
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
#pragma unroll
    for (int o = 0; o < ATTN_MAXO; ++o) {
      const int i = tid + o * ATTN_THREADS;
      if (i < nout) {
        const int h = i / HD, d = i - h * HD;
        float v = acc[o] * hal[h];
#pragma unroll
        for (int j = 0; j < ATTN_TP; ++j) v += sc[h * ATTN_TP + j] * vt[j * HD + d];
        acc[o] = v;
      }
    }
    __syncthreads();
  }
  trc.looped(a.trace);
  if (nvalid == 1) {  // the whole context in this CTA: finish here
    if (chunk == 0) {
      for (int h = tid; h < G; h += blockDim.x) hal[h] = 1.f / hl[h];
      // every gate value is loaded before the first output is stored (the
      // stores would otherwise order each following load behind them)
      float gate[ATTN_MAXO];
#pragma unroll
      for (int o = 0; o < ATTN_MAXO; ++o) {
        const int i = tid + o * ATTN_THREADS;
        const int h = i / HD, d = i - h * HD;
        gate[o] = i < nout ? __ldcg(a.qout + (kvh * G + h) * 2 * HD + HD + d) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int o = 0; o < ATTN_MAXO; ++o) {
        const int i = tid + o * ATTN_THREADS;
        if (i < nout) {
          const int h = i / HD, d = i - h * HD;
          a.out[(kvh * G + h) * HD + d] = (acc[o] * hal[h]) * fast_sigmoid(gate[o]);
        }
      }
    }
    trc.end(a.trace);
    return;
  }
  float* part = a.part + (int64_t(kvh) * a.nchunks + chunk) * G * (HD + 2);
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    if (i < nout) {
      const int h = i / HD, d = i - h * HD;
      part[h * (HD + 2) + 2 + d] = acc[o];
    }
  }
  for (int h = tid; h < G; h += blockDim.x) { part[h * (HD + 2)] = n > 0 ? hm[h] : -INFINITY; part[h * (HD + 2) + 1] = hl[h]; }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(a.counters + kvh, 1u) == unsigned(a.nchunks) - 1;
  }
  __syncthreads();
  if (!last) {
    trc.end(a.trace);
    return;
  }
  __threadfence();
  // combine: per head the chunk weights f_c = exp(m_c - m) first
  const float* pk = a.part + int64_t(kvh) * a.nchunks * G * (HD + 2);
  for (int h = warp; h < G; h += nw) {
    float m = -INFINITY;
    for (int c = lane; c < nvalid; c += 32) m = fmaxf(m, __ldcg(pk + (int64_t(c) * G + h) * (HD + 2)));
    m = warp_max(m);
    float l = 0.f;
    for (int c = lane; c < nvalid; c += 32) {
      const float* pc = pk + (int64_t(c) * G + h) * (HD + 2);
      const float mc = __ldcg(pc);
      const float f = mc == -INFINITY ? 0.f : expf(mc - m);
      fw[h * a.nchunks + c] = f;
      l += __ldcg(pc + 1) * f;
    }
    l = warp_sum(l);
    if (lane == 0) hl[h] = l;
  }
  __syncthreads();
  for (int h = tid; h < G; h += blockDim.x) hal[h] = 1.f / hl[h];
  // all partial reads (every chunk's values of this thread's outputs in one
  // batch per chunk) and gate loads first, then the stores
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) acc[o] = 0.f;
  for (int c = 0; c < nvalid; ++c) {
    const float* pc = pk + int64_t(c) * G * (HD + 2) + 2;
    float v[ATTN_MAXO];
#pragma unroll
    for (int o = 0; o < ATTN_MAXO; ++o) {
      const int i = tid + o * ATTN_THREADS;
      const int h = i / HD, d = i - h * HD;
      v[o] = i < nout ? __ldcg(pc + h * (HD + 2) + d) : 0.f;
    }
#pragma unroll
    for (int o = 0; o < ATTN_MAXO; ++o) {
      const int i = tid + o * ATTN_THREADS;
      if (i < nout) acc[o] += v[o] * fw[(i / HD) * a.nchunks + c];
    }
  }
  float gate[ATTN_MAXO];
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    const int h = i / HD, d = i - h * HD;
    gate[o] = i < nout ? __ldcg(a.qout + (kvh * G + h) * 2 * HD + HD + d) : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    if (i < nout) {
      const int h = i / HD, d = i - h * HD;
      a.out[(kvh * G + h) * HD + d] = (acc[o] * hal[h]) * fast_sigmoid(gate[o]);
    }
  }
  if (tid == 0) a.counters[kvh] = 0u;
  trc.end(a.trace);
}

// --------------------------------------------------------------- embed ----
__global__ void k_embed(const EmbedArgs a, int D) {
  TraceRec trc;
  trc.start(a.trace);
  pdl_wait();
  trc.waited(a.trace);
  const int tok = a.tokens[*a.cursor];
  pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (tok < 0 || tok >= a.vocab) {
    if (i == 0) *a.err = 1;
    if (i < D) a.h[i] = 0.f;
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
  a.h[i] = v;
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
void launch_delta(const DeltaArgs& a, cudaStream_t st, bool pdl) {
  if (a.dk > 32 * DELTA_EPL || a.rows_per_block > DELTA_RPW * (DELTA_THREADS / 32) || a.dv % a.rows_per_block)
    throw Error(ERR_UNSUPPORTED, "DeltaNet head dims outside the decode kernel's range");
  const int nch = 2 * a.dk + a.rows_per_block;
  const size_t smem = size_t(2 * a.dk + a.rows_per_block + nch * (2 * a.conv_k - 1)) * 4;
  launch(k_delta, dim3(a.nv, a.dv / a.rows_per_block), dim3(DELTA_THREADS), smem, st, pdl, a);
}

void launch_attn(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int G = a.H / a.Hkv;
  if (G > 63 || a.hd > 256 || a.rot > a.hd) throw Error(ERR_UNSUPPORTED, "attention geometry outside the decode kernel's range");
  if (G * a.hd > ATTN_MAXO * ATTN_THREADS || a.nchunks > 64)
    throw Error(ERR_UNSUPPORTED, "attention shape outside the decode kernel's limits");
  const size_t smem = size_t(G * a.hd + 2 * a.hd + 4 * ATTN_TP * a.hd + G * ATTN_TP + G * a.nchunks + a.rot) * 4;
  switch (a.hd) {
    case 16: launch(k_attn<16>, dim3(a.Hkv, a.nchunks), dim3(ATTN_THREADS), smem, st, pdl, a); break;
    case 32: launch(k_attn<32>, dim3(a.Hkv, a.nchunks), dim3(ATTN_THREADS), smem, st, pdl, a); break;
    case 64: launch(k_attn<64>, dim3(a.Hkv, a.nchunks), dim3(ATTN_THREADS), smem, st, pdl, a); break;
    case 128: launch(k_attn<128>, dim3(a.Hkv, a.nchunks), dim3(ATTN_THREADS), smem, st, pdl, a); break;
    case 256: launch(k_attn<256>, dim3(a.Hkv, a.nchunks), dim3(ATTN_THREADS), smem, st, pdl, a); break;
    default: throw Error(ERR_UNSUPPORTED, "attention head size must be 16, 32, 64, 128 or 256");
  }
}

void launch_embed(const EmbedArgs& a, int hidden, cudaStream_t st, bool pdl) {
  launch(k_embed, dim3((hidden + 255) / 256), dim3(256), 0, st, pdl, a, hidden);
}

void launch_dequant(const QLin& l, int64_t r0, int64_t r1, float* out, cudaStream_t st) {
  const int64_t n = (r1 - r0) * int64_t(l.in);
  const int grid = int(std::min<int64_t>((n + 255) / 256, 4096));
  launch(k_dequant, dim3(std::max(grid, 1)), dim3(256), 0, st, false, l, r0, r1, out);
}

}  // namespace swl
