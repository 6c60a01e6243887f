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
// A CTA walks its chunk in sub-tiles of ATTN_TP positions: the K and V rows
// are copied to shared memory in one asynchronous round trip, scores are
// half-dots by thread pairs (row index rotated by position: no bank
// conflicts), and an online softmax carries (max, sum, output) across
// sub-tiles. With one chunk the CTA writes the output; otherwise the last CTA
// of each kv head combines the chunks' partials.
// Output gate sigmoid with the fast exponential and divide (within a few
// ulp of 1 / (1 + exp(-v)); one per output element).
__device__ __forceinline__ float fast_sigmoid(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }

constexpr int ATTN_THREADS = 256;
constexpr int ATTN_MINP = 64;  // minimum positions per chunk
constexpr int ATTN_TP = 16;    // positions per staged sub-tile
constexpr int ATTN_MAXO = 16;  // output values per thread: G * hd <= ATTN_MAXO * ATTN_THREADS

__global__ void __launch_bounds__(ATTN_THREADS) k_attn(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int hd = a.hd, G = a.H / a.Hkv, kvh = blockIdx.x, chunk = blockIdx.y;
  const int half = a.rot / 2;
  float* q = sm;                      // [G][hd]
  float* kn = q + G * hd;             // [hd]
  float* vn = kn + hd;                // [hd]
  float* kt = vn + hd;                // [TP][hd]
  float* vt = kt + ATTN_TP * hd;      // [TP][hd]
  float* sc = vt + ATTN_TP * hd;      // [G][TP]
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
  float* Kc = sd->kc[a.layer] + int64_t(kvh) * sd->max_ctx * hd;
  float* Vc = sd->vc[a.layer] + int64_t(kvh) * sd->max_ctx * hd;
  // before the wait: L2 prefetch of this chunk's cached rows, RoPE table
  if (tid == 0 && n > 0) {
    const int old = min(p1, pos) - p0;  // rows < pos are already cached
    if (old > 0) {
      prefetch_l2(Kc + int64_t(p0) * hd, uint32_t(old) * hd * 4);
      prefetch_l2(Vc + int64_t(p0) * hd, uint32_t(old) * hd * 4);
    }
  }
  for (int j = tid; j < half; j += blockDim.x) {
    const float invf = powf(a.rope_theta, -float(2 * j) / float(a.rot));
    const float ang = float(pos) * invf;
    cs[j] = cosf(ang);
    sn[j] = sinf(ang);
  }
  for (int h = tid; h < G; h += blockDim.x) { hm[h] = -INFINITY; hl[h] = 0.f; }
  pdl_wait();
  trc.waited(a.trace);
  for (int h = 0; h < G; ++h) copy_async(q + h * hd, a.qout + (kvh * G + h) * 2 * hd, hd);
  copy_async(kn, a.knew + kvh * hd, hd);
  copy_async(vn, a.vnew + kvh * hd, hd);
  cp_async_wait_all();
  __syncthreads();
  pdl_launch();
  if (hd % 32 == 0 && hd <= 256 && half % 32 == 0) {
    // one warp per head (G q heads and the new k head), in registers: lane l
    // holds elements l + 32e, so RoPE partners (j, j + half) share a lane
    const int E = hd >> 5, hs = half >> 5;
    for (int h = warp; h <= G; h += nw) {
      float* x = h < G ? q + h * hd : kn;
      const float* w = h < G ? a.qn : a.kn;
      float v[8];
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[e] = e < E ? x[lane + 32 * e] : 0.f;
        ss += v[e] * v[e];
      }
      ss = warp_sum(ss);
      const float sc = 1.f / sqrtf(ss / float(hd) + a.eps);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < E) v[e] *= sc * w[lane + 32 * e];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < hs) {
          const int j = lane + 32 * e;
          const float xa = v[e], xb = v[e + hs];
          v[e] = xa * cs[j] - xb * sn[j];
          v[e + hs] = xb * cs[j] + xa * sn[j];
        }
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < E) x[lane + 32 * e] = v[e];
    }
    __syncthreads();
  } else {
    // RMSNorm of G q heads and the new k head, one warp per head
    for (int h = warp; h <= G; h += nw) {
      float* x = h < G ? q + h * hd : kn;
      float ss = 0.f;
      for (int i = lane; i < hd; i += 32) ss += x[i] * x[i];
      ss = warp_sum(ss);
      if (lane == 0) hn[h] = 1.f / sqrtf(ss / float(hd) + a.eps);
    }
    __syncthreads();
    for (int i = tid; i < (G + 1) * hd; i += blockDim.x) {
      const int h = i / hd, d = i % hd;
      float* x = h < G ? q + h * hd : kn;
      const float* w = h < G ? a.qn : a.kn;
      x[d] *= hn[h] * w[d];
    }
    __syncthreads();
    for (int i = tid; i < (G + 1) * half; i += blockDim.x) {
      const int h = i / half, j = i % half;
      float* x = h < G ? q + h * hd : kn;
      const float xa = x[j], xb = x[half + j];
      x[j] = xa * cs[j] - xb * sn[j];
      x[half + j] = xb * cs[j] + xa * sn[j];
    }
    __syncthreads();
  }
  if (chunk == 0)
    for (int i = tid; i < hd; i += blockDim.x) {
      Kc[int64_t(pos) * hd + i] = kn[i];
      Vc[int64_t(pos) * hd + i] = vn[i];
    }
  trc.staged(a.trace);
  const float scale = 1.f / sqrtf(float(hd));
  const int nout = G * hd;
  float acc[ATTN_MAXO];
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) acc[o] = 0.f;
  const int hq = hd >> 2;  // float4 per row
  for (int t0 = p0; t0 < p0 + n; t0 += ATTN_TP) {
    const int nt = min(ATTN_TP, p0 + n - t0);
    // stage rows t0 .. t0 + nt of K and V (the new position from kn / vn)
    for (int i = tid; i < nt * hq; i += blockDim.x) {
      const int j = i / hq, c = i - j * hq, p = t0 + j;
      if (p == pos) {
        reinterpret_cast<float4*>(kt + j * hd)[c] = reinterpret_cast<const float4*>(kn)[c];
        reinterpret_cast<float4*>(vt + j * hd)[c] = reinterpret_cast<const float4*>(vn)[c];
      } else {
        cp_async16(kt + j * hd + 4 * c, Kc + int64_t(p) * hd + 4 * c);
        cp_async16(vt + j * hd + 4 * c, Vc + int64_t(p) * hd + 4 * c);
      }
    }
    cp_async_wait_all();
    __syncthreads();
    // scores: one warp per position; lane l covers elements l + 32e of the
    // row, and the G head partials are reduced together, eight heads at a
    // time (transposed reduction)
    for (int j = warp; j < ATTN_TP; j += nw) {
      const bool live = j < nt;
      float kv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) kv[e] = live && lane + 32 * e < hd ? kt[j * hd + lane + 32 * e] : 0.f;
      for (int h0 = 0; h0 < G; h0 += 8) {
        float p[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float d = 0.f;
          if (h0 + r < G)
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (lane + 32 * e < hd) d += q[(h0 + r) * hd + lane + 32 * e] * kv[e];
          p[r] = d;
        }
        int rr;
        const float d = reduce_rows<8>(p, 32, lane, rr);
        if ((lane & 3) == 0 && h0 + rr < G) sc[(h0 + rr) * ATTN_TP + j] = live ? d * scale : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax: per head the new max, the rescale of what came before,
    // the weights of this sub-tile
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
        const int h = i / hd, d = i - h * hd;
        float v = acc[o] * hal[h];
        for (int j = 0; j < nt; ++j) v += sc[h * ATTN_TP + j] * vt[j * hd + d];
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
        const int h = i / hd, d = i - h * hd;
        gate[o] = i < nout ? __ldcg(a.qout + (kvh * G + h) * 2 * hd + hd + d) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int o = 0; o < ATTN_MAXO; ++o) {
        const int i = tid + o * ATTN_THREADS;
        if (i < nout) {
          const int h = i / hd, d = i - h * hd;
          a.out[(kvh * G + h) * hd + d] = (acc[o] * hal[h]) * fast_sigmoid(gate[o]);
        }
      }
    }
    trc.end(a.trace);
    return;
  }
  float* part = a.part + (int64_t(kvh) * a.nchunks + chunk) * G * (hd + 2);
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    if (i < nout) {
      const int h = i / hd, d = i - h * hd;
      part[h * (hd + 2) + 2 + d] = acc[o];
    }
  }
  for (int h = tid; h < G; h += blockDim.x) { part[h * (hd + 2)] = n > 0 ? hm[h] : -INFINITY; part[h * (hd + 2) + 1] = hl[h]; }
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
  const float* pk = a.part + int64_t(kvh) * a.nchunks * G * (hd + 2);
  for (int h = warp; h < G; h += nw) {
    float m = -INFINITY;
    for (int c = lane; c < nvalid; c += 32) m = fmaxf(m, __ldcg(pk + (int64_t(c) * G + h) * (hd + 2)));
    m = warp_max(m);
    float l = 0.f;
    for (int c = lane; c < nvalid; c += 32) {
      const float* pc = pk + (int64_t(c) * G + h) * (hd + 2);
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
  __syncthreads();
  // all partial reads and gate loads first, then the stores (see above)
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    acc[o] = 0.f;
    if (i < nout) {
      const int h = i / hd, d = i - h * hd;
      for (int c = 0; c < nvalid; ++c)
        acc[o] += __ldcg(pk + (int64_t(c) * G + h) * (hd + 2) + 2 + d) * fw[h * a.nchunks + c];
    }
  }
  float gate[ATTN_MAXO];
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    const int h = i / hd, d = i - h * hd;
    gate[o] = i < nout ? __ldcg(a.qout + (kvh * G + h) * 2 * hd + hd + d) : 0.f;
  }
#pragma unroll
  for (int o = 0; o < ATTN_MAXO; ++o) {
    const int i = tid + o * ATTN_THREADS;
    if (i < nout) {
      const int h = i / hd, d = i - h * hd;
      a.out[(kvh * G + h) * hd + d] = (acc[o] * hal[h]) * fast_sigmoid(gate[o]);
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
  if (G * a.hd > ATTN_MAXO * ATTN_THREADS || G > 64 || a.hd % 4 || a.nchunks > 64)
    throw Error(ERR_UNSUPPORTED, "attention shape outside the decode kernel's limits");
  const size_t smem = size_t(G * a.hd + 2 * a.hd + 2 * ATTN_TP * a.hd + G * ATTN_TP + G * a.nchunks + a.rot) * 4;
  launch(k_attn, dim3(a.Hkv, a.nchunks), dim3(ATTN_THREADS), smem, st, pdl, a);
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
