// Chunked-parallel gated delta rule for prompt (prefill) launches.
//
// The recurrence of one value head (QwenCPUModel.swift:459-488), state S
// [dv][dk]:  S <- g_t S;  u_t = beta_t (v_t - S k_t);  S <- S + u_t k_t^T;
// y_t = S q_t.  Over a chunk of C tokens starting from S_0, with the
// cumulative log-decay l_t = sum_{i<=t} log g_i (so g_t S_{t-1} = e^{l_t} S_0
// + sum_{j<t} e^{l_t - l_j} u_j k_j^T), the u_t solve a unit lower-triangular
// system and everything else is matrix products:
//   (I + L) U = R,   L_tj = beta_t e^{l_t - l_j} k_t.k_j   (j < t)
//                    R_t  = beta_t (v_t - e^{l_t} S_0 k_t)
//   y_t   = e^{l_t} S_0 q_t + sum_{j<=t} e^{l_t - l_j} (q_t.k_j) u_j
//   S_C   = e^{l_C} S_0 + sum_j e^{l_C - l_j} u_j k_j^T
// The rows of S (value dimensions) never mix, so a CTA takes 32 of them:
// grid (value heads, dv / 32, sequences), C = 64 tokens per chunk, the
// chunks of a sequence in order. Decays are formed as exponentials of
// log-decay differences (never ratios of products, which underflow).
// Arithmetic is f32 on the CUDA cores; the result equals the token-by-token
// recurrence up to f32 reassociation.
//
// k_delta_prep computes, per token, what the recurrence consumes: the causal
// conv over the token's sequence (history from the state's conv ring), SiLU,
// the q/k RMSNorms scaled 1/dk and 1/sqrt(dk), log g and beta
// (QwenCPUModel.swift:423-458) and the output gate silu(z).
#include <algorithm>

#include "kcommon.cuh"
#include "kernels.h"
#include "launch.h"

namespace swl {

constexpr int WY_C = 64;       // tokens per chunk
constexpr int WY_R = 32;       // state rows (value dims) per CTA
constexpr int WY_DK = 128;     // key head size the kernel takes
constexpr int WY_P = WY_DK + 4;  // padded row pitch of the token / state tiles (floats)
constexpr int WY_THREADS = 256;

struct WyLayout {
  static constexpr int Q = 0;                         // [C][P] normalised queries
  static constexpr int K = Q + WY_C * WY_P;           // [C][P] normalised keys
  static constexpr int S0 = K + WY_C * WY_P;          // [R][P] state rows
  static constexpr int L = S0 + WY_R * WY_P;          // [C][C+1] L (strictly lower)
  static constexpr int M = L + WY_C * (WY_C + 1);     // [C][C+1] e^{l_t - l_j} q_t.k_j (j <= t)
  static constexpr int V = M + WY_C * (WY_C + 1);     // [C][R+1] values, then R, then U
  static constexpr int W = V + WY_C * (WY_R + 1);     // [C][R+1] S_0 k_t
  static constexpr int Y = W + WY_C * (WY_R + 1);     // [C][R+1] S_0 q_t, then y
  static constexpr int LG = Y + WY_C * (WY_R + 1);    // [C] cumulative log decay
  static constexpr int BT = LG + WY_C;                // [C] beta
  static constexpr int TOTAL = BT + WY_C;             // floats
};

__global__ void __launch_bounds__(WY_THREADS, 1) k_delta_wy(const WyArgs a) {
  extern __shared__ __align__(16) float wsm[];
  float* Qs = wsm + WyLayout::Q;
  float* Ks = wsm + WyLayout::K;
  float* S0 = wsm + WyLayout::S0;
  float* Ls = wsm + WyLayout::L;
  float* Ms = wsm + WyLayout::M;
  float* Vs = wsm + WyLayout::V;
  float* Ws = wsm + WyLayout::W;
  float* Ys = wsm + WyLayout::Y;
  float* lg = wsm + WyLayout::LG;
  float* bt = wsm + WyLayout::BT;
  constexpr int LP = WY_C + 1, RP = WY_R + 1;
  const int hv = blockIdx.x, r0 = blockIdx.y * WY_R, sq = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = a.nv / a.nk, hk = hv / rep, dv = a.dv;
  float* S = a.state ? a.state : a.sd[sq].dstate[a.layer];
  S += (int64_t(hv) * dv + r0) * WY_DK;
  pdl_wait();
  const int t_first = a.seq_first ? a.seq_first[sq] : 0;
  const int n_all = a.seq_n ? a.seq_n[sq] : a.ntok;
  // the state rows of this CTA
  for (int i = tid; i < WY_R * (WY_DK / 4); i += WY_THREADS) {
    const int r = i / (WY_DK / 4), c = i % (WY_DK / 4);
    *reinterpret_cast<float4*>(S0 + r * WY_P + 4 * c) = reinterpret_cast<const float4*>(S + r * WY_DK)[c];
  }
  for (int c0 = 0; c0 < n_all; c0 += WY_C) {
    const int n = min(WY_C, n_all - c0);
    // ---- chunk inputs (rows past n are zero, beta 0, no further decay) ----
    for (int i = tid; i < WY_C * (WY_DK / 4); i += WY_THREADS) {
      const int t = i / (WY_DK / 4), c = i % (WY_DK / 4);
      float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), kv = qv;
      if (t < n) {
        const int64_t tok = t_first + c0 + t;
        qv = reinterpret_cast<const float4*>(a.q + tok * a.q_stride + hk * WY_DK)[c];
        kv = reinterpret_cast<const float4*>(a.k + tok * a.k_stride + hk * WY_DK)[c];
      }
      *reinterpret_cast<float4*>(Qs + t * WY_P + 4 * c) = qv;
      *reinterpret_cast<float4*>(Ks + t * WY_P + 4 * c) = kv;
    }
    for (int i = tid; i < WY_C * WY_R; i += WY_THREADS) {
      const int t = i / WY_R, c = i % WY_R;
      Vs[t * RP + c] = t < n ? a.v[(t_first + c0 + t) * a.v_stride + hv * dv + r0 + c] : 0.f;
    }
    if (warp == 0) {
      // inclusive scan of the log decays over the chunk (two per lane)
      float x0 = 0.f, x1 = 0.f, b0 = 0.f, b1 = 0.f;
      const int ta = 2 * lane, tb = 2 * lane + 1;
      if (ta < n) { x0 = a.lg[(t_first + c0 + ta) * a.gb_stride + 2 * hv]; b0 = a.lg[(t_first + c0 + ta) * a.gb_stride + 2 * hv + 1]; }
      if (tb < n) { x1 = a.lg[(t_first + c0 + tb) * a.gb_stride + 2 * hv]; b1 = a.lg[(t_first + c0 + tb) * a.gb_stride + 2 * hv + 1]; }
      float pair = x0 + x1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float up = __shfl_up_sync(0xffffffffu, pair, o);
        if (lane >= o) pair += up;
      }
      const float before = pair - (x0 + x1);
      lg[ta] = before + x0;
      lg[tb] = before + x0 + x1;
      bt[ta] = b0;
      bt[tb] = b1;
    }
    __syncthreads();
    // ---- K K^T (strictly lower) and Q K^T (lower): 4 x 4 tiles ----
    {
      const int ti = tid >> 4, tj = tid & 15;
      if (tj <= ti) {
        float A[4][4], B[4][4];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) { A[x][y] = 0.f; B[x][y] = 0.f; }
        for (int d = 0; d < WY_DK; d += 4) {
          float4 kt[4], qt[4], kj[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            kt[x] = *reinterpret_cast<const float4*>(Ks + (4 * ti + x) * WY_P + d);
            qt[x] = *reinterpret_cast<const float4*>(Qs + (4 * ti + x) * WY_P + d);
            kj[x] = *reinterpret_cast<const float4*>(Ks + (4 * tj + x) * WY_P + d);
          }
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              A[x][y] = fmaf(kt[x].x, kj[y].x, fmaf(kt[x].y, kj[y].y, fmaf(kt[x].z, kj[y].z, fmaf(kt[x].w, kj[y].w, A[x][y]))));
              B[x][y] = fmaf(qt[x].x, kj[y].x, fmaf(qt[x].y, kj[y].y, fmaf(qt[x].z, kj[y].z, fmaf(qt[x].w, kj[y].w, B[x][y]))));
            }
        }
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            const int t = 4 * ti + x, j = 4 * tj + y;
            const float dec = expf(lg[t] - lg[j]);
            Ls[t * LP + j] = j < t ? bt[t] * dec * A[x][y] : 0.f;
            Ms[t * LP + j] = j <= t ? dec * B[x][y] : 0.f;
          }
      }
    }
    // ---- S_0 k_t and S_0 q_t: 2 tokens x 4 rows per thread ----
    {
      const int tb = tid >> 3, ib = tid & 7;
      float w[2][4], y[2][4];
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int z = 0; z < 4; ++z) { w[x][z] = 0.f; y[x][z] = 0.f; }
      for (int d = 0; d < WY_DK; d += 4) {
        float4 kt[2], qt[2], sr[4];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          kt[x] = *reinterpret_cast<const float4*>(Ks + (2 * tb + x) * WY_P + d);
          qt[x] = *reinterpret_cast<const float4*>(Qs + (2 * tb + x) * WY_P + d);
        }
#pragma unroll
        for (int z = 0; z < 4; ++z) sr[z] = *reinterpret_cast<const float4*>(S0 + (4 * ib + z) * WY_P + d);
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int z = 0; z < 4; ++z) {
            w[x][z] = fmaf(kt[x].x, sr[z].x, fmaf(kt[x].y, sr[z].y, fmaf(kt[x].z, sr[z].z, fmaf(kt[x].w, sr[z].w, w[x][z]))));
            y[x][z] = fmaf(qt[x].x, sr[z].x, fmaf(qt[x].y, sr[z].y, fmaf(qt[x].z, sr[z].z, fmaf(qt[x].w, sr[z].w, y[x][z]))));
          }
      }
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int z = 0; z < 4; ++z) {
          Ws[(2 * tb + x) * RP + 4 * ib + z] = w[x][z];
          Ys[(2 * tb + x) * RP + 4 * ib + z] = y[x][z];
        }
    }
    __syncthreads();
    // ---- U = (I + L)^-1 R by forward substitution; the 8 lanes of a column
    // (same warp) split each row's sum ----
    {
      const int col = tid >> 3, part = tid & 7;
      for (int t = 0; t < n; ++t) {
        float s = 0.f;
        for (int j = part; j < t; j += 8) s = fmaf(Ls[t * LP + j], Vs[j * RP + col], s);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        // R_t in place of v_t, then u_t
        const float r = bt[t] * (Vs[t * RP + col] - expf(lg[t]) * Ws[t * RP + col]);
        __syncwarp();
        if (part == 0) Vs[t * RP + col] = r - s;
        __syncwarp();
      }
    }
    __syncthreads();
    // ---- y_t = e^{l_t} S_0 q_t + sum_{j<=t} M_tj u_j ----
    {
      const int tb = tid >> 3, ib = tid & 7;
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int t = 2 * tb + x;
        if (t >= n) continue;
        float acc[4];
        const float e = expf(lg[t]);
#pragma unroll
        for (int z = 0; z < 4; ++z) acc[z] = e * Ys[t * RP + 4 * ib + z];
        for (int j = 0; j <= t; ++j) {
          const float m = Ms[t * LP + j];
#pragma unroll
          for (int z = 0; z < 4; ++z) acc[z] = fmaf(m, Vs[j * RP + 4 * ib + z], acc[z]);
        }
        float* yo = a.y + (t_first + c0 + t) * a.y_stride + hv * dv + r0 + 4 * ib;
#pragma unroll
        for (int z = 0; z < 4; ++z) yo[z] = acc[z];
      }
    }
    // ---- S_C = e^{l_C} S_0 + sum_j e^{l_C - l_j} u_j k_j^T: 2 rows x 8 dims ----
    {
      const int ib = tid >> 4, db = tid & 15;
      const float lc = lg[n - 1], ec = expf(lc);
      float s[2][8];
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const float4 a0 = *reinterpret_cast<const float4*>(S0 + (2 * ib + x) * WY_P + 8 * db);
        const float4 a1 = *reinterpret_cast<const float4*>(S0 + (2 * ib + x) * WY_P + 8 * db + 4);
        s[x][0] = ec * a0.x; s[x][1] = ec * a0.y; s[x][2] = ec * a0.z; s[x][3] = ec * a0.w;
        s[x][4] = ec * a1.x; s[x][5] = ec * a1.y; s[x][6] = ec * a1.z; s[x][7] = ec * a1.w;
      }
      for (int j = 0; j < n; ++j) {
        const float c = expf(lc - lg[j]);
        const float u0 = c * Vs[j * RP + 2 * ib], u1 = c * Vs[j * RP + 2 * ib + 1];
        const float4 k0 = *reinterpret_cast<const float4*>(Ks + j * WY_P + 8 * db);
        const float4 k1 = *reinterpret_cast<const float4*>(Ks + j * WY_P + 8 * db + 4);
        const float kk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
        for (int z = 0; z < 8; ++z) {
          s[0][z] = fmaf(u0, kk[z], s[0][z]);
          s[1][z] = fmaf(u1, kk[z], s[1][z]);
        }
      }
      __syncthreads();  // every reader of S_0 above is done
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float* dst = S0 + (2 * ib + x) * WY_P + 8 * db;
        *reinterpret_cast<float4*>(dst) = make_float4(s[x][0], s[x][1], s[x][2], s[x][3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(s[x][4], s[x][5], s[x][6], s[x][7]);
      }
    }
    __syncthreads();
  }
  pdl_launch();
  for (int i = tid; i < WY_R * (WY_DK / 4); i += WY_THREADS) {
    const int r = i / (WY_DK / 4), c = i % (WY_DK / 4);
    reinterpret_cast<float4*>(S + r * WY_DK)[c] = *reinterpret_cast<const float4*>(S0 + r * WY_P + 4 * c);
  }
}

// Per token of a chunked launch: conv + SiLU of every mixed-qkv channel (the
// window slides over the token's own sequence, older inputs from the ring),
// the normalised q and k of every key head, v, log g and beta of every value
// head, and silu(z).
__global__ void __launch_bounds__(256) k_delta_prep(const DeltaArgs a, const WyArgs w) {
  extern __shared__ __align__(16) float xo[];  // [conv_dim]
  __shared__ float nrm[64];
  const int tok = blockIdx.x, tid = threadIdx.x;
  pdl_wait();
  const int s = w.tok_seq[tok], off = w.tok_off[tok];
  const StateDev* sd = a.sd + s;
  const int pos = *sd->pos, K = a.conv_k;
  const float* ring = sd->conv[a.layer];
  const int t0 = a.seq_first[s];
  const int dk = a.dk, keyDim = a.nk * dk, cd = a.conv_dim;
  for (int c = tid; c < cd; c += 256) {
    const int src = delta_src(a, c);
    float acc = 0.f;
    for (int jj = 0; jj < K; ++jj) {
      const int m = off - (K - 1) + jj;  // offset of the input within the sequence's launch tokens
      const float x = m >= 0 ? a.proj[int64_t(t0 + m) * a.proj_stride + src]
                             : ring[int64_t(((pos + m) % K + K) % K) * cd + c];
      acc += a.conv_w[c * K + jj] * x;
    }
    xo[c] = silu_ref(acc);
  }
  __syncthreads();
  // q / k RMSNorm per key head: warp w takes heads w, w + 8, ... of 2 * nk
  const int warp = tid >> 5, lane = tid & 31;
  for (int h = warp; h < 2 * a.nk; h += 8) {
    float ss = 0.f;
    for (int i = lane; i < dk; i += 32) ss += xo[h * dk + i] * xo[h * dk + i];
    ss = warp_sum(ss);
    if (lane == 0) nrm[h] = 1.f / sqrtf(ss / float(dk) + 1e-6f);
  }
  __syncthreads();
  pdl_launch();
  const float inv = 1.f / sqrtf(float(dk));
  float* qo = w.qw + int64_t(tok) * w.q_stride;
  float* ko = w.kw + int64_t(tok) * w.k_stride;
  for (int i = tid; i < keyDim; i += 256) {
    qo[i] = (xo[i] * nrm[i / dk]) * (inv * inv);
    ko[i] = (xo[keyDim + i] * nrm[a.nk + i / dk]) * inv;
  }
  float* vo = w.vw + int64_t(tok) * w.v_stride;
  for (int i = tid; i < a.nv * a.dv; i += 256) vo[i] = xo[2 * keyDim + i];
  const float* proj = a.proj + int64_t(tok) * a.proj_stride;
  for (int hv = tid; hv < a.nv; hv += 256) {
    int bi, ai;
    delta_ba(a, hv, bi, ai);
    // log g = -exp(A_log) softplus(a + dt_bias); g = exp(log g)
    w.lgw[int64_t(tok) * w.gb_stride + 2 * hv] = -expf(a.a_log[hv]) * softplus_ref(proj[ai] + a.dt_bias[hv]);
    w.lgw[int64_t(tok) * w.gb_stride + 2 * hv + 1] = sigmoid_ref(proj[bi]);
  }
  float* zo = a.z + int64_t(tok) * a.nv * a.dv;
  for (int i = tid; i < a.nv * a.dv; i += 256) {
    const int hv = i / a.dv, d = i - hv * a.dv;
    zo[i] = silu_ref(proj[delta_z(a, hv, d)]);
  }
}

// Decode-step inputs of the delta rule (one token per sequence, token t =
// sequence t), as k_delta_prep writes them for prompts, with one CTA per
// (token, block of 128 conv channels) and one channel per thread: the causal
// conv of the channel over the ring's K - 1 older inputs (read before the
// dependency wait) and the token's own, SiLU, and the token's input stored in
// ring slot pos % K (which none of its taps read). A q or k block is one key
// head: its RMSNorm (sum of squares in k_delta_prep's order) and scale
// 1/dk or 1/sqrt(dk) are applied in place. A value block also writes its
// channels' output gate silu(z), and its first thread the head's (log g,
// beta) (QwenCPUModel.swift:423-458).
__global__ void __launch_bounds__(128) k_delta_prep_dec(const DeltaArgs a, const WyArgs w) {
  __shared__ float sq[128];
  __shared__ float nrm;
  const int tok = blockIdx.x, c = blockIdx.y * 128 + threadIdx.x, lane = threadIdx.x & 31;
  const int K = a.conv_k, cd = a.conv_dim, dk = a.dk, keyDim = a.nk * dk;
  const StateDev* sd = a.sd + tok;
  const int pos = *sd->pos;
  float* ring = sd->conv[a.layer];
  float acc = 0.f;
  for (int jj = 0; jj < K - 1; ++jj)  // older inputs, oldest first: written by earlier steps
    acc += a.conv_w[c * K + jj] * ring[int64_t(((pos - (K - 1) + jj) % K + K) % K) * cd + c];
  pdl_wait();
  const float* proj = a.proj + int64_t(tok) * a.proj_stride;
  const float x = proj[delta_src(a, c)];
  acc += a.conv_w[c * K + K - 1] * x;
  ring[int64_t(pos % K) * cd + c] = x;
  const float o = silu_ref(acc);
  pdl_launch();
  if (c < 2 * keyDim) {
    sq[threadIdx.x] = o;
    __syncthreads();
    if (threadIdx.x < 32) {
      float ss = 0.f;
      for (int i = lane; i < dk; i += 32) ss += sq[i] * sq[i];
      ss = warp_sum(ss);
      if (lane == 0) nrm = 1.f / sqrtf(ss / float(dk) + 1e-6f);
    }
    __syncthreads();
    const float inv = 1.f / sqrtf(float(dk));
    if (c < keyDim) w.qw[int64_t(tok) * w.q_stride + c] = (o * nrm) * (inv * inv);
    else w.kw[int64_t(tok) * w.k_stride + c - keyDim] = (o * nrm) * inv;
  } else {
    const int i = c - 2 * keyDim, hv = i / a.dv, d = i - hv * a.dv;
    w.vw[int64_t(tok) * w.v_stride + i] = o;
    a.z[int64_t(tok) * a.nv * a.dv + i] = silu_ref(proj[delta_z(a, hv, d)]);
    if (d == 0) {
      int bi, ai;
      delta_ba(a, hv, bi, ai);
      w.lgw[int64_t(tok) * w.gb_stride + 2 * hv] = -expf(a.a_log[hv]) * softplus_ref(proj[ai] + a.dt_bias[hv]);
      w.lgw[int64_t(tok) * w.gb_stride + 2 * hv + 1] = sigmoid_ref(proj[bi]);
    }
  }
}

void launch_delta_prep_dec(const DeltaArgs& a, const WyArgs& w, int T, cudaStream_t st, bool pdl) {
  if (a.dk != 128 || a.conv_dim % 128 || a.dv > 128 || 128 % a.dv)
    throw Error(ERR_UNSUPPORTED, "delta rule decode inputs: head sizes outside the kernel's range");
  launch(k_delta_prep_dec, dim3(T, a.conv_dim / 128), dim3(128), 0, st, pdl, a, w);
}

// Decode step of the delta rule from k_delta_prep's per-token inputs (token
// blockIdx.z is its sequence's only token): RPW state rows of value head
// blockIdx.x per warp, lane l holding columns 4l..4l+3, loaded before the
// dependency wait; then S <- g S, S <- S + k beta (v - S k), y = S q
// (QwenCPUModel.swift:459-488, as k_delta4). With the per-head conv, norms
// and gates done once per token by the prep, a CTA's work after its wait is
// two float4 loads, its rows' v, the update and the stores, so the state
// streams at close to HBM rate.
template <int RPW, int NW>
__global__ void __launch_bounds__(NW * 32) k_delta_step(const WyArgs w) {
  constexpr int RB = RPW * NW, DK = WY_DK;
  const int hv = blockIdx.x, tok = blockIdx.z, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = hv / (w.nv / w.nk), dv = w.dv;
  const int row0 = blockIdx.y * RB + warp * RPW;
  float* S = w.sd[tok].dstate[w.layer];
  float4* S4 = reinterpret_cast<float4*>(S + (int64_t(hv) * dv + row0) * DK) + lane;
  float4 st[RPW];
#pragma unroll
  for (int j = 0; j < RPW; ++j) st[j] = S4[j * (DK / 4)];
  pdl_wait();
  const float4 qr = reinterpret_cast<const float4*>(w.q + int64_t(tok) * w.q_stride + hk * DK)[lane];
  const float4 kr = reinterpret_cast<const float4*>(w.k + int64_t(tok) * w.k_stride + hk * DK)[lane];
  const float lgv = w.lg[int64_t(tok) * w.gb_stride + 2 * hv], beta = w.lg[int64_t(tok) * w.gb_stride + 2 * hv + 1];
  const float vl = lane < RPW ? w.v[int64_t(tok) * w.v_stride + hv * dv + row0 + lane] : 0.f;
  pdl_launch();
  const float g = expf(lgv);
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
    const float delta = (__shfl_sync(0xffffffffu, vl, j) - kv[j]) * beta;
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
    w.y[int64_t(tok) * w.y_stride + hv * dv + row0 + lane] = yl;
  }
}

void launch_delta_step(const WyArgs& a, int T, cudaStream_t st, bool pdl) {
  constexpr int RPW = 4, NW = 8;
  if (a.dk != WY_DK || a.dv % (RPW * NW) || a.nv % a.nk)
    throw Error(ERR_UNSUPPORTED, "delta rule decode step: head sizes outside its range");
  launch(k_delta_step<RPW, NW>, dim3(a.nv, a.dv / (RPW * NW), T), dim3(NW * 32), 0, st, pdl, a);
  path_note("delta_step");
}

bool delta_wy_supported(int dk, int dv, int nk, int nv, int conv_dim) {
  return !std::getenv("SWL_NO_WY") && dk == WY_DK && dv % WY_R == 0 && 2 * nk <= 64 && nv % nk == 0 &&
         size_t(conv_dim) * 4 <= 64 * 1024;
}

void launch_delta_wy(const WyArgs& a, int S, cudaStream_t st, bool pdl) {
  if (a.dk != WY_DK || a.dv % WY_R) throw Error(ERR_UNSUPPORTED, "chunked delta rule: head sizes outside its range");
  launch(k_delta_wy, dim3(a.nv, a.dv / WY_R, S), dim3(WY_THREADS), size_t(WyLayout::TOTAL) * 4, st, pdl, a);
}

void launch_delta_prep(const DeltaArgs& a, const WyArgs& w, int T, cudaStream_t st, bool pdl) {
  launch(k_delta_prep, dim3(T), dim3(256), size_t(a.conv_dim) * 4, st, pdl, a, w);
}

}  // namespace swl
