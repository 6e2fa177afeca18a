// pb_attn_fast.cuh - the split-position decode attention of the fast mode
// for one query (head_dim 64), shared by k_attn_dec_fast (pb_ops.cu) and the
// fused projection + attention kernel k_qkv_attn (pb_q4.cu).
//
// The nsplit CTAs of a kv head g are one thread-block cluster; CTA sp holds
// the positions [sp * P, (sp + 1) * P), P = ceil(cache_len / nsplit), K rows
// padded to AQ_KLD floats in shared memory, V rows, and the PER query heads
// of the group.  aq_attend then computes, with AQ_THREADS threads (any
// further threads of the block only take part in the barriers):
//   scores (thread per position, f32 dots of the four 16-dim quarters), per
//   head the split's max m_c, p_j = exp(s_j - m_c), S_c = sum p_j, O_c = sum
//   p_j V_j (four position groups, summed in order);
//   cluster barrier, then CTA sp merges a slice of the PER x 64 outputs from
//   every split's shared memory (distributed shared memory), in split order:
//   M = max m_c, out = sum O_c e^(m_c - M) / sum S_c e^(m_c - M); a second
//   barrier keeps each CTA's shared memory alive until read.
// f32 throughout (the reference sums in double, llama-streaming.js:543-573):
// the differences are of f32 rounding, within the fast mode's tolerance; the
// split depends only on the cache length, so results do not depend on
// scheduling.
#pragma once

#include <cooperative_groups.h>

#include "pb_internal.cuh"

constexpr int AQ_THREADS = 128, AQ_HD = 64, AQ_KLD = 68, AQ_MAXP = 256, AQ_MAX_SPLIT = 8;

// Dynamic shared memory of the attention part: K [pmax][AQ_KLD], V
// [pmax][64], scores [PER][pmax], q [PER][64], PV partials [4][PER][64].
static inline size_t aq_smem(int per, int pmax) {
  return ((size_t)pmax * AQ_KLD + (size_t)pmax * AQ_HD + (size_t)per * pmax + (size_t)per * AQ_HD +
          (size_t)4 * per * AQ_HD) * 4;
}

// The split's partial state, kept in static shared memory by the kernel.
template <int PER>
struct aq_parts {
  float red_m[PER][AQ_THREADS / 32], red_s[PER][AQ_THREADS / 32];
  float part_m[PER], part_s[PER];
  __align__(16) float part_o[PER * AQ_HD];
};

// Every thread of the block calls it after the split's K/V rows (n of them)
// and q are in shared memory (and a block barrier); writes this CTA's slice
// of the group's outputs to out_g.
template <int PER>
__device__ __forceinline__ void aq_attend(cooperative_groups::cluster_group& cl, const float* ks, const float* vs,
                                          float* sc, const float* qs, float* gp, aq_parts<PER>& pt, int n, int pmax,
                                          float scale, float* __restrict__ out_g) {
  const int sp = (int)cl.block_rank(), nsplit = (int)cl.num_blocks(), tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const bool act = tid < AQ_THREADS;
  // scores: thread per position, four independent 16-dim chains per head
  for (int t = tid; act && t < n; t += AQ_THREADS) {
    const float4* kr = reinterpret_cast<const float4*>(ks + t * AQ_KLD);
    float a[PER][4];
#pragma unroll
    for (int h = 0; h < PER; ++h) a[h][0] = a[h][1] = a[h][2] = a[h][3] = 0.0f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float4 k4 = kr[u];
#pragma unroll
      for (int h = 0; h < PER; ++h) {
        const float4 q4 = reinterpret_cast<const float4*>(qs + h * AQ_HD)[u];
        float& acc = a[h][u & 3];
        acc = fmaf(q4.x, k4.x, acc);
        acc = fmaf(q4.y, k4.y, acc);
        acc = fmaf(q4.z, k4.z, acc);
        acc = fmaf(q4.w, k4.w, acc);
      }
    }
#pragma unroll
    for (int h = 0; h < PER; ++h) sc[h * pmax + t] = ((a[h][0] + a[h][1]) + (a[h][2] + a[h][3])) * scale;
  }
  __syncthreads();
  // per head: the split's max (`s > m` from -Infinity: NaN never wins), then p and its sum
  if (act) {
#pragma unroll
    for (int h = 0; h < PER; ++h) {
      float m = -INFINITY;
      for (int t = tid; t < n; t += AQ_THREADS) m = sc[h * pmax + t] > m ? sc[h * pmax + t] : m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float o_ = __shfl_xor_sync(0xffffffffu, m, o);
        m = o_ > m ? o_ : m;
      }
      if (lane == 0) pt.red_m[h][warp] = m;
    }
  }
  __syncthreads();
  if (act) {
#pragma unroll
    for (int h = 0; h < PER; ++h) {
      float m = pt.red_m[h][0];
      for (int w = 1; w < AQ_THREADS / 32; ++w) m = pt.red_m[h][w] > m ? pt.red_m[h][w] : m;
      float s_ = 0.0f;
      for (int t = tid; t < n; t += AQ_THREADS) {
        const float p = expf(sc[h * pmax + t] - m);
        sc[h * pmax + t] = p;
        s_ += p;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s_ += __shfl_xor_sync(0xffffffffu, s_, o);
      if (lane == 0) pt.red_s[h][warp] = s_;
    }
  }
  __syncthreads();
  // PV: thread (dim pair dp, position group jg), positions jg, jg + 4, ...
  if (act) {
    const int dp = tid & 31, jg = tid >> 5;
    float2 acc[PER];
#pragma unroll
    for (int h = 0; h < PER; ++h) acc[h] = make_float2(0.0f, 0.0f);
    for (int t = jg; t < n; t += 4) {
      const float2 v = reinterpret_cast<const float2*>(vs + t * AQ_HD)[dp];
#pragma unroll
      for (int h = 0; h < PER; ++h) {
        const float p = sc[h * pmax + t];
        acc[h].x = fmaf(p, v.x, acc[h].x);
        acc[h].y = fmaf(p, v.y, acc[h].y);
      }
    }
#pragma unroll
    for (int h = 0; h < PER; ++h) reinterpret_cast<float2*>(gp + ((size_t)jg * PER + h) * AQ_HD)[dp] = acc[h];
  }
  __syncthreads();
  for (int i = tid; act && i < PER * AQ_HD; i += AQ_THREADS)
    pt.part_o[i] = ((gp[i] + gp[PER * AQ_HD + i]) + gp[2 * PER * AQ_HD + i]) + gp[3 * PER * AQ_HD + i];
  if (tid < PER) {  // (from shared memory: a per-head register indexed by tid would go to local memory)
    float m = pt.red_m[tid][0];
    for (int w = 1; w < AQ_THREADS / 32; ++w) m = pt.red_m[tid][w] > m ? pt.red_m[tid][w] : m;
    pt.part_m[tid] = n > 0 ? m : -INFINITY;
    pt.part_s[tid] = n > 0 ? ((pt.red_s[tid][0] + pt.red_s[tid][1]) + pt.red_s[tid][2]) + pt.red_s[tid][3] : 0.0f;
  }
  cl.sync();  // every split's partial is written
  // this CTA's slice of the outputs, merged over the splits in order
  const int per_cta = (PER * AQ_HD + nsplit - 1) / nsplit;
  const int i = sp * per_cta + tid;
  if (tid < per_cta && i < PER * AQ_HD) {
    const int h = i / AQ_HD;
    float M = -INFINITY;
    for (int c = 0; c < nsplit; ++c) {
      const float s_ = *cl.map_shared_rank(&pt.part_s[h], c), m_ = *cl.map_shared_rank(&pt.part_m[h], c);
      if (s_ != 0.0f && m_ > M) M = m_;
    }
    float S = 0.0f, O = 0.0f;
    for (int c = 0; c < nsplit; ++c) {
      const float s_ = *cl.map_shared_rank(&pt.part_s[h], c);
      if (s_ == 0.0f) continue;  // an empty split
      const float f = expf(*cl.map_shared_rank(&pt.part_m[h], c) - M);
      S = fmaf(s_, f, S);
      O = fmaf(*cl.map_shared_rank(&pt.part_o[i], c), f, O);
    }
    out_g[i] = O / S;
  }
  cl.sync();  // the other CTAs have read this one's partial
}
