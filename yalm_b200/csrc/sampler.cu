// On-device sampler: yalm's Sampler (src/sampler.cpp:11-64) over the logits the classifier just
// wrote, so a decode loop reads back 4 bytes per token instead of the vocab_size fp32 logits.
//
//  op 0  sample_argmax: the first index of the maximum (strict `>` from -FLT_MAX, so NaN logits
//        are skipped and index 0 is returned when no logit exceeds -FLT_MAX).
//  op 1  sample(temperature): max m as above, S = sum_i exp((l_i - m) / T); the first index whose
//        running sum of exp((l_i - m) / T) / S reaches coin (the host draws coin, as yalm draws
//        rand() / RAND_MAX), else vocab_size - 1.  The running sum is formed per thread segment
//        plus a block scan, so it is rounded differently from yalm's sequential float sum: the
//        returned index can differ only when coin lies within rounding error of a boundary.
//  op 2  sample_prob(target): exp(l_target - m) / sum_i exp(l_i - m).
#include "sampler.cuh"

#include <cfloat>

namespace yb {

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const float* logits, int vocab_size,
                                                                const StepState* step, SampleParams direct,
                                                                SampleResult* out) {
  __shared__ float s_val[kSampleThreads / 32];
  __shared__ int s_idx[kSampleThreads / 32];
  __shared__ float s_seg[kSampleThreads];
  __shared__ float s_m, s_sum;
  __shared__ int s_pick;
  pdl_trigger();
  pdl_wait();  // the logits come from the classifier (and, tensor parallel, the gather)
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int op = step ? step->sample_op : direct.op;
  const float T = op == 1 ? (step ? step->temperature : direct.temperature) : 1.0f;
  const unsigned epoch = step ? step->epoch : direct.epoch;
  const int seg = (vocab_size + kSampleThreads - 1) / kSampleThreads;
  const int i0 = t * seg, i1 = min(vocab_size, i0 + seg);

  // max and first index of the max
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = i0; i < i1; ++i) {
    const float v = logits[i];
    if (v > best) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_val[warp] = best;
    s_idx[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kSampleThreads / 32 ? s_val[lane] : -FLT_MAX;
    bi = lane < kSampleThreads / 32 ? s_idx[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_m = best;
      s_pick = bi == 0x7fffffff ? 0 : bi;
    }
  }
  __syncthreads();
  const float m = s_m;
  if (op == 0) {
    if (t == 0) {
      out->token = s_pick;
      out->prob = 0.f;
      out->epoch = epoch;
    }
    return;
  }

  // per-thread segment sums of exp((l - m) / T), then an inclusive block scan
  float local = 0.f;
  for (int i = i0; i < i1; ++i) local += expf((logits[i] - m) / T);
  s_seg[t] = local;
  __syncthreads();
  for (int o = 1; o < kSampleThreads; o <<= 1) {
    const float v = t >= o ? s_seg[t - o] : 0.f;
    __syncthreads();
    s_seg[t] += v;
    __syncthreads();
  }
  if (t == kSampleThreads - 1) s_sum = s_seg[t];
  if (t == 0) s_pick = vocab_size - 1;
  __syncthreads();
  const float sum = s_sum;
  if (op == 2) {
    if (t == 0) {
      const int tg = step ? step->sample_target : direct.target;
      out->token = tg;
      out->prob = (tg >= 0 && tg < vocab_size) ? expf(logits[tg] - m) / sum : 0.f;
      out->epoch = epoch;
    }
    return;
  }
  // op 1: the first segment whose inclusive sum reaches coin * sum scans its own elements
  const float target = (step ? step->coin : direct.coin) * sum;
  const float before = t > 0 ? s_seg[t - 1] : 0.f;
  if (s_seg[t] >= target && (t == 0 || before < target)) {
    float c = before;
    int pick = i1 - 1;
    for (int i = i0; i < i1; ++i) {
      c += expf((logits[i] - m) / T);
      if (c >= target) {
        pick = i;
        break;
      }
    }
    if (i1 > i0) s_pick = pick;
  }
  __syncthreads();
  if (t == 0) {
    out->token = s_pick;
    out->prob = 0.f;
    out->epoch = epoch;
  }
}

}  // namespace yb
