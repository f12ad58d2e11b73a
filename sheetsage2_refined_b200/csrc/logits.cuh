// Fused tied-logits projection, grammar mask, greedy argmax and slot commit.
//
// Replaces engine.py:315-357 (+ grammar.py:114-180): the final LayerNorm of
// the last layer, logits = bf16(x . E_v) widened to float32, plus an optional
// additive bias (mode_bias, engine.py:316-317), masked by the grammar, argmax
// with the lowest index winning ties (torch.argmax), then for every live slot:
// write the token to out[slot, position+1], advance the grammar, stop on
// EOS / stop time / context limit.
//
// Every CTA scores an interleaved subset of the vocabulary for all rows and
// publishes its best (value, index) per row with one 64-bit atomicMax on a key
// whose high word orders the float value and whose low word is ~index, so the
// maximum is the largest logit and, among equal logits, the lowest index.  The
// last CTA to finish (a ticket counter) commits the step and resets the keys
// and the counter for the next step.  The grammar mask is never materialised:
// the class grammar evaluates its 13 class predicates once per row and reads
// bit token_class[v]; the table grammar reads table[state, v].
#pragma once

#include "common.cuh"
#include "proj.cuh"
#include "select.cuh"

namespace s2r {

struct Grammar {
  int kind;  // 0 class, 1 table
  const int8_t* token_class;
  const int32_t* field_of_class;
  const double* time_seconds;
  int states;
  int multiplier;
  const uint8_t* table;
};

// Frame-head rescoring (engine.py:81-116,318-347,358-369): additive terms
// from per-slot per-frame tables, looked up at the slot's current frame, on
// the chord detail, bass, key, eighth-position and meter spans, and the state
// they read (current frame, key stated, active meter, last meter a change).
// Weights in the reference's FRAME_TERMS order.
enum FrameTerm { FT_ROOT = 0, FT_BASS, FT_DETAIL, FT_QUALITY, FT_KEY, FT_KEY_BOUNDARY, FT_DOWNBEAT, FT_METER, FT_COUNT };

struct Rescore {
  int on;
  float w[FT_COUNT];
  int b0, b1, d0, d1, k0, k1, e0, e1, m0, m1;  // bass, detail, key, eighth-position and meter spans
  int frames;                                  // table rows per slot
  const float* table[FT_COUNT];                // [slots][frames][width of the term]
  const int32_t* meter_beats;                  // [meters] min(numerator, 16) - 1
  const int32_t* meter_unit;                   // [meters] denominator
  int32_t* frame_now;                          // [slots]
  uint8_t* key_seen;                           // [slots]
  int32_t* active_meter;                       // [slots], -1 none
  uint8_t* meter_changed;                      // [slots]
};

struct LogitsArgs {
  int M, V, D, max_tokens;
  SlotState st;
  Grammar gr;
  const float* r;  // [M, D] residual sums before the last final_norm; with acc: the residual input x
  const unsigned long long* acc;  // null, or [M, D] fixed-point fc2 sums: the input is x + bf16(acc + acc_bias)
  const bf16* acc_bias;           // [D] fc2 bias
  const float* gamma;
  const float* beta;
  const bf16* emb;    // tied output embedding [V, D], bfloat16
  const float* bias;  // [V] or null
  unsigned long long* keys;  // [M * kKeyStride] (row m at m * kKeyStride), zero between steps
  unsigned int* counter;     // zero between steps
  const int64_t* forced;     // [M] or null: commit forced[m] >= 0 instead of the greedy token
  float* logits_out;         // [M, V] or null: raw logits
  int64_t* greedy_out;       // [M] or null
  Rescore rs;                // frame-head rescoring (rs.on == 0: none)
  L2Ahead ahead;              // what the next step's first kernel reads, prefetched into the L2
};

// Class grammar constants (grammar.py:19-55).
constexpr int kEosT = 0, kShiftT = 1, kTimeT = 2, kMeterT = 3, kPitchT = 8, kBassT = 10;
constexpr int kNone = 0, kAfterMeter = 1, kAfterPitch = 2, kAfterBass = 3, kMaxShiftRun = 4;

// The 13 class predicates of grammar.py:117-137 as a bit mask.
__device__ __forceinline__ uint32_t class_mask(const SlotState& st, int s) {
  const int64_t last = st.last_field[s], inc = st.incomplete[s], payload = st.payload[s], run = st.shift_run[s];
  const bool in_shift = st.in_shift[s] != 0;
  const bool free_ = inc == kNone, open_chord = inc == kAfterBass;
  uint32_t m = 0;
  m |= (uint32_t)((payload > 0) && !open_chord) << 0;
  m |= (uint32_t)(((payload > 0) || in_shift) && (run < kMaxShiftRun) && !open_chord) << 1;
  m |= (uint32_t)(free_ && last < 0) << 2;
  m |= (uint32_t)(free_ && last < 1) << 3;
  m |= (uint32_t)((inc == kAfterMeter) || (free_ && last < 1)) << 4;
  m |= (uint32_t)(free_ && last < 2) << 5;
  m |= (uint32_t)(free_ && last < 3) << 6;
  m |= (uint32_t)(free_ && last < 4) << 7;
  m |= (uint32_t)((inc == kAfterPitch) || (free_ && last <= 5)) << 8;
  m |= (uint32_t)(inc == kAfterPitch) << 9;
  m |= (uint32_t)(free_ && last < 4) << 10;
  m |= (uint32_t)open_chord << 11;
  return m;  // bit 12 (other) is never set
}

// grammar.py:140-180 for one slot (class grammar) or the table rule.
__device__ __forceinline__ void grammar_update(const Grammar& gr, const SlotState& st, int s, int64_t tok, bool active,
                                               bool at_limit) {
  if (gr.kind == 1) {
    const int64_t g = (gr.multiplier * st.g[s] + tok) % gr.states;
    const int64_t count = st.count[s] + 1;
    const bool done = count >= st.target[s];
    const bool fin = done || at_limit;
    if (active) {
      st.g[s] = g;
      st.count[s] = count;
      if (fin) {
        st.ended[s] = done ? 1 : 3;
        st.finished[s] = 1;
      }
    }
    return;
  }
  const int kind = gr.token_class[tok];
  const bool is_shift = kind == kShiftT;
  const bool is_field = kind != kShiftT && kind != kEosT;
  const bool in_shift = st.in_shift[s] != 0;
  const bool new_event = is_shift && !in_shift && st.payload[s] > 0;
  int64_t payload = new_event ? 0 : st.payload[s];
  if (is_field) payload += 1;
  int64_t last = new_event ? -1 : st.last_field[s];
  if (is_field) last = gr.field_of_class[kind];
  int64_t inc = new_event ? kNone : st.incomplete[s];
  if (is_field) inc = kind == kMeterT ? kAfterMeter : kind == kPitchT ? kAfterPitch : kind == kBassT ? kAfterBass : kNone;
  const bool new_in_shift = is_shift ? true : (is_field ? false : in_shift);
  const int64_t run = is_shift ? st.shift_run[s] + 1 : (is_field ? 0 : st.shift_run[s]);
  const bool eos = kind == kEosT;
  const bool stopped = kind == kTimeT && gr.time_seconds[tok] >= st.stop[s];
  const bool fin = eos || stopped || at_limit;
  if (active) {
    st.payload[s] = payload;
    st.last_field[s] = last;
    st.incomplete[s] = inc;
    st.in_shift[s] = new_in_shift;
    st.shift_run[s] = run;
    if (fin) {
      st.ended[s] = eos ? 1 : stopped ? 2 : 3;
      st.finished[s] = 1;
    }
  }
}

__host__ __device__ constexpr int frame_term_width(int term, int no_chord) {
  return term == FT_ROOT || term == FT_BASS ? 12
         : term == FT_DETAIL || term == FT_QUALITY ? no_chord
         : term == FT_KEY ? 24
         : term == FT_METER ? 16
                            : 1;
}

// The per-slot rescoring state a row's logits read: loaded once per row.
struct RescoreRow {
  int now;            // current frame
  int active;         // active meter, -1 none
  uint8_t key_seen;   // a key has been stated
  uint8_t no_eighth;  // the last token changed the meter (eighth positions after 0 are barred)
};

__device__ __forceinline__ RescoreRow rescore_row(const Rescore& r, const SlotState& st, int s) {
  RescoreRow rr{0, -1, 0, 0};
  if (r.on) {
    rr.now = r.frame_now[s];
    rr.active = r.active_meter[s];
    rr.key_seen = r.key_seen[s];
    rr.no_eighth = st.incomplete[s] == kAfterMeter && r.meter_changed[s];
  }
  return rr;
}

// x = logit + mode bias of token v for slot s, plus the rescoring terms in
// the reference's order (engine.py:318-347); -inf for the eighth positions
// after a meter change.  Terms with a zero weight are not added at all.
__device__ __forceinline__ float rescore_logit_row(const Rescore& r, const RescoreRow& rr, int s, int v, float x) {
  if (!r.on) return x;
  const int now = rr.now;
  auto row = [&](int term) {
    return r.table[term] + ((size_t)s * r.frames + now) * frame_term_width(term, r.d1 - r.d0);
  };
  if (v >= r.d0 && v < r.d1) {
    const int i = v - r.d0;
    if (r.w[FT_ROOT] != 0.f) x += r.w[FT_ROOT] * row(FT_ROOT)[i % 12];
    if (r.w[FT_DETAIL] != 0.f) x += r.w[FT_DETAIL] * row(FT_DETAIL)[i];
    if (r.w[FT_QUALITY] != 0.f) x += r.w[FT_QUALITY] * row(FT_QUALITY)[i];
  }
  if (v >= r.b0 && v < r.b1 && r.w[FT_BASS] != 0.f) x += r.w[FT_BASS] * row(FT_BASS)[v - r.b0];
  if (v >= r.k0 && v < r.k1) {
    if (r.w[FT_KEY] != 0.f) x += r.w[FT_KEY] * row(FT_KEY)[v - r.k0];
    if (r.w[FT_KEY_BOUNDARY] != 0.f)
      x += r.w[FT_KEY_BOUNDARY] * row(FT_KEY_BOUNDARY)[0] * (rr.key_seen ? 1.f : 0.f);
  }
  if (v == r.e0 && r.w[FT_DOWNBEAT] != 0.f) x += r.w[FT_DOWNBEAT] * row(FT_DOWNBEAT)[0];
  if (r.w[FT_METER] != 0.f) {
    if (v >= r.m0 && v < r.m1) {
      const int m = v - r.m0, act = rr.active, a = act < 0 ? 0 : act;
      const bool change = act >= 0 && m != a;
      const bool same_unit = r.meter_unit[m] == r.meter_unit[a];
      const float* t = row(FT_METER);
      x += r.w[FT_METER] * (t[r.meter_beats[m]] - t[r.meter_beats[a]]) * ((change && same_unit) ? 1.f : 0.f);
      if (r.w[FT_DOWNBEAT] != 0.f) x += r.w[FT_DOWNBEAT] * row(FT_DOWNBEAT)[0] * (change ? 1.f : 0.f);
    }
    if (v > r.e0 && v < r.e1 && rr.no_eighth) x = -INFINITY;
  }
  return x;
}

__device__ __forceinline__ float rescore_logit(const Rescore& r, const SlotState& st, int s, int v, float x) {
  if (!r.on) return x;
  return rescore_logit_row(r, rescore_row(r, st, s), s, v, x);
}

// Token v lies in a span some rescoring term can move.
__device__ __forceinline__ bool rescored_token(const Rescore& r, int v) {
  return r.on && ((v >= r.d0 && v < r.d1) || (v >= r.b0 && v < r.b1) || (v >= r.k0 && v < r.k1) ||
                  (v >= r.e0 && v < r.e1) || (v >= r.m0 && v < r.m1));
}

// The rescoring terms as one out-of-line function: the logits epilogues call it
// from loops unrolled over rows, which inlined copies would make too large for
// the instruction cache.  Only tokens in a rescored span call it.
static __device__ __noinline__ float rescore_logit_call(const Rescore& r, const RescoreRow& rr, int s, int v, float x) {
  return rescore_logit_row(r, rr, s, v, x);
}

// Rescoring state after slot s committed `tok` (engine.py:358-369).
__device__ __forceinline__ void rescore_commit(const Rescore& r, const Grammar& gr, int s, int64_t tok, bool active) {
  if (!r.on || !active) return;
  const double seconds = gr.time_seconds[tok];
  if (seconds > -INFINITY) {
    long long f = (long long)(seconds * 25.0);
    f = f < 0 ? 0 : (f > r.frames - 1 ? r.frames - 1 : f);
    r.frame_now[s] = (int32_t)f;
  }
  if (tok >= r.k0 && tok < r.k1) r.key_seen[s] = 1;
  if (tok >= r.m0 && tok < r.m1) {
    const int m = (int)(tok - r.m0);
    r.meter_changed[s] = r.active_meter[s] >= 0 && m != r.active_meter[s];
    r.active_meter[s] = m;
  }
}

// Commit one step for rows [0, M) once every key is final: the greedy token
// (or the forced one) is written to out[slot, position+1], the grammar
// advances and the keys return to zero.  Run by one CTA.
__device__ __forceinline__ void commit_rows(const LogitsArgs& a) {
  for (int s = threadIdx.x; s < a.M; s += blockDim.x) {
    const unsigned long long k = atomicExch(a.keys + (size_t)s * kKeyStride, 0ull);
    const int64_t greedy = key_token(k);
    if (a.greedy_out) a.greedy_out[s] = greedy;
    const bool active = a.st.finished[s] == 0;
    const int64_t tok = a.st.token[s], pos = a.st.position[s];
    int64_t choice = greedy;
    if (a.forced && a.forced[s] >= 0) choice = a.forced[s];
    if (!active) choice = tok;
    const int64_t new_pos = active ? pos + 1 : pos;
    if (active && new_pos < a.max_tokens) a.st.out[(size_t)s * a.max_tokens + new_pos] = choice;
    grammar_update(a.gr, a.st, s, choice, active, new_pos >= a.max_tokens - 1);
    rescore_commit(a.rs, a.gr, s, choice, active);
    a.st.token[s] = choice;
    a.st.position[s] = new_pos;
  }
}

// The grammar rule of row s: its class mask (class grammar) or its state (table grammar).
__device__ __forceinline__ uint32_t row_rule(const Grammar& gr, const SlotState& st, int s) {
  return gr.kind == 1 ? (uint32_t)st.g[s] : class_mask(st, s);
}

__device__ __forceinline__ bool token_allowed(const Grammar& gr, uint32_t rule, int V, int v) {
  return gr.kind == 1 ? gr.table[(size_t)rule * V + v] != 0 : ((rule >> gr.token_class[v]) & 1u) != 0;
}

constexpr int kLogitsThreads = 256;

template <int KCH, int MC>
__global__ void __launch_bounds__(kLogitsThreads) logits_kernel(const __grid_constant__ LogitsArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int KP = KCH * 256;
  constexpr int NW = kLogitsThreads / 32;
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);  // [MC][KP]
  __shared__ uint32_t rule[MC];                   // class mask or table state per row
  __shared__ RescoreRow rrow[MC];                 // rescoring state per row
  __shared__ unsigned long long wbest[NW][MC];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = a.D;
  const int stride = gridDim.x * NW;
  const int first = blockIdx.x * NW + warp;
  // Embedding rows a warp keeps in flight: narrow rows (D <= 512) of a large vocabulary leave a
  // warp ~14 rows of 1 KB, so it loads U of them before the first dot product; wide rows leave
  // it about one.
  constexpr int U = (KCH <= 2 && MC == 1) ? 4 : 1;

  uint4 w[U][KCH];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int v = first + u * stride;
#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      const int col = c * 256 + lane * 8;
      w[u][c] = (v < a.V && col < D) ? ld_stream(a.emb + (size_t)v * D + col) : make_uint4(0, 0, 0, 0);
    }
  }
  if (threadIdx.x == 0) l2_ahead(a.ahead, blockIdx.x, gridDim.x);
  pdl_launch_dependents();
  pdl_wait();

  // LayerNorm staging shares the projection kernel's code path.
  ProjArgs pa{};
  pa.M = a.M;
  pa.K = D;
  pa.r = a.r;
  pa.acc = a.acc;
  pa.acc_bias = a.acc_bias;
  pa.gamma = a.gamma;
  pa.beta = a.beta;
  pa.x_out = nullptr;

  for (int m0 = 0; m0 < a.M; m0 += MC) {
    const int mc = min(MC, a.M - m0);
    if (m0 > 0) __syncthreads();
    if constexpr (MC == 1) {
      if (a.acc)
        stage_ln_row_block<KCH, IN_ACC, NW * 32>(pa, xs, m0, a.gamma, a.beta, false);
      else
        stage_ln_row_block<KCH, IN_LN, NW * 32>(pa, xs, m0, a.gamma, a.beta, false);
    } else if (a.acc) {
      stage_ln_rows<KCH, IN_ACC>(pa, xs, m0, mc, warp, lane, NW);
    } else {
      stage_ln_rows<KCH, IN_LN>(pa, xs, m0, mc, warp, lane, NW);
    }
    for (int idx = threadIdx.x; idx < (MC - mc) * (KP / 8); idx += blockDim.x) {
      const int i = mc + idx / (KP / 8), col = (idx % (KP / 8)) * 8;
      *reinterpret_cast<uint4*>(xs + (size_t)i * KP + col) = make_uint4(0, 0, 0, 0);
    }
    if (threadIdx.x < MC) {
      const int s = m0 + threadIdx.x;
      rule[threadIdx.x] = threadIdx.x < mc ? row_rule(a.gr, a.st, s) : 0u;
      rrow[threadIdx.x] = threadIdx.x < mc ? rescore_row(a.rs, a.st, s) : RescoreRow{0, -1, 0, 0};
    }
    __syncthreads();

    unsigned long long best[MC];
#pragma unroll
    for (int i = 0; i < MC; ++i) best[i] = 0ull;
    // rows v0 + u * stride, u < U, of this warp per pass (a row's arithmetic does not depend on U)
    for (int v0 = first; v0 < a.V; v0 += U * stride) {
      if (v0 != first || m0 > 0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int v = v0 + u * stride;
#pragma unroll
          for (int c = 0; c < KCH; ++c) {
            const int col = c * 256 + lane * 8;
            w[u][c] = (v < a.V && col < D) ? ld_stream(a.emb + (size_t)v * D + col) : make_uint4(0, 0, 0, 0);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * stride;
        if (U > 1 && v >= a.V) break;  // uniform across the warp (with U = 1 the loop bound checks it)
        const float bias = a.bias ? a.bias[v] : 0.f;
        const int cls = a.gr.kind == 1 ? 0 : a.gr.token_class[v];
        const bool rescored = rescored_token(a.rs, v);
#pragma unroll
        for (int i = 0; i < MC; ++i) {
          float acc = 0.f;
#pragma unroll
          for (int c = 0; c < KCH; ++c)
            acc += dot8(w[u][c], *reinterpret_cast<const uint4*>(xs + (size_t)i * KP + c * 256 + lane * 8));
          acc = warp_sum(acc);
          if (i < mc) {
            const float logit = round_bf16(acc);
            if (a.logits_out && lane == 0) a.logits_out[(size_t)(m0 + i) * a.V + v] = logit;
            const bool ok =
                a.gr.kind == 1 ? a.gr.table[(size_t)rule[i] * a.V + v] != 0 : ((rule[i] >> cls) & 1u) != 0;
            if (ok) {
              const float x = rescored ? rescore_logit_call(a.rs, rrow[i], m0 + i, v, logit + bias) : logit + bias;
              const unsigned long long k = argmax_key(x, v);
              best[i] = k > best[i] ? k : best[i];
            }
          }
        }
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < MC; ++i) wbest[warp][i] = best[i];
    }
    __syncthreads();
    if (threadIdx.x < mc) {
      unsigned long long k = 0ull;
      for (int ww = 0; ww < NW; ++ww) k = wbest[ww][threadIdx.x] > k ? wbest[ww][threadIdx.x] : k;
      if (k) atomicMax(a.keys + (size_t)(m0 + threadIdx.x) * kKeyStride, k);
    }
  }

  // ---- the last CTA commits the step
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  commit_rows(a);
  if (threadIdx.x == 0) *a.counter = 0u;
}

}  // namespace s2r
