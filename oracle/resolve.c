/*
 * CPU ORACLE -- test infrastructure only.
 *
 * Plain-C restatement of the reference's device expert cache, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg as
 * the CHECKER.  Nothing in the product path links or calls this file.
 *
 * Pinned against the reference itself: tests/golden/make_golden.py runs the
 * reference's own Triton kernels (_resolve_slots, _fetch_experts) under
 * TRITON_INTERPRET=1 on CPU and commits their outputs; tests/test_oracle_golden.py
 * checks every function below against those fixtures bit for bit.
 *
 *   oracle_resolve      bin/devcache.py:45-98   (_resolve_slots, LRU, one call)
 *   oracle_resolve_lfu  bin/simulate_cache.py:64-97 policy "lfu" (count reset to 1
 *                       on insert, ties to the earliest insertion), plus the
 *                       devcache.py:77-79 guard that a slot used in the current
 *                       step is never the victim
 *   oracle_fetch        bin/devcache.py:101-130, csrc/fetch_experts.cu:49-69
 *   oracle_replay       repeated oracle_resolve over a [steps][layers][k] trace,
 *                       per-layer caches as install_dev_cache builds them
 *                       (bin/devcache.py:280-301)
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

/* init_dev_cache, bin/devcache.py:147-152: slot_of=-1, slot_expert=-1,
 * stamp = -(C..1) so the first C misses fill slots 0,1,2,... in order, step=0. */
void oracle_init(int32_t* slot_of, int E, int32_t* slot_expert, int64_t* stamp, int C,
                 int64_t* step) {
  for (int e = 0; e < E; ++e) slot_of[e] = -1;
  for (int c = 0; c < C; ++c) {
    slot_expert[c] = -1;
    stamp[c] = -(int64_t)(C - c);
  }
  *step = 0;
}

/* One call of _resolve_slots (bin/devcache.py:45-98). Sequential over the k ids;
 * a miss takes the slot with the smallest stamp, strict '<' so the lowest index
 * wins ties (devcache.py:80-86); the victim's slot_of entry is cleared
 * (devcache.py:87-89). Returns nmiss. */
int oracle_resolve(const int32_t* ids, int k, int32_t* slot_of, int E, int32_t* slot_expert,
                   int64_t* stamp, int C, int32_t* out_slot, int32_t* fetch_slot,
                   int32_t* fetch_expert, int32_t* nmiss_out, int64_t* step_io) {
  (void)E;
  int64_t step = *step_io + 1;
  *step_io = step;
  int nmiss = 0;
  for (int i = 0; i < k; ++i) {
    int32_t e = ids[i];
    int32_t s = slot_of[e];
    if (s < 0) {
      int best = 0;
      int64_t best_stamp = stamp[0];
      for (int c = 1; c < C; ++c) {
        if (stamp[c] < best_stamp) { best_stamp = stamp[c]; best = c; }
      }
      int32_t victim = slot_expert[best];
      if (victim >= 0) slot_of[victim] = -1;
      slot_of[e] = best;
      slot_expert[best] = e;
      fetch_slot[nmiss] = best;
      fetch_expert[nmiss] = e;
      nmiss++;
      s = best;
    }
    stamp[s] = step;
    out_slot[i] = s;
  }
  *nmiss_out = nmiss;
  return nmiss;
}

/* LFU variant. Per slot: freq (uses since insertion, 1 on insert, 0 = empty)
 * and ins (insertion sequence; initial -(C-c) so empty slots fill in index
 * order). Victim = lexicographic min of (used_this_step, freq, ins, index).
 * Mirrors simulate_cache.py's lfu, which evicts min(count) with ties going to
 * the earliest-inserted key, with the devcache.py:77-79 current-step guard. */
int oracle_resolve_lfu(const int32_t* ids, int k, int32_t* slot_of, int E, int32_t* slot_expert,
                       int64_t* stamp, int64_t* freq, int64_t* ins, int C, int32_t* out_slot,
                       int32_t* fetch_slot, int32_t* fetch_expert, int32_t* nmiss_out,
                       int64_t* step_io) {
  (void)E;
  int64_t step = *step_io + 1;
  *step_io = step;
  int nmiss = 0;
  for (int i = 0; i < k; ++i) {
    int32_t e = ids[i];
    int32_t s = slot_of[e];
    if (s < 0) {
      int best = -1;
      int bu = 0; int64_t bf = 0, bi = 0;
      for (int c = 0; c < C; ++c) {
        int u = stamp[c] == step;
        int64_t f = freq[c], n = ins[c];
        if (best < 0 || u < bu || (u == bu && (f < bf || (f == bf && n < bi)))) {
          best = c; bu = u; bf = f; bi = n;
        }
      }
      int32_t victim = slot_expert[best];
      if (victim >= 0) slot_of[victim] = -1;
      slot_of[e] = best;
      slot_expert[best] = e;
      freq[best] = 0;
      ins[best] = (step << 8) | i;
      fetch_slot[nmiss] = best;
      fetch_expert[nmiss] = e;
      nmiss++;
      s = best;
    }
    freq[s] += 1;
    stamp[s] = step;
    out_slot[i] = s;
  }
  *nmiss_out = nmiss;
  return nmiss;
}

/* _fetch_experts / fetch_kernel: for j < njobs, copy expert idx[j]'s bytes from
 * src[idx[j]*bytes ...] to dst[slot[j]*bytes ...]. */
void oracle_fetch(const uint8_t* src, uint8_t* dst, const int32_t* idx, const int32_t* slot,
                  int njobs, int64_t bytes) {
  for (int j = 0; j < njobs; ++j)
    memcpy(dst + (int64_t)slot[j] * bytes, src + (int64_t)idx[j] * bytes, (size_t)bytes);
}

/* Replay a whole trace through per-layer caches of capacity C (policy 0 = LRU
 * oracle_resolve, 1 = LFU). trace is int16 [steps][layers][k]. Outputs:
 * per-step misses [steps] (summed over layers), totals hits/misses, and the
 * concatenated out slots [steps][layers][k] if out_slots != NULL. */
int oracle_replay(const int16_t* trace, int steps, int layers, int k, int E, int C, int policy,
                  int32_t* misses_per_step, int64_t* hits_total, int64_t* misses_total,
                  int32_t* out_slots) {
  int32_t* slot_of = (int32_t*)malloc(sizeof(int32_t) * (size_t)E * layers);
  int32_t* slot_expert = (int32_t*)malloc(sizeof(int32_t) * (size_t)C * layers);
  int64_t* stamp = (int64_t*)malloc(sizeof(int64_t) * (size_t)C * layers);
  int64_t* freq = (int64_t*)calloc((size_t)C * layers, sizeof(int64_t));
  int64_t* ins = (int64_t*)malloc(sizeof(int64_t) * (size_t)C * layers);
  int64_t* step = (int64_t*)calloc((size_t)layers, sizeof(int64_t));
  if (!slot_of || !slot_expert || !stamp || !freq || !ins || !step) return -1;
  for (int l = 0; l < layers; ++l) {
    oracle_init(slot_of + (size_t)l * E, E, slot_expert + (size_t)l * C, stamp + (size_t)l * C,
                C, step + l);
    for (int c = 0; c < C; ++c) ins[(size_t)l * C + c] = -(int64_t)(C - c);
  }
  int32_t ids[64], out[64], fs[64], fe[64], nm;
  int64_t hits = 0, misses = 0;
  for (int t = 0; t < steps; ++t) {
    int32_t ms = 0;
    for (int l = 0; l < layers; ++l) {
      const int16_t* row = trace + ((size_t)t * layers + l) * k;
      for (int i = 0; i < k; ++i) ids[i] = row[i];
      if (policy == 1)
        oracle_resolve_lfu(ids, k, slot_of + (size_t)l * E, E, slot_expert + (size_t)l * C,
                           stamp + (size_t)l * C, freq + (size_t)l * C, ins + (size_t)l * C, C,
                           out, fs, fe, &nm, step + l);
      else
        oracle_resolve(ids, k, slot_of + (size_t)l * E, E, slot_expert + (size_t)l * C,
                       stamp + (size_t)l * C, C, out, fs, fe, &nm, step + l);
      ms += nm;
      hits += k - nm;
      misses += nm;
      if (out_slots) memcpy(out_slots + ((size_t)t * layers + l) * k, out, sizeof(int32_t) * k);
    }
    if (misses_per_step) misses_per_step[t] = ms;
  }
  *hits_total = hits;
  *misses_total = misses;
  free(slot_of); free(slot_expert); free(stamp); free(freq); free(ins); free(step);
  return 0;
}
