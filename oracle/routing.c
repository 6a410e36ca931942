/*
 * oracle/routing.c — CPU restatement of the MoE routing plan.  TEST INFRASTRUCTURE ONLY: it verifies
 * the GPU router/permute kernels, is never linked into libkdb200 and is never on the product path.
 *
 * The reference's routing plan is the `up_moe` plan stage (okc-challenge/engines/x3_h.cu:346-385):
 * per-expert token masks, popcount counts, an exclusive scan giving each expert's base row, and the
 * list of routed (token, expert) pairs grouped by expert in token order.  The bf16 layer
 * routes with an fp32 router inside the layer (softmax over logits, top-k, renormalised
 * weights), so the plan here starts from router logits:
 *
 *   1. logits[t, e] = fl32( dot(x[t, :], w[e, :]) ) (+ bias[e] as one fp32 add), where the dot
 *      product of the bf16 activation row and the fp32 router row is accumulated in fp64 in a fixed
 *      order (below) and rounded once to fp32.  Every product bf16*fp32 is exact in fp64, so the fp32
 *      logit is the correctly rounded dot product except when the fp64 sum lands within ~2^-29
 *      relative of an fp32 rounding boundary; the fixed order makes the GPU and this oracle agree
 *      bit for bit even then.
 *      Fixed order: 32 partial sums; h is cut into blocks of 256 and partial l accumulates, block by
 *      block in ascending order, the 8 consecutive elements h = 256*b + 8*l + j, j = 0..7 (those below
 *      H), with fma; then an xor butterfly over the 32 partials with offsets 16, 8, 4, 2, 1
 *      (p[l] + p[l^o]).  The order lets a GPU lane read 8 consecutive elements (16/32-byte vectors).
 *   2. top-k per token: the k largest logits in descending order; equal logits: lower expert first
 *      (torch.topk on a stable sort, and the `lst` order of x3_h.cu:371-385).
 *   3. permutation: rows grouped by expert (ascending), within an expert by token (ascending);
 *      counts, exclusive offsets, perm_slot[p] = t*k + j, slot_pos[t*k + j] = p.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static double canon_dot(const uint16_t* x, const float* w, int64_t H) {
  double part[32];
  for (int l = 0; l < 32; ++l) {
    double acc = 0.0;
    for (int64_t base = 0; base < H; base += 256)
      for (int j = 0; j < 8; ++j) {
        const int64_t h = base + 8 * l + j;
        if (h < H) acc = fma((double)bf16_to_f32(x[h]), (double)w[h], acc);
      }
    part[l] = acc;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    double nxt[32];
    for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ off];
    memcpy(part, nxt, sizeof nxt);
  }
  return part[0];
}

/* logits[T, E] (fp32) from x[T, H] (bf16 bits) and w[E, H] (fp32); bias may be NULL. */
void oracle_router_logits(const uint16_t* x, const float* w, const float* bias, int64_t T, int64_t H, int64_t E,
                          float* logits) {
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t e = 0; e < E; ++e) {
      float l = (float)canon_dot(x + t * H, w + e * H, H);
      if (bias) l = l + bias[e];
      logits[t * E + e] = l;
    }
  }
}

static int ranks_before(float va, int ia, float vb, int ib) {
  /* true when (va, ia) ranks before (vb, ib): larger value first, then lower index */
  return va > vb || (va == vb && ia < ib);
}

/* ids[T, k] (int32) and vals[T, k] (fp32): top-k logits per token, descending, ties -> lower index. */
void oracle_topk(const float* logits, int64_t T, int64_t E, int k, int32_t* ids, float* vals) {
  for (int64_t t = 0; t < T; ++t) {
    const float* row = logits + t * E;
    for (int j = 0; j < k; ++j) {
      int best = -1;
      for (int64_t e = 0; e < E; ++e) {
        int taken = 0;
        for (int q = 0; q < j; ++q)
          if (ids[t * k + q] == (int32_t)e) { taken = 1; break; }
        if (taken) continue;
        if (best < 0 || ranks_before(row[e], (int)e, row[best], best)) best = (int)e;
      }
      ids[t * k + j] = best;
      vals[t * k + j] = row[best];
    }
  }
}

/*
 * Permutation plan for ids[T, k] over E experts.
 *   counts[E], offsets[E + 1] (exclusive scan, offsets[E] = T*k),
 *   perm_slot[T*k]: the routed slot (t*k + j) at each permuted row,
 *   slot_pos[T*k]:  the permuted row of each slot.
 * Returns 0, or -1 if an id is out of range.
 */
int oracle_permute(const int32_t* ids, int64_t T, int k, int64_t E, int32_t* counts, int32_t* offsets,
                   int32_t* perm_slot, int32_t* slot_pos) {
  for (int64_t e = 0; e < E; ++e) counts[e] = 0;
  for (int64_t s = 0; s < T * k; ++s) {
    if (ids[s] < 0 || ids[s] >= E) return -1;
    counts[ids[s]]++;
  }
  offsets[0] = 0;
  for (int64_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  for (int64_t e = 0; e < E; ++e) counts[e] = 0; /* reused as fill cursors */
  for (int64_t s = 0; s < T * k; ++s) {
    const int32_t e = ids[s];
    const int32_t p = offsets[e] + counts[e]++;
    perm_slot[p] = (int32_t)s;
    slot_pos[s] = p;
  }
  for (int64_t e = 0; e < E; ++e) counts[e] = offsets[e + 1] - offsets[e];
  return 0;
}
