/*
 * CPU oracle for the cu_roaring B200 engine — TEST INFRASTRUCTURE ONLY.
 * See roaring_oracle.h for the contract. Every function cites the reference
 * file:line whose behaviour it restates.
 */
#include "roaring_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define CHUNK_WORDS 1024u
#define T_ARRAY 0
#define T_BITMAP 1
#define T_RUN 2
#define PROMOTE_KEEP_DEFAULT 4096u
#define PROMOTE_AUTO 0xFFFFFFFFu

/* ---------------------------------------------------------------- helpers */

static uint32_t popc64(uint64_t x) { return (uint32_t)__builtin_popcountll(x); }

/* Number of valid bits of chunk `key` inside [0, U). */
static uint32_t chunk_valid_bits(uint32_t key, uint32_t U)
{
  uint64_t lo = (uint64_t)key << 16;
  if (lo >= U) return 0;
  uint64_t rem = (uint64_t)U - lo;
  return rem >= 65536u ? 65536u : (uint32_t)rem;
}

static void mask_valid(uint64_t* w, uint32_t valid)
{
  for (uint32_t i = 0; i < CHUNK_WORDS; ++i) {
    uint32_t lo = i * 64u;
    if (lo >= valid) w[i] = 0;
    else if (valid - lo < 64u) w[i] &= (1ull << (valid - lo)) - 1ull;
  }
}

static uint32_t chunk_popcount(const uint64_t* w)
{
  uint32_t c = 0;
  for (uint32_t i = 0; i < CHUNK_WORDS; ++i) c += popc64(w[i]);
  return c;
}

/* A run starts at every set bit whose predecessor bit is clear. */
static uint32_t chunk_runs(const uint64_t* w)
{
  uint32_t r = 0;
  uint64_t carry = 0;
  for (uint32_t i = 0; i < CHUNK_WORDS; ++i) {
    r += popc64(w[i] & ~((w[i] << 1) | carry));
    carry = w[i] >> 63;
  }
  return r;
}

void or_image_free(or_image* im)
{
  if (!im) return;
  free(im->keys); free(im->types); free(im->offsets); free(im->cards);
  free(im->key_index); free(im->bitmap); free(im->array); free(im->run);
  memset(im, 0, sizeof(*im));
}

/* ------------------------------------------------------ canonical typing */

/* The canonical container rule of this engine (stated in prose, not taken
 * from CRoaring):
 *   t < 4096 (an explicit promotion request, reference src/upload.cpp:106 and
 *            src/upload_ids.cu:493): BITMAP if c > t else ARRAY;
 *   otherwise: ARRAY if c <= 4096 (the Roaring array/bitmap cut-off);
 *              RUN if 4r < 8192 and the run form is smaller than the
 *                  alternative (BITMAP when c > t, ARRAY when c <= t);
 *              ARRAY if c <= t; else BITMAP.
 * Runs therefore only replace containers that would otherwise be large. */
int or_container_type(uint32_t c, uint32_t r, uint32_t t)
{
  if (t < PROMOTE_KEEP_DEFAULT) return c > t ? T_BITMAP : T_ARRAY;
  if (c <= PROMOTE_KEEP_DEFAULT) return T_ARRAY;
  if (r < 2048u && (c > t || 4ull * r < 2ull * c)) return T_RUN;
  if (c <= t) return T_ARRAY;
  return T_BITMAP;
}

/* Reference src/promote.cu:334-367: PROMOTE_ALL iff 2*ceil(U/8) > L2. */
uint32_t or_resolve_auto_threshold(uint32_t U, uint64_t l2_bytes)
{
  if (U == 0) return PROMOTE_KEEP_DEFAULT;
  uint64_t flat = ((uint64_t)U + 7u) / 8u;
  return flat * 2u > l2_bytes ? 0u : PROMOTE_KEEP_DEFAULT;
}

/* ------------------------------------------------------- image assembly */

typedef struct chunk_list {
  uint32_t n;
  uint16_t* keys;
  uint64_t* words; /* n * 1024, stored (physical) contents */
} chunk_list;

static void chunk_list_free(chunk_list* cl)
{
  free(cl->keys); free(cl->words);
  cl->keys = NULL; cl->words = NULL; cl->n = 0;
}

static uint32_t max_key_of(uint32_t U) { return U == 0 ? 0u : ((U - 1u) >> 16); }

/* Emits the compact packed image of the stored chunks. `types_in` forces a
 * per-chunk type (NULL = canonical rule with threshold t). Empty chunks are
 * dropped. total = cardinality of the logical set. */
static void assemble(const chunk_list* cl, const uint8_t* types_in, uint32_t t, uint32_t U,
                     int negated, uint64_t total, or_image* out)
{
  memset(out, 0, sizeof(*out));
  out->universe_size = U;
  out->negated = negated;
  out->total_cardinality = total;
  uint32_t n = 0;
  uint8_t* ty = (uint8_t*)malloc(cl->n + 1);
  uint32_t* card = (uint32_t*)malloc(sizeof(uint32_t) * (cl->n + 1));
  uint32_t* runs = (uint32_t*)malloc(sizeof(uint32_t) * (cl->n + 1));
  uint64_t arr_elems = 0, run_pairs = 0;
  uint32_t nb = 0, na = 0, nr = 0;
  for (uint32_t i = 0; i < cl->n; ++i) {
    const uint64_t* w = cl->words + (size_t)i * CHUNK_WORDS;
    card[i] = chunk_popcount(w);
    runs[i] = chunk_runs(w);
    if (card[i] == 0) { ty[i] = 0xFF; continue; }
    ty[i] = types_in ? types_in[i] : (uint8_t)or_container_type(card[i], runs[i], t);
    ++n;
    if (ty[i] == T_BITMAP) ++nb;
    else if (ty[i] == T_ARRAY) { ++na; arr_elems += card[i]; }
    else { ++nr; run_pairs += runs[i]; }
  }
  out->n_containers = n;
  out->n_bitmap = nb; out->n_array = na; out->n_run = nr;
  out->array_pool_bytes = (uint32_t)(arr_elems * 2u);
  out->run_pool_bytes = (uint32_t)(run_pairs * 4u);
  if (n == 0) { free(ty); free(card); free(runs); return; }
  out->max_key = max_key_of(U);
  out->keys = (uint16_t*)malloc(2u * n);
  out->types = (uint8_t*)malloc(n);
  out->offsets = (uint32_t*)malloc(4u * n);
  out->cards = (uint16_t*)malloc(2u * n);
  out->key_index = (uint16_t*)malloc(2u * (out->max_key + 1u));
  memset(out->key_index, 0xFF, 2u * (out->max_key + 1u));
  out->bitmap = (uint64_t*)calloc((size_t)nb * CHUNK_WORDS + 1, 8);
  out->array = (uint16_t*)calloc(arr_elems + 1, 2);
  out->run = (uint16_t*)calloc(run_pairs * 2 + 1, 2);
  uint32_t ci = 0, sb = 0;
  uint64_t ae = 0, rp = 0;
  for (uint32_t i = 0; i < cl->n; ++i) {
    if (ty[i] == 0xFF) continue;
    const uint64_t* w = cl->words + (size_t)i * CHUNK_WORDS;
    out->keys[ci] = cl->keys[i];
    out->types[ci] = ty[i];
    if (cl->keys[i] <= out->max_key) out->key_index[cl->keys[i]] = (uint16_t)ci;
    if (ty[i] == T_BITMAP) {
      out->offsets[ci] = sb * 8192u;
      out->cards[ci] = (uint16_t)(card[i] & 0xFFFFu); /* 65536 -> 0 */
      memcpy(out->bitmap + (size_t)sb * CHUNK_WORDS, w, 8192);
      ++sb;
    } else if (ty[i] == T_ARRAY) {
      out->offsets[ci] = (uint32_t)(ae * 2u);
      out->cards[ci] = (uint16_t)card[i];
      for (uint32_t j = 0; j < CHUNK_WORDS; ++j) {
        uint64_t x = w[j];
        while (x) {
          out->array[ae++] = (uint16_t)(j * 64u + (uint32_t)__builtin_ctzll(x));
          x &= x - 1;
        }
      }
    } else {
      out->offsets[ci] = (uint32_t)(rp * 4u);
      out->cards[ci] = (uint16_t)runs[i];
      uint32_t b = 0;
      while (b < 65536u) {
        if ((w[b >> 6] >> (b & 63)) & 1u) {
          uint32_t s = b;
          while (b < 65536u && ((w[b >> 6] >> (b & 63)) & 1u)) ++b;
          out->run[2 * rp] = (uint16_t)s;
          out->run[2 * rp + 1] = (uint16_t)(b - 1 - s);
          ++rp;
        } else {
          ++b;
        }
      }
    }
    ++ci;
  }
  free(ty); free(card); free(runs);
}

/* Materialises container `i` of an image into 1024 words (physical set). */
static void container_words(const or_image* im, uint32_t i, uint64_t* w)
{
  memset(w, 0, 8192);
  uint32_t off = im->offsets[i];
  uint32_t c = im->cards[i];
  if (im->types[i] == T_BITMAP) {
    memcpy(w, im->bitmap + off / 8u, 8192);
  } else if (im->types[i] == T_ARRAY) {
    const uint16_t* a = im->array + off / 2u;
    for (uint32_t j = 0; j < c; ++j) w[a[j] >> 6] |= 1ull << (a[j] & 63);
  } else {
    const uint16_t* r = im->run + off / 2u;
    for (uint32_t j = 0; j < c; ++j) {
      uint32_t s = r[2 * j], e = s + r[2 * j + 1];
      for (uint32_t b = s; b <= e && b < 65536u; ++b) w[b >> 6] |= 1ull << (b & 63);
    }
  }
}

static int find_key(const or_image* im, uint32_t key)
{
  uint32_t lo = 0, hi = im->n_containers;
  while (lo < hi) {
    uint32_t mid = (lo + hi) / 2;
    if (im->keys[mid] < key) lo = mid + 1; else hi = mid;
  }
  return (lo < im->n_containers && im->keys[lo] == key) ? (int)lo : -1;
}

/* ---------------------------------------------------------------- uploads */

/* Resolves PROMOTE_AUTO for a build with `n_nonempty` stored containers,
 * including the compression guard of reference src/upload.cpp:102-118
 * (promotion is dropped when n*8 KiB*2 >= ceil(U/8)). */
static uint32_t resolve_threshold(uint32_t thr, uint32_t U, uint32_t n_nonempty, uint64_t l2)
{
  if (thr != PROMOTE_AUTO) return thr;
  uint32_t t = or_resolve_auto_threshold(U, l2);
  if (t < PROMOTE_KEEP_DEFAULT) {
    uint64_t promoted = (uint64_t)n_nonempty * 8192u;
    uint64_t flat = ((uint64_t)U + 7u) / 8u;
    if (promoted * 2u >= flat) t = PROMOTE_KEEP_DEFAULT;
  }
  return t;
}

/* Builds from a flat logical bitset of n_chunks*1024 u64 words (modified in
 * place). Complement rule: stored set = complement within [0,U) iff the
 * cardinality is > U/2 (strict; reference src/upload_ids.cu:359,437,837). */
static void from_flat(uint64_t* flat, uint32_t n_chunks, uint32_t U, uint32_t thr, uint64_t l2,
                      or_image* out)
{
  uint64_t total = 0;
  for (uint32_t c = 0; c < n_chunks; ++c) {
    mask_valid(flat + (size_t)c * CHUNK_WORDS, chunk_valid_bits(c, U));
    total += chunk_popcount(flat + (size_t)c * CHUNK_WORDS);
  }
  int neg = total > (uint64_t)(U / 2u);
  chunk_list cl = {0, NULL, NULL};
  cl.keys = (uint16_t*)malloc(2u * (n_chunks + 1));
  cl.words = (uint64_t*)malloc((size_t)(n_chunks + 1) * 8192u);
  for (uint32_t c = 0; c < n_chunks; ++c) {
    uint64_t* w = flat + (size_t)c * CHUNK_WORDS;
    if (neg) {
      for (uint32_t i = 0; i < CHUNK_WORDS; ++i) w[i] = ~w[i];
      mask_valid(w, chunk_valid_bits(c, U));
    }
    if (chunk_popcount(w) == 0) continue;
    cl.keys[cl.n] = (uint16_t)c;
    memcpy(cl.words + (size_t)cl.n * CHUNK_WORDS, w, 8192);
    ++cl.n;
  }
  uint32_t t = resolve_threshold(thr, U, cl.n, l2);
  assemble(&cl, NULL, t, U, neg, total, out);
  chunk_list_free(&cl);
}

static uint32_t n_chunks_of(uint32_t U) { return (uint32_t)(((uint64_t)U + 65535u) >> 16); }

/* upload_from_ids (reference src/upload_ids.cu:567-591): unsorted, duplicates
 * ignored. IDs >= U are an error here (-4); the reference does not check. */
int or_from_ids(const uint32_t* ids, uint64_t n, uint32_t U, uint32_t thr, uint64_t l2,
                or_image* out)
{
  memset(out, 0, sizeof(*out));
  out->universe_size = U;
  for (uint64_t i = 0; i < n; ++i)
    if (ids[i] >= U) return -4;
  if (n == 0 || U == 0) return 0;
  uint32_t nc = n_chunks_of(U);
  uint64_t* flat = (uint64_t*)calloc((size_t)nc * CHUNK_WORDS, 8);
  for (uint64_t i = 0; i < n; ++i) flat[ids[i] >> 6] |= 1ull << (ids[i] & 63);
  from_flat(flat, nc, U, thr, l2, out);
  free(flat);
  return 0;
}

/* upload_from_bitset (reference src/upload_ids.cu:806-893); bits >= U are
 * ignored, missing words (n_words < ceil(U/32)) read as zero. */
int or_from_bitset(const uint32_t* words, uint64_t n_words, uint32_t U, uint32_t thr,
                   uint64_t l2, or_image* out)
{
  memset(out, 0, sizeof(*out));
  out->universe_size = U;
  if (n_words == 0 || U == 0) return 0;
  uint32_t nc = n_chunks_of(U);
  uint64_t* flat = (uint64_t*)calloc((size_t)nc * CHUNK_WORDS, 8);
  uint64_t lim = (uint64_t)nc * 2048u;
  for (uint64_t i = 0; i < n_words && i < lim; ++i)
    flat[i >> 1] |= (uint64_t)words[i] << (32 * (i & 1));
  from_flat(flat, nc, U, thr, l2, out);
  free(flat);
  return 0;
}

/* ----------------------------------------------------------- set algebra */

enum { MODE_AND_SUB = 0, MODE_OR = 1, MODE_XOR = 2 };

/* The engine's k-way combine. MODE_AND_SUB: result = AND(P) \ OR(N) over the
 * keys common to every P operand. MODE_OR / MODE_XOR: combine every operand
 * (all in P) over the union of keys. Output typing is structural:
 *   a key held by exactly one contributing operand (AND_SUB with |P| = 1 and
 *   no N operand holding the key; OR/XOR with one holder) is copied through
 *   with its type; AND_SUB with an ARRAY among the P containers -> ARRAY;
 *   OR/XOR whose holders are all ARRAYs with summed cardinality <= 4096 ->
 *   ARRAY; everything else -> BITMAP. Empty results are dropped (reference
 *   src/set_ops.cu:1111-1145). */
static void kway(const or_image* const* P, uint32_t np, const or_image* const* N, uint32_t nn,
                 int mode, int negated, uint32_t U, or_image* out)
{
  chunk_list cl = {0, NULL, NULL};
  cl.keys = (uint16_t*)malloc(2u * 65536u);
  uint8_t* ty = (uint8_t*)malloc(65536u);
  size_t cap = 64;
  cl.words = (uint64_t*)malloc(cap * 8192u);
  uint64_t tmp[CHUNK_WORDS];
  for (uint32_t key = 0; key < 65536u; ++key) {
    int holders = 0, any_array = 0, all_array = 1, missing = 0;
    uint32_t sum_card = 0;
    int first_i = -1;
    const or_image* first_im = NULL;
    for (uint32_t j = 0; j < np; ++j) {
      int i = find_key(P[j], key);
      if (i < 0) { missing = 1; continue; }
      ++holders;
      if (!first_im) { first_im = P[j]; first_i = i; }
      if (P[j]->types[i] == T_ARRAY) { any_array = 1; sum_card += P[j]->cards[i]; }
      else all_array = 0;
    }
    if (mode == MODE_AND_SUB && (missing || holders == 0)) continue;
    if (holders == 0) continue;
    int n_holders_n = 0;
    for (uint32_t j = 0; j < nn; ++j) n_holders_n += find_key(N[j], key) >= 0;
    if (cl.n == cap) { cap *= 2; cl.words = (uint64_t*)realloc(cl.words, cap * 8192u); }
    uint64_t* acc = cl.words + (size_t)cl.n * CHUNK_WORDS;
    uint8_t t;
    if (holders == 1 && n_holders_n == 0) {
      container_words(first_im, (uint32_t)first_i, acc);
      t = first_im->types[first_i];
    } else if (mode == MODE_AND_SUB) {
      for (uint32_t w = 0; w < CHUNK_WORDS; ++w) acc[w] = ~0ull;
      for (uint32_t j = 0; j < np; ++j) {
        container_words(P[j], (uint32_t)find_key(P[j], key), tmp);
        for (uint32_t w = 0; w < CHUNK_WORDS; ++w) acc[w] &= tmp[w];
      }
      for (uint32_t j = 0; j < nn; ++j) {
        int i = find_key(N[j], key);
        if (i < 0) continue;
        container_words(N[j], (uint32_t)i, tmp);
        for (uint32_t w = 0; w < CHUNK_WORDS; ++w) acc[w] &= ~tmp[w];
      }
      t = any_array ? T_ARRAY : T_BITMAP;
    } else {
      memset(acc, 0, 8192);
      for (uint32_t j = 0; j < np; ++j) {
        int i = find_key(P[j], key);
        if (i < 0) continue;
        container_words(P[j], (uint32_t)i, tmp);
        for (uint32_t w = 0; w < CHUNK_WORDS; ++w)
          acc[w] = (mode == MODE_OR) ? (acc[w] | tmp[w]) : (acc[w] ^ tmp[w]);
      }
      t = (all_array && sum_card <= PROMOTE_KEEP_DEFAULT) ? T_ARRAY : T_BITMAP;
    }
    cl.keys[cl.n] = (uint16_t)key;
    ty[cl.n] = t;
    ++cl.n;
  }
  uint64_t stored = 0;
  for (uint32_t i = 0; i < cl.n; ++i) stored += chunk_popcount(cl.words + (size_t)i * CHUNK_WORDS);
  assemble(&cl, ty, 0, U, negated, negated ? (uint64_t)U - stored : stored, out);
  free(ty);
  chunk_list_free(&cl);
}

/* set_operation with the DeMorgan rewrite of negated operands
 * (reference src/set_ops.cu:512-565); result universe = max(Ua, Ub)
 * (reference src/set_ops.cu:1164). */
int or_set_operation(const or_image* a, const or_image* b, int op, or_image* out)
{
  if (op < 0 || op > 3) return -1;
  int na = a->negated != 0, nb = b->negated != 0, neg = 0;
  const or_image* x = a;
  const or_image* y = b;
  const or_image* tmp;
  if (na || nb) {
    switch (op) {
      case 0:
        if (na && !nb) { op = 2; tmp = x; x = y; y = tmp; }
        else if (!na && nb) { op = 2; }
        else { op = 1; neg = 1; }
        break;
      case 1:
        if (na && !nb) { op = 2; neg = 1; }
        else if (!na && nb) { op = 2; tmp = x; x = y; y = tmp; neg = 1; }
        else { op = 0; neg = 1; }
        break;
      case 2:
        if (na && !nb) { op = 1; neg = 1; }
        else if (!na && nb) { op = 0; }
        else { op = 2; tmp = x; x = y; y = tmp; }
        break;
      default:
        neg = (na != nb);
        break;
    }
  }
  uint32_t U = a->universe_size > b->universe_size ? a->universe_size : b->universe_size;
  const or_image* pp[2] = {x, y};
  if (op == 0) kway(pp, 2, NULL, 0, MODE_AND_SUB, neg, U, out);
  else if (op == 2) kway(pp, 1, pp + 1, 1, MODE_AND_SUB, neg, U, out);
  else kway(pp, 2, NULL, 0, op == 1 ? MODE_OR : MODE_XOR, neg, U, out);
  return 0;
}

/* multi_and (reference src/set_ops.cu:1715-1745, fused negation handling
 * :1489-1710): AND of the non-negated inputs minus the stored sets of the
 * negated ones; with no non-negated input the result is the complement of
 * the OR of the stored sets (stored negated). */
/* More than OR_MAX_PASS inputs: the engine combines the first 64 in one
 * k-way pass, then the running result with the next 63 per pass (its
 * structural output typing then applies per pass); this restates that. */
#define OR_MAX_PASS 64u
static int multi_chained(const or_image* const* ims, uint32_t count, or_image* out,
                         int (*one)(const or_image* const*, uint32_t, or_image*))
{
  or_image acc;
  one(ims, OR_MAX_PASS, &acc);
  const or_image* grp[OR_MAX_PASS];
  for (uint32_t i = OR_MAX_PASS; i < count;) {
    uint32_t n = count - i < OR_MAX_PASS - 1 ? count - i : OR_MAX_PASS - 1;
    grp[0] = &acc;
    for (uint32_t j = 0; j < n; ++j) grp[1 + j] = ims[i + j];
    or_image next;
    one(grp, n + 1, &next);
    or_image_free(&acc);
    acc = next;
    i += n;
  }
  *out = acc;
  return 0;
}

int or_multi_and(const or_image* const* ims, uint32_t count, or_image* out)
{
  memset(out, 0, sizeof(*out));
  if (count == 0) return 0;
  if (count > OR_MAX_PASS) return multi_chained(ims, count, out, or_multi_and);
  const or_image** P = (const or_image**)malloc(sizeof(void*) * count);
  const or_image** N = (const or_image**)malloc(sizeof(void*) * count);
  uint32_t np = 0, nn = 0, U = 0;
  for (uint32_t i = 0; i < count; ++i) {
    if (ims[i]->universe_size > U) U = ims[i]->universe_size;
    if (ims[i]->negated) N[nn++] = ims[i]; else P[np++] = ims[i];
  }
  if (np > 0) kway(P, np, N, nn, MODE_AND_SUB, 0, U, out);
  else kway(N, nn, NULL, 0, MODE_OR, 1, U, out);
  free(P); free(N);
  return 0;
}

/* multi_or (reference src/set_ops.cu:1747-1762) as ~multi_and(~inputs). */
int or_multi_or(const or_image* const* ims, uint32_t count, or_image* out)
{
  memset(out, 0, sizeof(*out));
  if (count == 0) return 0;
  if (count > OR_MAX_PASS) return multi_chained(ims, count, out, or_multi_or);
  const or_image** P = (const or_image**)malloc(sizeof(void*) * count);
  const or_image** N = (const or_image**)malloc(sizeof(void*) * count);
  uint32_t np = 0, nn = 0, U = 0;
  for (uint32_t i = 0; i < count; ++i) {
    if (ims[i]->universe_size > U) U = ims[i]->universe_size;
    if (ims[i]->negated) P[np++] = ims[i]; else N[nn++] = ims[i];
  }
  if (np > 0) kway(P, np, N, nn, MODE_AND_SUB, 1, U, out);
  else kway(N, nn, NULL, 0, MODE_OR, 0, U, out);
  free(P); free(N);
  return 0;
}

/* promote_to_bitmap (reference src/promote.cu:242-328): every container
 * becomes a BITMAP; cardinality fields become popcounts; universe and
 * negation are kept (the reference drops them for an empty input). */
int or_promote_to_bitmap(const or_image* in, or_image* out)
{
  chunk_list cl = {0, NULL, NULL};
  cl.n = in->n_containers;
  cl.keys = (uint16_t*)malloc(2u * (cl.n + 1));
  cl.words = (uint64_t*)malloc((size_t)(cl.n + 1) * 8192u);
  uint8_t* ty = (uint8_t*)malloc(cl.n + 1);
  for (uint32_t i = 0; i < cl.n; ++i) {
    cl.keys[i] = in->keys[i];
    container_words(in, i, cl.words + (size_t)i * CHUNK_WORDS);
    ty[i] = T_BITMAP;
  }
  assemble(&cl, ty, 0, in->universe_size, in->negated, in->total_cardinality, out);
  free(ty);
  chunk_list_free(&cl);
  return 0;
}

/* -------------------------------------------------------- point queries */

/* GpuRoaringView::contains (reference include/cu_roaring/device/
 * roaring_view.cuh:39-157): container lookup, type dispatch, run test
 * low <= start + len, result XOR negated. */
static int contains_one(const or_image* im, uint32_t id)
{
  uint32_t key = id >> 16, low = id & 0xFFFFu;
  int i = find_key(im, key);
  int hit = 0;
  if (i >= 0) {
    uint32_t off = im->offsets[i], c = im->cards[i];
    if (im->types[i] == T_BITMAP) {
      hit = (int)((im->bitmap[off / 8u + (low >> 6)] >> (low & 63)) & 1u);
    } else if (im->types[i] == T_ARRAY) {
      const uint16_t* a = im->array + off / 2u;
      uint32_t lo = 0, hi = c;
      while (lo < hi) { uint32_t m = (lo + hi) / 2; if (a[m] < low) lo = m + 1; else hi = m; }
      hit = lo < c && a[lo] == low;
    } else {
      const uint16_t* r = im->run + off / 2u;
      for (uint32_t j = 0; j < c && !hit; ++j)
        hit = low >= r[2 * j] && low <= (uint32_t)r[2 * j] + r[2 * j + 1];
    }
  }
  return hit != (im->negated != 0);
}

typedef struct contains_job {
  const or_image* im;
  const uint32_t* ids;
  uint64_t lo, hi; /* in 32-id words */
  uint64_t n;
  uint32_t* out;
} contains_job;

static void* contains_worker(void* p)
{
  contains_job* j = (contains_job*)p;
  for (uint64_t w = j->lo; w < j->hi; ++w) {
    uint32_t bits = 0;
    for (uint32_t b = 0; b < 32u; ++b) {
      uint64_t i = w * 32u + b;
      if (i < j->n && contains_one(j->im, j->ids[i])) bits |= 1u << b;
    }
    j->out[w] = bits;
  }
  return NULL;
}

void or_contains_batch(const or_image* im, const uint32_t* ids, uint64_t n, uint32_t* out_bits,
                       int n_threads)
{
  uint64_t words = (n + 31u) / 32u;
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  pthread_t th[256];
  contains_job jobs[256];
  for (int t = 0; t < n_threads; ++t) {
    jobs[t].im = im; jobs[t].ids = ids; jobs[t].n = n; jobs[t].out = out_bits;
    jobs[t].lo = words * (uint64_t)t / (uint64_t)n_threads;
    jobs[t].hi = words * (uint64_t)(t + 1) / (uint64_t)n_threads;
    pthread_create(&th[t], NULL, contains_worker, &jobs[t]);
  }
  for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* decompress_to_bitset (reference src/decompress.cu:104-162): logical set as
 * u32 words; negation inverts only [0, U); words past ceil(U/32) are zero. */
void or_decompress(const or_image* im, uint32_t* out, uint64_t n_words)
{
  memset(out, 0, n_words * 4u);
  uint64_t w64[CHUNK_WORDS];
  for (uint32_t i = 0; i < im->n_containers; ++i) {
    container_words(im, i, w64);
    uint64_t base = (uint64_t)im->keys[i] * 2048u;
    for (uint32_t j = 0; j < 2048u && base + j < n_words; ++j)
      out[base + j] = (uint32_t)(w64[j >> 1] >> (32 * (j & 1)));
  }
  if (im->negated) {
    uint64_t U = im->universe_size;
    for (uint64_t j = 0; j < n_words && j * 32u < U; ++j) {
      uint64_t valid = U - j * 32u;
      uint32_t m = valid >= 32u ? 0xFFFFFFFFu : ((1u << valid) - 1u);
      out[j] = ~out[j] & m;
    }
  }
}

/* enumerate_ids (reference src/to_csr.cu:161-220) as the sorted LOGICAL set
 * (the reference ignores `negated`; this engine honours it). */
uint64_t or_enumerate(const or_image* im, uint32_t* out)
{
  uint64_t n = 0;
  uint64_t w64[CHUNK_WORDS];
  uint32_t U = im->universe_size;
  uint32_t nchunks = (uint32_t)(((uint64_t)U + 65535u) >> 16);
  uint32_t ci = 0;
  for (uint32_t key = 0; key < 65536u; ++key) {
    int present = ci < im->n_containers && im->keys[ci] == key;
    if (!im->negated && !present) {
      if (ci >= im->n_containers) break;
      continue;
    }
    if (im->negated && key >= nchunks) break;
    if (present) container_words(im, ci++, w64);
    else memset(w64, 0, sizeof(w64));
    if (im->negated) {
      for (uint32_t j = 0; j < CHUNK_WORDS; ++j) w64[j] = ~w64[j];
      mask_valid(w64, chunk_valid_bits(key, U));
    }
    for (uint32_t j = 0; j < CHUNK_WORDS; ++j) {
      uint64_t x = w64[j];
      while (x) {
        uint32_t b = (uint32_t)__builtin_ctzll(x);
        x &= x - 1;
        if (out) out[n] = ((uint32_t)key << 16) | (j * 64u + b);
        ++n;
      }
    }
  }
  return n;
}

/* Structural checks of the packed layout: keys strictly increasing, offsets
 * in range and consistent with the type sizes, key_index consistent,
 * cardinality fields matching payloads, counts matching types. */
int or_validate(const or_image* im)
{
  uint32_t nb = 0, na = 0, nr = 0;
  uint64_t stored = 0;
  uint64_t w64[CHUNK_WORDS];
  for (uint32_t i = 0; i < im->n_containers; ++i) {
    if (i && im->keys[i] <= im->keys[i - 1]) return -1;
    if (im->keys[i] > im->max_key) return -2;
    if (im->key_index[im->keys[i]] != i) return -3;
    uint32_t off = im->offsets[i], c = im->cards[i];
    if (im->types[i] == T_BITMAP) {
      if (off % 8192u || off / 8192u >= im->n_bitmap) return -4;
      ++nb;
    } else if (im->types[i] == T_ARRAY) {
      if (c == 0 || off % 2u || off + 2u * c > im->array_pool_bytes) return -5;
      const uint16_t* a = im->array + off / 2u;
      for (uint32_t j = 1; j < c; ++j) if (a[j] <= a[j - 1]) return -6;
      ++na;
    } else if (im->types[i] == T_RUN) {
      if (c == 0 || off % 4u || off + 4u * c > im->run_pool_bytes) return -7;
      ++nr;
    } else {
      return -8;
    }
    container_words(im, i, w64);
    uint32_t pc = chunk_popcount(w64);
    if (pc == 0) return -9;
    if (im->types[i] != T_RUN && (pc & 0xFFFFu) != c) return -10;
    stored += pc;
  }
  if (nb != im->n_bitmap || na != im->n_array || nr != im->n_run) return -11;
  uint64_t logical = im->negated ? (uint64_t)im->universe_size - stored : stored;
  if (logical != im->total_cardinality) return -12;
  if (im->n_containers && im->key_index) {
    uint32_t cnt = 0;
    for (uint32_t k = 0; k <= im->max_key; ++k) cnt += im->key_index[k] != 0xFFFFu;
    if (cnt != im->n_containers) return -13;
  }
  return 0;
}

/* ------------------------------------------------------ filtered top-k */

/* IEEE binary16 -> binary32 from the bit pattern. */
static float half_to_float(uint16_t h)
{
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
  if (e == 0) {
    if (m == 0) bits = s;
    else {
      int sh = 0;
      while (!(m & 0x400u)) { m <<= 1; ++sh; }
      m &= 0x3FFu;
      bits = s | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = s | 0x7F800000u | (m << 13);
  } else {
    bits = s | ((e - 15u + 127u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

typedef struct topk_job {
  const float* dbf; /* fp32 copy of the database */
  const float* norms;
  const uint16_t* queries;
  const uint32_t* pass;
  uint64_t n_rows;
  uint32_t dim, k, q0, q1;
  int metric;
  float* out_dist;
  int64_t* out_ids;
} topk_job;

/* Is (d1, i1) strictly better than (d2, i2)? Ties -> smaller id. */
static int better(int metric, float d1, int64_t i1, float d2, int64_t i2)
{
  if (d1 != d2) return metric == 0 ? d1 > d2 : d1 < d2;
  return i1 < i2;
}

static void* topk_worker(void* p)
{
  topk_job* j = (topk_job*)p;
  float* q = (float*)malloc(sizeof(float) * j->dim);
  for (uint32_t qi = j->q0; qi < j->q1; ++qi) {
    float qn = 0.f;
    for (uint32_t d = 0; d < j->dim; ++d) {
      q[d] = half_to_float(j->queries[(size_t)qi * j->dim + d]);
      qn += q[d] * q[d];
    }
    float* bd = j->out_dist + (size_t)qi * j->k;
    int64_t* bi = j->out_ids + (size_t)qi * j->k;
    uint32_t cnt = 0;
    for (uint64_t r = 0; r < j->n_rows; ++r) {
      if (j->pass && !((j->pass[r >> 5] >> (r & 31)) & 1u)) continue;
      const float* x = j->dbf + r * j->dim;
      float dot = 0.f;
      for (uint32_t d = 0; d < j->dim; ++d) dot += q[d] * x[d];
      float s = j->metric == 0 ? dot : (j->norms[r] - 2.f * dot + qn);
      if (cnt == j->k && !better(j->metric, s, (int64_t)r, bd[cnt - 1], bi[cnt - 1])) continue;
      uint32_t pos = cnt < j->k ? cnt++ : j->k - 1;
      while (pos > 0 && better(j->metric, s, (int64_t)r, bd[pos - 1], bi[pos - 1])) {
        bd[pos] = bd[pos - 1];
        bi[pos] = bi[pos - 1];
        --pos;
      }
      bd[pos] = s;
      bi[pos] = (int64_t)r;
    }
    for (uint32_t c = cnt; c < j->k; ++c) {
      bd[c] = j->metric == 0 ? -INFINITY : INFINITY;
      bi[c] = -1;
    }
  }
  free(q);
  return NULL;
}

/* Exact fp32 brute force: fp16 inputs widened, IP = sum q_d x_d, L2 =
 * |x|^2 - 2 q.x + |q|^2, the filter applied before selection, ties broken
 * by the smaller row id. */
void or_widen_f16(const uint16_t* src, uint64_t n, float* dst)
{
  for (uint64_t i = 0; i < n; ++i) dst[i] = half_to_float(src[i]);
}

void or_row_norms_f32(const float* dbf, uint64_t n_rows, uint32_t dim, float* norms)
{
  for (uint64_t r = 0; r < n_rows; ++r) {
    float s = 0.f;
    for (uint32_t d = 0; d < dim; ++d) s += dbf[r * dim + d] * dbf[r * dim + d];
    norms[r] = s;
  }
}

void or_topk(const uint16_t* db, uint64_t n_rows, uint32_t dim, const uint16_t* queries,
             uint32_t n_queries, const uint32_t* pass_bits, uint32_t k, int metric,
             float* out_dist, int64_t* out_ids, int n_threads)
{
  float* dbf = (float*)malloc(sizeof(float) * n_rows * dim);
  float* norms = (float*)malloc(sizeof(float) * (n_rows + 1));
  or_widen_f16(db, n_rows * dim, dbf);
  or_row_norms_f32(dbf, n_rows, dim, norms);
  or_topk_f32(dbf, norms, n_rows, dim, queries, n_queries, pass_bits, k, metric, out_dist, out_ids,
              n_threads);
  free(dbf);
  free(norms);
}

void or_topk_f32(const float* dbf, const float* norms, uint64_t n_rows, uint32_t dim,
                 const uint16_t* queries, uint32_t n_queries, const uint32_t* pass_bits, uint32_t k,
                 int metric, float* out_dist, int64_t* out_ids, int n_threads)
{
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  pthread_t th[256];
  topk_job jobs[256];
  for (int t = 0; t < n_threads; ++t) {
    topk_job* j = &jobs[t];
    j->dbf = dbf; j->norms = norms; j->queries = queries; j->pass = pass_bits;
    j->n_rows = n_rows; j->dim = dim; j->k = k; j->metric = metric;
    j->out_dist = out_dist; j->out_ids = out_ids;
    j->q0 = (uint32_t)((uint64_t)n_queries * t / n_threads);
    j->q1 = (uint32_t)((uint64_t)n_queries * (t + 1) / n_threads);
    pthread_create(&th[t], NULL, topk_worker, j);
  }
  for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}


/* ---- portable serialization (published RoaringFormatSpec) ---------------- */

static void put16(uint8_t* p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static void put32(uint8_t* p, uint32_t v) { put16(p, v & 0xFFFFu); put16(p + 2, v >> 16); }

uint64_t or_serialize_portable(const uint32_t* ids, uint64_t n, int allow_runs, uint8_t* out, uint64_t cap)
{
  /* Containers: [begin, end) ranges of ids with one high half. */
  uint64_t n_cont = 0;
  for (uint64_t i = 0; i < n; ++i)
    if (i == 0 || (ids[i] >> 16) != (ids[i - 1] >> 16)) ++n_cont;
  uint64_t* begin = (uint64_t*)malloc(sizeof(uint64_t) * (n_cont + 1));
  uint32_t* runs = (uint32_t*)malloc(sizeof(uint32_t) * (n_cont + 1));
  uint8_t* kind = (uint8_t*)malloc(n_cont + 1); /* 0 array, 1 bitmap, 2 run */
  uint64_t c = 0;
  for (uint64_t i = 0; i < n; ++i)
    if (i == 0 || (ids[i] >> 16) != (ids[i - 1] >> 16)) begin[c++] = i;
  begin[n_cont] = n;
  int any_run = 0;
  for (c = 0; c < n_cont; ++c) {
    const uint64_t b = begin[c], e = begin[c + 1], card = e - b;
    uint32_t r = 0;
    for (uint64_t i = b; i < e; ++i)
      if (i == b || ids[i] != ids[i - 1] + 1) ++r;
    runs[c] = r;
    const uint64_t plain = card <= 4096 ? 2 * card : 8192;
    kind[c] = (allow_runs && 2 + 4 * (uint64_t)r < plain) ? 2 : (card <= 4096 ? 0 : 1);
    if (kind[c] == 2) any_run = 1;
  }
  const int offsets = !any_run || n_cont >= 4;
  uint64_t head = any_run ? 4 + (n_cont + 7) / 8 : 8;
  head += 4 * n_cont + (offsets ? 4 * n_cont : 0);
  uint64_t total = head;
  for (c = 0; c < n_cont; ++c) {
    const uint64_t card = begin[c + 1] - begin[c];
    total += kind[c] == 2 ? 2 + 4 * (uint64_t)runs[c] : (kind[c] == 0 ? 2 * card : 8192);
  }
  if (out && cap >= total) {
    memset(out, 0, total);
    uint64_t pos;
    if (any_run) {
      put32(out, 12347u | ((uint32_t)(n_cont - 1) << 16));
      for (c = 0; c < n_cont; ++c)
        if (kind[c] == 2) out[4 + c / 8] |= (uint8_t)(1u << (c % 8));
      pos = 4 + (n_cont + 7) / 8;
    } else {
      put32(out, 12346u);
      put32(out + 4, (uint32_t)n_cont);
      pos = 8;
    }
    for (c = 0; c < n_cont; ++c) {
      put16(out + pos + 4 * c, ids[begin[c]] >> 16);
      put16(out + pos + 4 * c + 2, (uint32_t)(begin[c + 1] - begin[c] - 1));
    }
    pos += 4 * n_cont;
    const uint64_t offs = pos;
    if (offsets) pos += 4 * n_cont;
    for (c = 0; c < n_cont; ++c) {
      const uint64_t b = begin[c], e = begin[c + 1];
      if (offsets) put32(out + offs + 4 * c, (uint32_t)pos);
      if (kind[c] == 0) {
        for (uint64_t i = b; i < e; ++i, pos += 2) put16(out + pos, ids[i] & 0xFFFFu);
      } else if (kind[c] == 1) {
        for (uint64_t i = b; i < e; ++i) {
          const uint32_t lo = ids[i] & 0xFFFFu;
          out[pos + lo / 8] |= (uint8_t)(1u << (lo % 8)); /* little-endian words: bit lo at byte lo/8 */
        }
        pos += 8192;
      } else {
        put16(out + pos, runs[c]);
        pos += 2;
        for (uint64_t i = b; i < e;) {
          uint64_t j = i;
          while (j + 1 < e && ids[j + 1] == ids[j] + 1) ++j;
          put16(out + pos, ids[i] & 0xFFFFu);
          put16(out + pos + 2, (uint32_t)(j - i));
          pos += 4;
          i = j + 1;
        }
      }
    }
  }
  free(begin);
  free(runs);
  free(kind);
  return total;
}
