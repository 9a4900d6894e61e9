/*
 * c_abi_consumer.c — a plain C99 user of include/headshot_cuda.h, the way a
 * foreign-language binding (bindgen for the Rust engine, cgo, ctypes) sees
 * the library.
 *
 * Built with -std=c99 -pedantic -Wall -Wextra -Werror and run by
 * tests/test_c_consumer.py on a machine without a GPU.  It
 *   - takes the address of every entry point the header declares, so each
 *     one must resolve when the program is linked against the library;
 *   - checks the host-side calls (ABI version, RoPE periods and tables, the
 *     ring's shard rule and step plan) and the error contract: argument
 *     errors come back as status codes with a message from hs_last_error(),
 *     never as an abort;
 *   - with argv[2] == "nogpu", checks that creating a context fails cleanly;
 *   - writes the 37 x 37 RoPE tables (sin then cos, f32) to the file named
 *     by argv[1], for the test to compare with the oracle bit for bit.
 * Exit status 0 when every check passed.
 */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "headshot_cuda.h"

typedef void (*any_fn)(void);
#define FN(f) ((any_fn)(f))

/* One entry per function in the header (tests/test_c_consumer.py checks the list is complete). */
static const any_fn entry_points[] = {
    FN(hs_abi_version),           FN(hs_last_error),
    FN(hs_ctx_create),            FN(hs_ctx_destroy),
    FN(hs_ctx_set_stream),        FN(hs_ctx_use_own_stream),
    FN(hs_ctx_stream),            FN(hs_ctx_set_wait_timeout_ms),
    FN(hs_ctx_request_cancel),    FN(hs_ctx_clear_cancel),
    FN(hs_prof_enable),           FN(hs_prof_reset),
    FN(hs_prof_read),             FN(hs_alloc),
    FN(hs_free),                  FN(hs_memset),
    FN(hs_memcpy_h2d),            FN(hs_memcpy_d2h),
    FN(hs_sync),                  FN(hs_attention),
    FN(hs_attention_fused),       FN(hs_attention_block_fused),
    FN(hs_attention_fused_noalloc), FN(hs_linear),
    FN(hs_layernorm),             FN(hs_rope_apply),
    FN(hs_split_heads),           FN(hs_attn_merge),
    FN(hs_ring_shard),            FN(hs_ring_plan),
    FN(hs_ring_id_bytes),         FN(hs_ring_unique_id),
    FN(hs_ring_create),           FN(hs_ring_destroy),
    FN(hs_ring_attention_fused),  FN(hs_ring_attention_block_fused),
    FN(hs_ring_sync),             FN(hs_ring_set_reserved_sms),
    FN(hs_ring_ulysses_attention_fused),
    FN(hs_copy_row_blocks),
    FN(hs_im2col_patch),          FN(hs_cache_build),
    FN(hs_rope_periods),          FN(hs_rope_tables),
};

static int failures = 0;

#define CHECK(cond)                                                         \
  do {                                                                      \
    if (!(cond)) {                                                          \
      fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);       \
      ++failures;                                                           \
    }                                                                       \
  } while (0)

/* A failed call must leave a non-empty message. */
static int has_message(void) {
  const char* m = hs_last_error();
  return m != NULL && m[0] != '\0';
}

static void check_error_contract(void) {
  float tab[64];
  uint32_t start = 0, len = 0;
  void* p = NULL;
  CHECK(hs_attention(NULL, NULL, NULL, NULL, NULL, 1, 1, 16, 64, HS_BF16, 0.0f) == HS_ERR_INVALID);
  CHECK(has_message());
  CHECK(hs_attention_fused(NULL, NULL, NULL, NULL, NULL, 1, 1, 16, 64, HS_BF16, 0.0f, NULL, NULL, NULL, NULL,
                           1e-6f, NULL, NULL, 0, 0, 0) == HS_ERR_INVALID);
  CHECK(hs_linear(NULL, NULL, NULL, NULL, NULL, 8, 8, 8, HS_BF16, HS_LINEAR_PLAIN, NULL, NULL) == HS_ERR_INVALID);
  CHECK(hs_sync(NULL) == HS_ERR_INVALID);
  CHECK(hs_alloc(NULL, 16, &p) == HS_ERR_INVALID && p == NULL);
  CHECK(hs_ctx_set_stream(NULL, NULL) == HS_ERR_INVALID);
  CHECK(hs_ctx_stream(NULL) == NULL);
  CHECK(hs_ctx_destroy(NULL) == HS_OK); /* like free(NULL) */
  CHECK(hs_rope_periods(NULL) == HS_ERR_INVALID);
  CHECK(hs_rope_tables(NULL, 2, 2, NULL, tab) == HS_ERR_INVALID);
  CHECK(hs_ring_shard(10, 0, 0, &start, &len) == HS_ERR_INVALID);
  CHECK(hs_ring_shard(10, 4, 4, &start, &len) == HS_ERR_INVALID);
  CHECK(has_message());
}

static void check_rope(const char* path) {
  static float sn[37 * 37 * 64], cs[37 * 37 * 64];
  float per[16];
  FILE* f;
  int i;
  CHECK(hs_rope_periods(per) == HS_OK);
  /* rope.rs: periods()[i] = 100^(2i/32); periods()[8] == 10 */
  CHECK(fabsf(per[0] - 1.0f) < 1e-6f);
  CHECK(fabsf(per[8] - 10.0f) < 1e-5f);
  for (i = 1; i < 16; ++i) CHECK(per[i] > per[i - 1]);
  CHECK(hs_rope_tables(NULL, 37, 37, sn, cs) == HS_OK);
  for (i = 0; i < 37 * 37 * 64; ++i) CHECK(fabsf(sn[i] * sn[i] + cs[i] * cs[i] - 1.0f) < 1e-5f);
  f = fopen(path, "wb");
  CHECK(f != NULL);
  if (f) {
    CHECK(fwrite(sn, sizeof(float), 37 * 37 * 64, f) == 37 * 37 * 64);
    CHECK(fwrite(cs, sizeof(float), 37 * 37 * 64, f) == 37 * 37 * 64);
    fclose(f);
  }
}

/* Shards tile [0, n) in rank order and differ in length by at most one. */
static void check_ring_shards(void) {
  static const uint32_t ns[] = {1, 7, 1001, 43968, 274800};
  size_t a;
  int world, rank;
  for (a = 0; a < sizeof(ns) / sizeof(ns[0]); ++a) {
    for (world = 1; world <= 8; ++world) {
      uint32_t next = 0, lmin = 0xffffffffu, lmax = 0;
      if (ns[a] < (uint32_t)world) continue;
      for (rank = 0; rank < world; ++rank) {
        uint32_t start = 0, len = 0;
        CHECK(hs_ring_shard(ns[a], world, rank, &start, &len) == HS_OK);
        CHECK(start == next);
        next = start + len;
        if (len < lmin) lmin = len;
        if (len > lmax) lmax = len;
      }
      CHECK(next == ns[a]);
      CHECK(lmax - lmin <= 1);
    }
  }
}

/* Every rank attends to every block exactly once; what rank r sends at step s
 * is what rank send_to attends to at step s + 1; state is loaded on every step
 * but the first and stored on every step but the last. */
static void check_ring_plan(void) {
  int world, rank, step;
  for (world = 1; world <= 8; ++world) {
    for (rank = 0; rank < world; ++rank) {
      int seen[8] = {0};
      for (step = 0; step < world; ++step) {
        int src = -1, to = -1, from = -1, load = -1, store = -1;
        CHECK(hs_ring_plan(rank, world, step, &src, &to, &from, &load, &store) == HS_OK);
        CHECK(src >= 0 && src < world);
        if (src >= 0 && src < world) ++seen[src];
        CHECK(load == (step > 0));
        CHECK(store == (step < world - 1));
        if (step == 0) CHECK(src == rank);
        if (step + 1 < world) {
          int src2 = -1, to2, from2, load2, store2;
          CHECK(to >= 0 && to < world);
          CHECK(hs_ring_plan(to, world, step + 1, &src2, &to2, &from2, &load2, &store2) == HS_OK);
          CHECK(src2 == src);
        } else {
          CHECK(to == -1);
        }
      }
      for (step = 0; step < world; ++step) CHECK(seen[step] == 1);
    }
    {
      int src, to, from, load, store;
      CHECK(hs_ring_plan(0, world, world, &src, &to, &from, &load, &store) == HS_ERR_INVALID);
    }
  }
}

int main(int argc, char** argv) {
  size_t i;
  if (argc < 2) {
    fprintf(stderr, "usage: %s <rope table output file> [nogpu]\n", argv[0]);
    return 2;
  }
  for (i = 0; i < sizeof(entry_points) / sizeof(entry_points[0]); ++i) CHECK(entry_points[i] != NULL);
  CHECK(hs_abi_version() == HS_ABI_VERSION);
  CHECK(hs_last_error() != NULL);
  CHECK(hs_ring_id_bytes() >= 128);
  check_error_contract();
  check_rope(argv[1]);
  check_ring_shards();
  check_ring_plan();
  if (argc > 2 && strcmp(argv[2], "nogpu") == 0) {
    hs_ctx* ctx = NULL;
    CHECK(hs_ctx_create(0, &ctx) != HS_OK);
    CHECK(ctx == NULL);
    CHECK(has_message());
  }
  printf("entry points: %u, failures: %d\n", (unsigned)(sizeof(entry_points) / sizeof(entry_points[0])), failures);
  return failures == 0 ? 0 : 1;
}
