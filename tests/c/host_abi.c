/*
 * A C caller of libqmoe's host-only objects, compiled as C11 and as C++ with
 * warnings as errors: include/qmoe.h is usable from the reference's C port
 * (and from C++ hosts) and its host parts work without a GPU. Mirrors a few
 * cases of the reference's c/tests/test_cache.c and c/tests/test_safetensors.c
 * through the C ABI. Exit status 0 = every check passed.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qmoe.h"

static int failures = 0;
#define CHECK(c)                                                              \
    do {                                                                      \
        if (!(c)) {                                                           \
            fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #c); \
            failures++;                                                       \
        }                                                                     \
    } while (0)

static void cache_cases(void) {
    /* LRU victim choice and pin refusal, c/tests/test_cache.c:24-38, :69-90 */
    qmoe_cache *c = qmoe_cache_new(200, QMOE_POLICY_LRU, 0);
    uint64_t v = 0, ev[4];
    size_t nev = 0;
    CHECK(c != NULL);
    CHECK(qmoe_cache_put(c, 1, 11, 100, 0, 0, ev, 4, &nev) == 1);
    CHECK(qmoe_cache_put(c, 2, 22, 100, 0, 0, ev, 4, &nev) == 1);
    CHECK(qmoe_cache_get(c, 1, &v) == 1 && v == 11);
    CHECK(qmoe_cache_put(c, 3, 33, 100, 0, 0, ev, 4, &nev) == 1);
    CHECK(nev == 1 && ev[0] == 22); /* 2 was least recently used */
    CHECK(qmoe_cache_pin(c, 1) == 1 && qmoe_cache_pin(c, 3) == 1);
    CHECK(qmoe_cache_put(c, 4, 44, 100, 0, 0, ev, 4, &nev) == 0);
    qmoe_cache_stats s = qmoe_cache_stats_get(c);
    CHECK(s.rejected == 1 && s.pinned == 2 && s.size == 2);
    qmoe_cache_free(c);
}

static void predictor_cases(void) {
    /* tests/test_streaming.py:201-213 through the C ABI */
    qmoe_cache *c = qmoe_cache_new(4096, QMOE_POLICY_ADAPTIVE, 1);
    qmoe_predictor *p = qmoe_predictor_new(2, 4);
    const int32_t routed[5] = {1, 1, 1, 1, 2};
    int32_t sel[4];
    CHECK(qmoe_cache_put(c, (0ull << 32) | 1u, 7, 1, 0, 0, NULL, 0, NULL) == 1);
    CHECK(qmoe_predictor_record(p, c, 0, routed, 5, sel) == 2 && sel[0] == 1 && sel[1] == 2);
    CHECK(qmoe_predictor_routes(p) == 5 && qmoe_predictor_count(p, 0, 1) == 4);
    CHECK(qmoe_cache_stats_get(c).hot == 1);
    int32_t l[2], e[2];
    uint64_t n[2];
    CHECK(qmoe_predictor_frequent(p, 2, l, e, n) == 2 && l[0] == 0 && e[0] == 1 && n[0] == 4);
    int64_t pick[4], next[4];
    int np = -1, nn = -1;
    CHECK(qmoe_predictor_predict(p, 0, sel, 2, 2, pick, &np, next, &nn) == 0);
    CHECK(np == 2 && pick[0] == 1 && pick[1] == 2 && nn == 0);
    qmoe_predictor_free(p);
    qmoe_cache_free(c);
}

static void checkpoint_cases(const char *dir) {
    /* c/tests/test_safetensors.c:63-110: prefix lookup and whole reads */
    qmoe_err err;
    char path[4096];
    snprintf(path, sizeof(path), "%s/model.safetensors", dir);
    FILE *f = fopen(path, "wb");
    CHECK(f != NULL);
    if (!f) return;
    const char *hdr = "{\"language_model.model.w\":{\"dtype\":\"U16\",\"shape\":[2,3],"
                      "\"data_offsets\":[0,12]}}";
    uint64_t hlen = strlen(hdr);
    uint16_t data[6] = {1, 2, 3, 4, 5, 6};
    fwrite(&hlen, 8, 1, f);
    fwrite(hdr, 1, hlen, f);
    fwrite(data, 2, 6, f);
    fclose(f);
    qmoe_ckpt *ck = qmoe_ckpt_open(dir, 2, &err);
    CHECK(ck != NULL);
    if (!ck) {
        fprintf(stderr, "%s\n", err.msg);
        return;
    }
    qmoe_tensor_info t;
    CHECK(qmoe_ckpt_find(ck, "model.w", &t) == 0 && t.dtype == QMOE_ST_U16 && t.ndim == 2 &&
          t.shape[0] == 2 && t.shape[1] == 3 && t.row_bytes == 6);
    uint16_t out[6] = {0};
    CHECK(qmoe_ckpt_read_tensor(ck, "model.w", out, sizeof(out), &err) == 0 &&
          memcmp(out, data, sizeof(data)) == 0);
    const int64_t rows[3] = {1, 0, 1};
    uint16_t r[9];
    CHECK(qmoe_ckpt_read_rows(ck, "model.w", rows, 3, r, sizeof(r), &err) == 0);
    CHECK(r[0] == 4 && r[3] == 1 && r[6] == 4);
    qmoe_io_stats st;
    CHECK(qmoe_ckpt_io_stats(ck, &st) == 0 && st.rows_read == 3 && st.tensors_read == 1);
    const int64_t past[1] = {2};
    CHECK(qmoe_ckpt_read_rows(ck, "model.w", past, 1, r, sizeof(r), &err) == -1 &&
          strstr(err.msg, "outside") != NULL);
    qmoe_ckpt_close(ck);
    remove(path);
}

int main(int argc, char **argv) {
    cache_cases();
    predictor_cases();
    if (argc > 1) checkpoint_cases(argv[1]);
    printf("%s: %d failure(s)\n", qmoe_version(), failures);
    return failures ? 1 : 0;
}
