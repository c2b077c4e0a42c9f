/*
 * qmoe_ckpt.c - safetensors checkpoint reader feeding the expert pools.
 *
 * Replaces the reference's storage layer on the MoE path:
 *   index + validation   c/src/safetensors.c:49-286, storage.py:69-152
 *   name lookup          c/src/safetensors.c:289-309 (language_model. prefix)
 *   row reads            c/src/reader.c:11-112, storage.py:200-243 (sorted
 *                        unique rows, one pread per contiguous run, rows
 *                        returned in request order, duplicates read once)
 *   expert rows          c/src/model.c:539-674 (the nine rows of an expert)
 *   layer tensors        c/src/model.c:215-266, :1902-1923
 *
 * Reads are plain pread(2) calls spread over io_workers threads: whole
 * tensors in pieces of at most QK_PIECE bytes, row reads one contiguous run
 * per work item. The header parser is a small JSON reader of its own that
 * accepts what the reference's parsers accept for a safetensors header.
 */
#include <dirent.h>
#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include "../../include/qmoe.h"
#include "qmoe_internal.h"

#define QK_PIECE (32u << 20) /* largest single work item of a whole-tensor read */

static void ck_err(qmoe_err *err, const char *fmt, ...) {
    if (!err) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err->msg, sizeof(err->msg), fmt, ap);
    va_end(ap);
}

static double ck_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* dtype names and element sizes, c/src/safetensors.c:13-22 (QMOE_ST_* order) */
static const struct {
    const char *name;
    int size;
} kDtypes[QMOE_ST_COUNT] = {
    {"BOOL", 1}, {"U8", 1}, {"I8", 1},  {"U16", 2},  {"I16", 2},  {"U32", 4}, {"I32", 4},
    {"U64", 8},  {"I64", 8}, {"F16", 2}, {"BF16", 2}, {"F32", 4}, {"F64", 8},
};

typedef struct {
    char *name; /* stored name without the language_model. prefix */
    int file, dtype, ndim;
    int64_t shape[8];
    uint64_t offset; /* absolute, in the file */
    uint64_t nbytes;
} ck_tensor;

struct qmoe_ckpt {
    char **paths;
    int *fds;
    int nfiles;
    ck_tensor *t;
    size_t n, cap;
    int workers;
    pthread_mutex_t lock;
    qmoe_io_stats stats;
};

/* ------------------------------------------------------- header parsing */

typedef struct {
    const char *p, *end;
    int depth;
} jcur;

static void jws(jcur *c) {
    while (c->p < c->end && (*c->p == ' ' || *c->p == '\t' || *c->p == '\n' || *c->p == '\r'))
        c->p++;
}

static int jlit(jcur *c, const char *lit) {
    size_t n = strlen(lit);
    if ((size_t)(c->end - c->p) < n || memcmp(c->p, lit, n)) return -1;
    c->p += n;
    return 0;
}

static int hexv(char ch) {
    if (ch >= '0' && ch <= '9') return ch - '0';
    if (ch >= 'a' && ch <= 'f') return ch - 'a' + 10;
    if (ch >= 'A' && ch <= 'F') return ch - 'A' + 10;
    return -1;
}

static int jhex4(jcur *c, unsigned *out) {
    if (c->end - c->p < 4) return -1;
    unsigned v = 0;
    for (int i = 0; i < 4; i++) {
        int h = hexv(c->p[i]);
        if (h < 0) return -1;
        v = v * 16 + (unsigned)h;
    }
    c->p += 4;
    *out = v;
    return 0;
}

static size_t put_utf8(char *o, unsigned cp) {
    if (cp < 0x80) {
        o[0] = (char)cp;
        return 1;
    }
    if (cp < 0x800) {
        o[0] = (char)(0xC0 | (cp >> 6));
        o[1] = (char)(0x80 | (cp & 0x3F));
        return 2;
    }
    if (cp < 0x10000) {
        o[0] = (char)(0xE0 | (cp >> 12));
        o[1] = (char)(0x80 | ((cp >> 6) & 0x3F));
        o[2] = (char)(0x80 | (cp & 0x3F));
        return 3;
    }
    o[0] = (char)(0xF0 | (cp >> 18));
    o[1] = (char)(0x80 | ((cp >> 12) & 0x3F));
    o[2] = (char)(0x80 | ((cp >> 6) & 0x3F));
    o[3] = (char)(0x80 | (cp & 0x3F));
    return 4;
}

/* length of the UTF-8 sequence at p (at most `left` bytes), 0 if invalid.
 * Encoded surrogates (ED A0-BF ..) pass, as Python's json.loads decodes a
 * header with 'surrogatepass'; overlong forms and code points above
 * U+10FFFF do not. */
static int utf8_len(const unsigned char *p, ptrdiff_t left) {
    const unsigned char b = p[0];
    int n;
    unsigned char lo = 0x80, hi = 0xBF;
    if (b >= 0xC2 && b <= 0xDF) n = 2;
    else if (b >= 0xE0 && b <= 0xEF) {
        n = 3;
        if (b == 0xE0) lo = 0xA0;
    } else if (b >= 0xF0 && b <= 0xF4) {
        n = 4;
        if (b == 0xF0) lo = 0x90;
        if (b == 0xF4) hi = 0x8F;
    } else
        return 0;
    if (left < n || p[1] < lo || p[1] > hi) return 0;
    for (int i = 2; i < n; i++)
        if (p[i] < 0x80 || p[i] > 0xBF) return 0;
    return n;
}

/* a JSON string at c->p; *out (malloc'd, NUL-terminated, escapes decoded)
 * when out is not NULL. The text must be UTF-8. */
static int jstr(jcur *c, char **out) {
    if (c->p >= c->end || *c->p != '"') return -1;
    c->p++;
    char *buf = out ? malloc((size_t)(c->end - c->p) + 1) : NULL;
    if (out && !buf) return -1;
    size_t n = 0;
    while (c->p < c->end && *c->p != '"') {
        unsigned char ch = (unsigned char)*c->p;
        if (ch < 0x20) goto bad;
        if (ch >= 0x80) {
            const int u = utf8_len((const unsigned char *)c->p, c->end - c->p);
            if (!u) goto bad;
            if (buf) memcpy(buf + n, c->p, (size_t)u);
            n += buf ? (size_t)u : 0;
            c->p += u;
            continue;
        }
        c->p++;
        if (ch != '\\') {
            if (buf) buf[n++] = (char)ch;
            continue;
        }
        if (c->p >= c->end) goto bad;
        char e = *c->p++;
        unsigned cp;
        switch (e) {
        case '"': cp = '"'; break;
        case '\\': cp = '\\'; break;
        case '/': cp = '/'; break;
        case 'b': cp = '\b'; break;
        case 'f': cp = '\f'; break;
        case 'n': cp = '\n'; break;
        case 'r': cp = '\r'; break;
        case 't': cp = '\t'; break;
        case 'u':
            if (jhex4(c, &cp)) goto bad;
            if (cp >= 0xD800 && cp < 0xDC00 && c->end - c->p >= 6 && c->p[0] == '\\' &&
                c->p[1] == 'u') {
                jcur save = *c;
                unsigned lo;
                c->p += 2;
                if (!jhex4(c, &lo) && lo >= 0xDC00 && lo < 0xE000)
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                else
                    *c = save;
            }
            break;
        default: goto bad;
        }
        if (buf) n += put_utf8(buf + n, cp);
    }
    if (c->p >= c->end) goto bad;
    c->p++;
    if (buf) {
        buf[n] = 0;
        *out = buf;
    }
    return 0;
bad:
    free(buf);
    return -1;
}

/* kinds of scalar the header fields care about */
enum { J_OTHER = 0, J_INT = 1 };

/* a JSON number; J_INT with *v when it is an integer token (no fraction or
 * exponent) that fits in int64, *ovf set when it is an integer that does not */
static int jnum(jcur *c, int *kind, int64_t *v, int *ovf) {
    int neg = 0;
    if (c->p < c->end && *c->p == '-') {
        neg = 1;
        c->p++;
    }
    if (c->p >= c->end || *c->p < '0' || *c->p > '9') return -1;
    if (*c->p == '0' && c->p + 1 < c->end && c->p[1] >= '0' && c->p[1] <= '9') return -1;
    uint64_t acc = 0;
    int big = 0;
    while (c->p < c->end && *c->p >= '0' && *c->p <= '9') {
        unsigned dgt = (unsigned)(*c->p - '0');
        if (acc > (UINT64_MAX - dgt) / 10) big = 1;
        else acc = acc * 10 + dgt;
        c->p++;
    }
    int integer = 1;
    if (c->p < c->end && *c->p == '.') {
        integer = 0;
        c->p++;
        if (c->p >= c->end || *c->p < '0' || *c->p > '9') return -1;
        while (c->p < c->end && *c->p >= '0' && *c->p <= '9') c->p++;
    }
    if (c->p < c->end && (*c->p == 'e' || *c->p == 'E')) {
        integer = 0;
        c->p++;
        if (c->p < c->end && (*c->p == '+' || *c->p == '-')) c->p++;
        if (c->p >= c->end || *c->p < '0' || *c->p > '9') return -1;
        while (c->p < c->end && *c->p >= '0' && *c->p <= '9') c->p++;
    }
    *kind = integer ? J_INT : J_OTHER;
    *ovf = 0;
    if (integer) {
        if (big || acc > (uint64_t)INT64_MAX) {
            *ovf = 1;
            *v = neg ? INT64_MIN : INT64_MAX;
        } else {
            *v = neg ? -(int64_t)acc : (int64_t)acc;
        }
    }
    return 0;
}

static int jskip(jcur *c);

/* nesting deeper than this is refused (json.loads accepts several hundred
 * levels; the bound keeps the recursion's stack use small) */
#define QK_JSON_DEPTH 512

static int jskip_container(jcur *c, char open, char close) {
    if (++c->depth > QK_JSON_DEPTH) return -1;
    c->p++; /* open */
    jws(c);
    if (c->p < c->end && *c->p == close) {
        c->p++;
        c->depth--;
        return 0;
    }
    for (;;) {
        jws(c);
        if (open == '{') {
            if (jstr(c, NULL)) return -1;
            jws(c);
            if (c->p >= c->end || *c->p != ':') return -1;
            c->p++;
            jws(c);
        }
        if (jskip(c)) return -1;
        jws(c);
        if (c->p >= c->end) return -1;
        if (*c->p == ',') {
            c->p++;
            continue;
        }
        if (*c->p == close) {
            c->p++;
            c->depth--;
            return 0;
        }
        return -1;
    }
}

static int jskip(jcur *c) {
    jws(c);
    if (c->p >= c->end) return -1;
    switch (*c->p) {
    case '{': return jskip_container(c, '{', '}');
    case '[': return jskip_container(c, '[', ']');
    case '"': return jstr(c, NULL);
    case 't': return jlit(c, "true");
    case 'f': return jlit(c, "false");
    case 'n': return jlit(c, "null");
    default: {
        int k, o;
        int64_t v;
        return jnum(c, &k, &v, &o);
    }
    }
}

/* an array of JSON values; ints[] gets the first `cap` of them, *n their
 * count, *all_int whether every one is an integer token (one beyond int64
 * saturates, and then fails the range checks as an unbounded integer would) */
static int jint_array(jcur *c, int64_t *ints, int cap, int *n, int *all_int) {
    if (c->p >= c->end || *c->p != '[') return -1;
    c->p++;
    *n = 0;
    *all_int = 1;
    jws(c);
    if (c->p < c->end && *c->p == ']') {
        c->p++;
        return 0;
    }
    for (;;) {
        jws(c);
        if (c->p >= c->end) return -1;
        char ch = *c->p;
        if (ch == '-' || (ch >= '0' && ch <= '9')) {
            int kind, ovf;
            int64_t v;
            if (jnum(c, &kind, &v, &ovf)) return -1;
            if (kind != J_INT) *all_int = 0; /* an integer too large for int64 saturates */
            if (*n < cap) ints[*n] = v;
        } else {
            if (jskip(c)) return -1;
            *all_int = 0;
        }
        (*n)++;
        jws(c);
        if (c->p >= c->end) return -1;
        if (*c->p == ',') {
            c->p++;
            continue;
        }
        if (*c->p == ']') {
            c->p++;
            return 0;
        }
        return -1;
    }
}

/* one header entry's fields (storage.py:110-140) */
typedef struct {
    int is_obj;
    int has_dtype;
    char *dtype;
    char dtype_repr[32]; /* a non-string dtype as Python prints it ("" = None) */
    int offs_is_arr, offs_n, offs_int;
    int64_t offs[2];
    int shape_is_arr, shape_n, shape_int;
    int64_t shape[9];
} jentry;

static int jentry_parse(jcur *c, jentry *e) {
    memset(e, 0, sizeof(*e));
    jws(c);
    if (c->p >= c->end) return -1;
    if (*c->p != '{') return jskip(c); /* not an object: reported by the caller */
    e->is_obj = 1;
    c->p++;
    jws(c);
    if (c->p < c->end && *c->p == '}') {
        c->p++;
        return 0;
    }
    for (;;) {
        jws(c);
        char *key = NULL;
        if (jstr(c, &key)) return -1;
        jws(c);
        if (c->p >= c->end || *c->p != ':') {
            free(key);
            return -1;
        }
        c->p++;
        jws(c);
        int rc = 0;
        if (!strcmp(key, "dtype")) {
            free(e->dtype);
            e->dtype = NULL;
            e->has_dtype = 0;
            e->dtype_repr[0] = 0;
            if (c->p < c->end && *c->p == '"') {
                rc = jstr(c, &e->dtype);
                e->has_dtype = rc == 0;
            } else {
                /* how Python prints a non-string dtype in the error message */
                const char *t0 = c->p;
                rc = jskip(c);
                const size_t tl = (size_t)(c->p - t0);
                if (!rc && tl == 4 && !memcmp(t0, "true", 4)) snprintf(e->dtype_repr, 32, "True");
                else if (!rc && tl == 5 && !memcmp(t0, "false", 5)) snprintf(e->dtype_repr, 32, "False");
                else if (!rc && (*t0 == '-' || (*t0 >= '0' && *t0 <= '9'))) {
                    jcur nc = {t0, c->p, 0};
                    int kind, ovf;
                    int64_t v;
                    if (!jnum(&nc, &kind, &v, &ovf) && kind == J_INT && !ovf)
                        snprintf(e->dtype_repr, 32, "%lld", (long long)v);
                    else
                        snprintf(e->dtype_repr, 32, "%.*s", (int)(tl < 31 ? tl : 31), t0);
                }
            }
        } else if (!strcmp(key, "data_offsets") || !strcmp(key, "shape")) {
            const int offs = key[0] == 'd';
            int *is_arr = offs ? &e->offs_is_arr : &e->shape_is_arr;
            if (c->p < c->end && *c->p == '[') {
                *is_arr = 1;
                rc = offs ? jint_array(c, e->offs, 2, &e->offs_n, &e->offs_int)
                          : jint_array(c, e->shape, 9, &e->shape_n, &e->shape_int);
            } else {
                *is_arr = 0;
                rc = jskip(c);
            }
        } else {
            rc = jskip(c);
        }
        free(key);
        if (rc) return -1;
        jws(c);
        if (c->p >= c->end) return -1;
        if (*c->p == ',') {
            c->p++;
            continue;
        }
        if (*c->p == '}') {
            c->p++;
            return 0;
        }
        return -1;
    }
}

/* ------------------------------------------------------------ the index */

static ck_tensor *ck_add(qmoe_ckpt *ck) {
    if (ck->n == ck->cap) {
        size_t nc = ck->cap ? ck->cap * 2 : 256;
        ck_tensor *t = realloc(ck->t, nc * sizeof(ck_tensor));
        if (!t) return NULL;
        ck->t = t;
        ck->cap = nc;
    }
    ck_tensor *t = &ck->t[ck->n++];
    memset(t, 0, sizeof(*t));
    return t;
}

typedef struct {
    uint64_t lo, hi;
    const char *name;
} ck_range;

static int cmp_range(const void *a, const void *b) {
    const ck_range *x = a, *y = b;
    if (x->lo != y->lo) return x->lo < y->lo ? -1 : 1;
    if (x->hi != y->hi) return x->hi < y->hi ? -1 : 1;
    return 0;
}

static int find_dtype(const char *s) {
    for (int i = 0; i < QMOE_ST_COUNT; i++)
        if (!strcmp(kDtypes[i].name, s)) return i;
    return -1;
}

/* one file's header into the index (storage.py:92-152 checks and messages;
 * c/src/safetensors.c:49-236). On failure the file's tensors are dropped. */
static int parse_file(qmoe_ckpt *ck, const char *path, int fi, qmoe_err *err) {
    int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        ck_err(err, "cannot open %s: %s", path, strerror(errno));
        return -1;
    }
    struct stat sb;
    if (fstat(fd, &sb)) {
        ck_err(err, "cannot stat %s: %s", path, strerror(errno));
        close(fd);
        return -1;
    }
    const uint64_t fsize = (uint64_t)sb.st_size;
    uint8_t lb[8];
    if (pread(fd, lb, 8, 0) != 8) {
        ck_err(err, "truncated safetensors header: %s", path);
        close(fd);
        return -1;
    }
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | lb[i];
    if (hlen > fsize - 8) {
        ck_err(err, "truncated safetensors JSON: %s", path);
        close(fd);
        return -1;
    }
    char *hdr = malloc((size_t)hlen + 1);
    if (!hdr) {
        ck_err(err, "out of host memory reading %s", path);
        close(fd);
        return -1;
    }
    size_t got = 0;
    while (got < hlen) {
        ssize_t r = pread(fd, hdr + got, (size_t)hlen - got, (off_t)(8 + got));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) {
            ck_err(err, "truncated safetensors JSON: %s", path);
            free(hdr);
            close(fd);
            return -1;
        }
        got += (size_t)r;
    }
    hdr[hlen] = 0;
    const uint64_t base = 8 + hlen;
    const size_t first = ck->n;
    ck_range *ranges = NULL;
    size_t nr = 0, rcap = 0;
    int failed = 1;
    jcur c = {hdr, hdr + hlen, 0};
    /* a leading UTF-8 byte-order mark is dropped, as json.loads does for a
     * header given as bytes */
    if (hlen >= 3 && !memcmp(hdr, "\xEF\xBB\xBF", 3)) c.p += 3;
    jws(&c);
    if (c.p >= c.end || *c.p != '{') {
        /* valid JSON of another kind, or not JSON at all */
        jcur t = c;
        if (!jskip(&t)) {
            jws(&t);
            if (t.p == t.end) {
                ck_err(err, "safetensors header must be an object: %s", path);
                goto out;
            }
        }
        ck_err(err, "invalid safetensors JSON: %s", path);
        goto out;
    }
    c.p++;
    jws(&c);
    int empty = c.p < c.end && *c.p == '}';
    if (empty) c.p++;
    while (!empty) {
        jws(&c);
        char *stored = NULL;
        if (jstr(&c, &stored)) {
            ck_err(err, "invalid safetensors JSON: %s", path);
            goto out;
        }
        jws(&c);
        if (c.p >= c.end || *c.p != ':') {
            free(stored);
            ck_err(err, "invalid safetensors JSON: %s", path);
            goto out;
        }
        c.p++;
        if (!strcmp(stored, "__metadata__")) {
            free(stored);
            if (jskip(&c)) {
                ck_err(err, "invalid safetensors JSON: %s", path);
                goto out;
            }
        } else {
            jentry e;
            int prc = jentry_parse(&c, &e);
            const char *name = stored;
            if (!strncmp(name, "language_model.", 15)) name += 15;
            int bad = 0;
            if (prc) {
                ck_err(err, "invalid safetensors JSON: %s", path);
                bad = 1;
            } else if (!e.is_obj) {
                ck_err(err, "invalid safetensors entry in %s", path);
                bad = 1;
            } else if (!e.has_dtype || find_dtype(e.dtype) < 0) {
                ck_err(err, "unsupported safetensors dtype %s for %s",
                       e.has_dtype ? e.dtype : e.dtype_repr[0] ? e.dtype_repr : "None", name);
                bad = 1;
            } else if (!e.offs_is_arr || e.offs_n != 2 || !e.shape_is_arr) {
                ck_err(err, "invalid safetensors metadata for %s", name);
                bad = 1;
            } else if (!e.offs_int) {
                ck_err(err, "invalid data offsets for %s", name);
                bad = 1;
            } else if (!e.shape_int || e.shape_n > 8) {
                ck_err(err, e.shape_n > 8 ? "tensor %s has too many dims" : "invalid tensor shape for %s",
                       name);
                bad = 1;
            }
            for (int i = 0; !bad && i < e.shape_n; i++)
                if (e.shape[i] < 0) {
                    ck_err(err, "invalid tensor shape for %s", name);
                    bad = 1;
                }
            const int dt = bad ? -1 : find_dtype(e.dtype);
            uint64_t expect = 0;
            int ovf = 0;
            if (!bad) {
                unsigned __int128 prod = (unsigned __int128)kDtypes[dt].size;
                for (int i = 0; i < e.shape_n; i++) {
                    prod *= (uint64_t)e.shape[i];
                    if (prod > (unsigned __int128)UINT64_MAX) {
                        ovf = 1;
                        prod = 0;
                    }
                }
                expect = (uint64_t)prod;
                const int64_t lo = e.offs[0], hi = e.offs[1];
                if (ovf || lo < 0 || hi < lo || (uint64_t)(hi - lo) != expect ||
                    (uint64_t)hi > fsize - base) {
                    ck_err(err, "invalid safetensors range for %s", name);
                    bad = 1;
                }
            }
            if (!bad)
                for (size_t i = 0; i < ck->n; i++)
                    if (!strcmp(ck->t[i].name, name)) {
                        ck_err(err, "duplicate tensor %s", name);
                        bad = 1;
                        break;
                    }
            ck_tensor *t = bad ? NULL : ck_add(ck);
            if (!bad && !t) {
                ck_err(err, "out of host memory indexing %s", path);
                bad = 1;
            }
            if (!bad) {
                t->name = strdup(name);
                t->file = fi;
                t->dtype = dt;
                t->ndim = e.shape_n;
                for (int i = 0; i < e.shape_n; i++) t->shape[i] = e.shape[i];
                t->offset = base + (uint64_t)e.offs[0];
                t->nbytes = expect;
                if (nr == rcap) {
                    rcap = rcap ? rcap * 2 : 64;
                    ck_range *r2 = realloc(ranges, rcap * sizeof(ck_range));
                    if (!r2 || !t->name) {
                        ck_err(err, "out of host memory indexing %s", path);
                        bad = 1;
                    } else {
                        ranges = r2;
                    }
                }
                if (!bad) ranges[nr++] = (ck_range){(uint64_t)e.offs[0], (uint64_t)e.offs[1], t->name};
            }
            free(e.dtype);
            free(stored);
            if (bad) goto out;
        }
        jws(&c);
        if (c.p < c.end && *c.p == ',') {
            c.p++;
            continue;
        }
        if (c.p < c.end && *c.p == '}') {
            c.p++;
            break;
        }
        ck_err(err, "invalid safetensors JSON: %s", path);
        goto out;
    }
    jws(&c);
    if (c.p != c.end) {
        ck_err(err, "invalid safetensors JSON: %s", path);
        goto out;
    }
    /* overlap check over the ranges sorted by start (storage.py:141-146) */
    qsort(ranges, nr, sizeof(ck_range), cmp_range);
    uint64_t prev_end = 0;
    for (size_t i = 0; i < nr; i++) {
        if (ranges[i].lo < prev_end) {
            ck_err(err, "overlapping safetensors ranges for %s", ranges[i].name);
            goto out;
        }
        prev_end = ranges[i].hi;
    }
    failed = 0;
out:
    free(ranges);
    free(hdr);
    if (failed) {
        while (ck->n > first) free(ck->t[--ck->n].name);
        close(fd);
        return -1;
    }
    ck->fds[fi] = fd;
    ck->paths[fi] = strdup(path);
    return 0;
}

static int cmp_name(const void *a, const void *b) {
    return strcmp(((const ck_tensor *)a)->name, ((const ck_tensor *)b)->name);
}

static int cmp_str(const void *a, const void *b) {
    return strcmp(*(char *const *)a, *(char *const *)b);
}

void qmoe_ckpt_close(qmoe_ckpt *ck) {
    if (!ck) return;
    for (int i = 0; i < ck->nfiles; i++) {
        if (ck->fds && ck->fds[i] >= 0) close(ck->fds[i]);
        if (ck->paths) free(ck->paths[i]);
    }
    free(ck->paths);
    free(ck->fds);
    for (size_t i = 0; i < ck->n; i++) free(ck->t[i].name);
    free(ck->t);
    pthread_mutex_destroy(&ck->lock);
    free(ck);
}

qmoe_ckpt *qmoe_ckpt_open(const char *dir, int io_workers, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!dir) {
        ck_err(err, "qmoe_ckpt_open: no directory");
        return NULL;
    }
    DIR *d = opendir(dir);
    if (!d) {
        ck_err(err, "cannot open model dir %s: %s", dir, strerror(errno));
        return NULL;
    }
    char **names = NULL;
    size_t nn = 0, ncap = 0;
    struct dirent *de;
    int oom = 0;
    while ((de = readdir(d)) != NULL) {
        size_t len = strlen(de->d_name);
        if (len <= 12 || strcmp(de->d_name + len - 12, ".safetensors")) continue;
        if (nn == ncap) {
            ncap = ncap ? ncap * 2 : 16;
            char **n2 = realloc(names, ncap * sizeof(char *));
            if (!n2) {
                oom = 1;
                break;
            }
            names = n2;
        }
        if (!(names[nn] = strdup(de->d_name))) {
            oom = 1;
            break;
        }
        nn++;
    }
    closedir(d);
    qmoe_ckpt *ck = NULL;
    if (oom) {
        ck_err(err, "qmoe_ckpt_open: out of host memory");
        goto done;
    }
    if (!nn) {
        ck_err(err, "no safetensors in %s", dir);
        goto done;
    }
    qsort(names, nn, sizeof(char *), cmp_str);
    ck = calloc(1, sizeof(*ck));
    if (!ck || !(ck->paths = calloc(nn, sizeof(char *))) || !(ck->fds = malloc(nn * sizeof(int)))) {
        ck_err(err, "qmoe_ckpt_open: out of host memory");
        if (ck) {
            free(ck->paths);
            free(ck);
        }
        ck = NULL;
        goto done;
    }
    pthread_mutex_init(&ck->lock, NULL);
    ck->nfiles = (int)nn;
    for (size_t i = 0; i < nn; i++) ck->fds[i] = -1;
    ck->workers = io_workers < 1 ? 1 : io_workers > 64 ? 64 : io_workers;
    for (size_t i = 0; i < nn; i++) {
        size_t pl = strlen(dir) + strlen(names[i]) + 2;
        char *path = malloc(pl);
        if (!path) {
            ck_err(err, "qmoe_ckpt_open: out of host memory");
            qmoe_ckpt_close(ck);
            ck = NULL;
            goto done;
        }
        snprintf(path, pl, "%s/%s", dir, names[i]);
        int rc = parse_file(ck, path, (int)i, err);
        free(path);
        if (rc) {
            qmoe_ckpt_close(ck);
            ck = NULL;
            goto done;
        }
    }
    qsort(ck->t, ck->n, sizeof(ck_tensor), cmp_name);
done:
    for (size_t i = 0; i < nn; i++) free(names[i]);
    free(names);
    return ck;
}

static const ck_tensor *find_exact(const qmoe_ckpt *ck, const char *name) {
    size_t lo = 0, hi = ck->n;
    while (lo < hi) {
        size_t mid = (lo + hi) / 2;
        int c = strcmp(ck->t[mid].name, name);
        if (!c) return &ck->t[mid];
        if (c < 0) lo = mid + 1;
        else hi = mid;
    }
    return NULL;
}

/* c/src/safetensors.c:302-309: exact name, then under language_model. */
static const ck_tensor *ck_find(const qmoe_ckpt *ck, const char *name) {
    if (!ck || !name) return NULL;
    const ck_tensor *t = find_exact(ck, name);
    if (t || strncmp(name, "model.", 6)) return t;
    char pre[1024];
    if (snprintf(pre, sizeof(pre), "language_model.%s", name) >= (int)sizeof(pre)) return NULL;
    return find_exact(ck, pre);
}

static uint64_t row_bytes_of(const ck_tensor *t) {
    return t->ndim && t->shape[0] ? t->nbytes / (uint64_t)t->shape[0] : 0;
}

size_t qmoe_ckpt_count(const qmoe_ckpt *ck) { return ck ? ck->n : 0; }

const char *qmoe_ckpt_name(const qmoe_ckpt *ck, size_t i) {
    return ck && i < ck->n ? ck->t[i].name : NULL;
}

int qmoe_ckpt_find(const qmoe_ckpt *ck, const char *name, qmoe_tensor_info *out) {
    const ck_tensor *t = ck_find(ck, name);
    if (!t) return -1;
    if (out) {
        memset(out, 0, sizeof(*out));
        out->dtype = t->dtype;
        out->ndim = t->ndim;
        for (int i = 0; i < t->ndim; i++) out->shape[i] = t->shape[i];
        out->nbytes = t->nbytes;
        out->row_bytes = row_bytes_of(t);
        out->file = t->file;
        out->offset = t->offset;
    }
    return 0;
}

int qmoe_ckpt_io_stats(const qmoe_ckpt *ck, qmoe_io_stats *out) {
    if (!ck || !out) return -1;
    pthread_mutex_lock((pthread_mutex_t *)&ck->lock);
    *out = ck->stats;
    pthread_mutex_unlock((pthread_mutex_t *)&ck->lock);
    return 0;
}

/* --------------------------------------------------------- parallel I/O */

typedef struct {
    int fd;
    uint64_t off, len;
    uint8_t *dst;
} ck_item;

typedef struct {
    const ck_item *items;
    size_t n;
    atomic_size_t next;
    atomic_ullong calls;
    atomic_int err; /* first errno seen */
} ck_batch;

static void *ck_worker(void *arg) {
    ck_batch *b = arg;
    for (;;) {
        size_t i = atomic_fetch_add(&b->next, 1);
        if (i >= b->n || atomic_load(&b->err)) break;
        const ck_item *it = &b->items[i];
        uint64_t done = 0;
        while (done < it->len) {
            ssize_t r = pread(it->fd, it->dst + done, (size_t)(it->len - done), (off_t)(it->off + done));
            if (r < 0 && errno == EINTR) continue;
            atomic_fetch_add(&b->calls, 1);
            if (r <= 0) {
                int e = r < 0 ? errno : EIO;
                int z = 0;
                atomic_compare_exchange_strong(&b->err, &z, e);
                return NULL;
            }
            done += (uint64_t)r;
        }
    }
    return NULL;
}

/* run the items on up to ck->workers threads (this one included); returns
 * 0 or an errno, and adds the pread calls made to *calls */
static int run_items(const qmoe_ckpt *ck, const ck_item *items, size_t n, uint64_t *calls) {
    ck_batch b;
    b.items = items;
    b.n = n;
    atomic_init(&b.next, 0);
    atomic_init(&b.calls, 0);
    atomic_init(&b.err, 0);
    int nt = ck->workers;
    if ((size_t)nt > n) nt = (int)n;
    pthread_t th[64];
    int started = 0;
    for (int i = 1; i < nt; i++) {
        if (pthread_create(&th[started], NULL, ck_worker, &b)) break;
        started++;
    }
    ck_worker(&b);
    for (int i = 0; i < started; i++) pthread_join(th[i], NULL);
    *calls += atomic_load(&b.calls);
    return atomic_load(&b.err);
}

int qmoe_ckpt_read_tensor(qmoe_ckpt *ck, const char *name, void *out, size_t out_bytes,
                          qmoe_err *err) {
    if (err) err->msg[0] = 0;
    const ck_tensor *t = ck_find(ck, name);
    if (!t) {
        ck_err(err, "missing tensor %s", name ? name : "(null)");
        return -1;
    }
    if (!out || out_bytes < t->nbytes) {
        ck_err(err, "qmoe_ckpt_read_tensor: %s needs %llu bytes", t->name,
               (unsigned long long)t->nbytes);
        return -1;
    }
    const double t0 = ck_now();
    size_t n = (size_t)((t->nbytes + QK_PIECE - 1) / QK_PIECE);
    ck_item stack_items[8], *items = n <= 8 ? stack_items : malloc(n * sizeof(ck_item));
    if (!items) {
        ck_err(err, "qmoe_ckpt_read_tensor: out of host memory");
        return -1;
    }
    for (size_t i = 0; i < n; i++) {
        uint64_t o = (uint64_t)i * QK_PIECE;
        items[i] = (ck_item){ck->fds[t->file], t->offset + o,
                             t->nbytes - o < QK_PIECE ? t->nbytes - o : QK_PIECE, (uint8_t *)out + o};
    }
    uint64_t calls = 0;
    int e = run_items(ck, items, n, &calls);
    if (items != stack_items) free(items);
    pthread_mutex_lock(&ck->lock);
    ck->stats.pread_calls += calls;
    if (!e) {
        ck->stats.bytes_read += t->nbytes;
        ck->stats.tensors_read++;
    }
    ck->stats.read_seconds += ck_now() - t0;
    pthread_mutex_unlock(&ck->lock);
    if (e) {
        ck_err(err, "read failed for %s: %s", t->name, strerror(e));
        return -1;
    }
    return 0;
}

static int cmp_i64(const void *a, const void *b) {
    int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

/* rows of t into out in request order (c/src/reader.c:11-112): the unique
 * rows sorted, one item per contiguous run, duplicates copied from the one
 * read. Rows in strictly increasing order are read straight into out. */
static int read_rows_t(qmoe_ckpt *ck, const ck_tensor *t, const int64_t *rows, size_t n, void *out,
                       qmoe_err *err) {
    if (!t->ndim) {
        ck_err(err, "scalar tensor %s has no rows", t->name);
        return -1;
    }
    for (size_t i = 0; i < n; i++)
        if (rows[i] < 0 || rows[i] >= t->shape[0]) {
            ck_err(err, "row %lld outside %s shape %lld", (long long)rows[i], t->name,
                   (long long)t->shape[0]);
            return -1;
        }
    if (!n) return 0;
    const double t0 = ck_now();
    const uint64_t rb = row_bytes_of(t);
    int increasing = 1;
    for (size_t i = 1; i < n && increasing; i++) increasing = rows[i] > rows[i - 1];
    int64_t *u = malloc(n * sizeof(int64_t));
    ck_item *items = malloc(n * sizeof(ck_item));
    uint8_t *stage = NULL;
    int rc = -1;
    if (!u || !items) {
        ck_err(err, "qmoe_ckpt_read_rows: out of host memory");
        goto out;
    }
    memcpy(u, rows, n * sizeof(int64_t));
    size_t nu = n;
    if (!increasing) {
        qsort(u, n, sizeof(int64_t), cmp_i64);
        nu = 0;
        for (size_t i = 0; i < n; i++)
            if (!nu || u[i] != u[nu - 1]) u[nu++] = u[i];
        stage = malloc((size_t)(nu * rb) + 1);
        if (!stage) {
            ck_err(err, "qmoe_ckpt_read_rows: out of host memory");
            goto out;
        }
    }
    uint8_t *dst = increasing ? (uint8_t *)out : stage;
    size_t ni = 0;
    for (size_t i = 0; i < nu;) {
        size_t j = i + 1;
        while (j < nu && u[j] == u[j - 1] + 1) j++;
        items[ni++] = (ck_item){ck->fds[t->file], t->offset + (uint64_t)u[i] * rb,
                                (uint64_t)(j - i) * rb, dst + (uint64_t)i * rb};
        i = j;
    }
    uint64_t calls = 0;
    int e = rb ? run_items(ck, items, ni, &calls) : 0;
    if (!rb) calls = 1; /* c/src/reader.c:19-22 */
    if (!e && !increasing)
        for (size_t i = 0; i < n; i++) {
            const int64_t *p = bsearch(&rows[i], u, nu, sizeof(int64_t), cmp_i64);
            memcpy((uint8_t *)out + i * rb, stage + (size_t)(p - u) * rb, (size_t)rb);
        }
    pthread_mutex_lock(&ck->lock);
    ck->stats.pread_calls += calls;
    if (!e) {
        ck->stats.bytes_read += (uint64_t)nu * rb;
        ck->stats.rows_read += n;
    }
    ck->stats.read_seconds += ck_now() - t0;
    pthread_mutex_unlock(&ck->lock);
    if (e) {
        ck_err(err, "row read failed for %s: %s", t->name, strerror(e));
        goto out;
    }
    rc = 0;
out:
    free(u);
    free(items);
    free(stage);
    return rc;
}

int qmoe_ckpt_read_rows(qmoe_ckpt *ck, const char *name, const int64_t *rows, size_t n, void *out,
                        size_t out_bytes, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    const ck_tensor *t = ck_find(ck, name);
    if (!t) {
        ck_err(err, "missing tensor %s", name ? name : "(null)");
        return -1;
    }
    if (n && (!rows || !out || out_bytes / (n ? n : 1) < row_bytes_of(t))) {
        ck_err(err, "qmoe_ckpt_read_rows: %s needs %zu rows of %llu bytes", t->name, n,
               (unsigned long long)row_bytes_of(t));
        return -1;
    }
    return read_rows_t(ck, t, rows, n, out, err);
}

/* ---------------------------------------------------- the MoE tensors */

/* the 20 tensors of one MoE layer, in the order they sit in the buffer of
 * qmoe_ckpt_read_layer */
enum {
    P_ROUTER, P_SGATE,
    P_GQ, P_GS, P_GB, P_UQ, P_US, P_UB, P_DQ, P_DS, P_DB,
    P_SGQ, P_SGS, P_SGB, P_SUQ, P_SUS, P_SUB, P_SDQ, P_SDS, P_SDB,
    P_COUNT
};

typedef struct {
    char name[P_COUNT][160];
    int64_t shape[P_COUNT][3];
    int ndim[P_COUNT], dtype[P_COUNT];
    uint64_t bytes[P_COUNT], off[P_COUNT], total;
} layer_plan;

static int plan_layer(const qmoe_config *cfg, int layer, layer_plan *p) {
    if (!cfg || layer < 0) return -1;
    const int64_t E = cfg->num_experts, d = cfg->hidden, I = cfg->moe_inter, g = cfg->group_size;
    if (E < 1 || d < 8 || I < 8 || g < 1 || d % g || I % g || d % 8 || I % 8 || cfg->bits != 4)
        return -1;
    memset(p, 0, sizeof(*p));
    static const char *proj[3] = {"gate_proj", "up_proj", "down_proj"};
    static const char *part[3] = {"weight", "scales", "biases"};
    snprintf(p->name[P_ROUTER], 160, "model.layers.%d.mlp.gate.weight", layer);
    snprintf(p->name[P_SGATE], 160, "model.layers.%d.mlp.shared_expert_gate.weight", layer);
    p->ndim[P_ROUTER] = p->ndim[P_SGATE] = 2;
    p->shape[P_ROUTER][0] = E, p->shape[P_ROUTER][1] = d;
    p->shape[P_SGATE][0] = 1, p->shape[P_SGATE][1] = d;
    p->dtype[P_ROUTER] = p->dtype[P_SGATE] = QMOE_ST_BF16;
    for (int s = 0; s < 2; s++)      /* routed (switch_mlp), shared (shared_expert) */
        for (int j = 0; j < 3; j++)  /* gate, up, down */
            for (int k = 0; k < 3; k++) {
                int i = (s ? P_SGQ : P_GQ) + 3 * j + k;
                snprintf(p->name[i], 160, "model.layers.%d.mlp.%s.%s.%s", layer,
                         s ? "shared_expert" : "switch_mlp", proj[j], part[k]);
                const int64_t rows = j == 2 ? d : I, cols = j == 2 ? I : d;
                const int64_t last = k ? cols / g : cols / 8;
                p->dtype[i] = k ? QMOE_ST_BF16 : QMOE_ST_U32;
                if (s) {
                    p->ndim[i] = 2;
                    p->shape[i][0] = rows, p->shape[i][1] = last;
                } else {
                    p->ndim[i] = 3;
                    p->shape[i][0] = E, p->shape[i][1] = rows, p->shape[i][2] = last;
                }
            }
    uint64_t o = 0;
    for (int i = 0; i < P_COUNT; i++) {
        uint64_t b = i == P_ROUTER || i == P_SGATE || (i - P_GQ) % 3 ? 2 : 4;
        for (int k = 0; k < p->ndim[i]; k++) b *= (uint64_t)p->shape[i][k];
        p->bytes[i] = b;
        p->off[i] = o;
        o += (b + 63) / 64 * 64;
    }
    p->total = o;
    return 0;
}

/* the tensor for plan entry i, checked against the configuration, in *out:
 * 0 and the tensor, or 0 and NULL for an absent biases tensor of the shared
 * expert (which reads as zeros, c/src/model.c:251-257), or -1 */
static int plan_tensor(const qmoe_ckpt *ck, const layer_plan *p, int i, const ck_tensor **out,
                       qmoe_err *err) {
    const ck_tensor *t = ck_find(ck, p->name[i]);
    *out = NULL;
    if (!t) {
        if (i == P_SGB || i == P_SUB || i == P_SDB) return 0;
        if (i >= P_GQ && i <= P_DB)
            ck_err(err, "missing expert tensor %s", p->name[i]); /* model.c:551, :583 */
        else
            ck_err(err, "missing tensor %s", p->name[i]);
        return -1;
    }
    if (t->dtype != p->dtype[i]) {
        ck_err(err, "tensor %s has dtype %s, expected %s", p->name[i], kDtypes[t->dtype].name,
               kDtypes[p->dtype[i]].name);
        return -1;
    }
    int ok = t->ndim == p->ndim[i];
    for (int k = 0; ok && k < t->ndim; k++) ok = t->shape[k] == p->shape[i][k];
    if (!ok) {
        char want[96];
        if (p->ndim[i] == 3)
            snprintf(want, sizeof(want), "[%lld, %lld, %lld]", (long long)p->shape[i][0],
                     (long long)p->shape[i][1], (long long)p->shape[i][2]);
        else
            snprintf(want, sizeof(want), "[%lld, %lld]", (long long)p->shape[i][0],
                     (long long)p->shape[i][1]);
        ck_err(err, "tensor %s does not have the configured shape %s", p->name[i], want);
        return -1;
    }
    *out = t;
    return 0;
}

size_t qmoe_ckpt_layer_bytes(const qmoe_config *cfg) {
    layer_plan p;
    return plan_layer(cfg, 0, &p) ? 0 : (size_t)p.total;
}

int qmoe_ckpt_read_layer(qmoe_ckpt *ck, const qmoe_config *cfg, int layer, void *buf,
                         size_t buf_bytes, qmoe_layer_weights *w, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    layer_plan p;
    if (!ck || !w || plan_layer(cfg, layer, &p)) {
        ck_err(err, "qmoe_ckpt_read_layer: bad arguments");
        return -1;
    }
    if (!buf || buf_bytes < p.total) {
        ck_err(err, "qmoe_ckpt_read_layer: the buffer needs %llu bytes", (unsigned long long)p.total);
        return -1;
    }
    const ck_tensor *t[P_COUNT];
    for (int i = 0; i < P_COUNT; i++)
        if (plan_tensor(ck, &p, i, &t[i], err)) return -1;
    /* one batch of pieces over every tensor, so the workers stay busy across
     * tensor boundaries */
    size_t n = 0;
    for (int i = 0; i < P_COUNT; i++)
        if (t[i]) n += (size_t)((p.bytes[i] + QK_PIECE - 1) / QK_PIECE);
    ck_item *items = malloc((n ? n : 1) * sizeof(ck_item));
    if (!items) {
        ck_err(err, "qmoe_ckpt_read_layer: out of host memory");
        return -1;
    }
    uint8_t *b = buf;
    size_t m = 0;
    int ntensors = 0;
    uint64_t bytes = 0;
    for (int i = 0; i < P_COUNT; i++) {
        if (!t[i]) {
            memset(b + p.off[i], 0, (size_t)p.bytes[i]);
            continue;
        }
        ntensors++;
        bytes += p.bytes[i];
        for (uint64_t o = 0; o < p.bytes[i]; o += QK_PIECE)
            items[m++] = (ck_item){ck->fds[t[i]->file], t[i]->offset + o,
                                   p.bytes[i] - o < QK_PIECE ? p.bytes[i] - o : QK_PIECE,
                                   b + p.off[i] + o};
    }
    const double t0 = ck_now();
    uint64_t calls = 0;
    int e = run_items(ck, items, m, &calls);
    free(items);
    pthread_mutex_lock(&ck->lock);
    ck->stats.pread_calls += calls;
    if (!e) {
        ck->stats.bytes_read += bytes;
        ck->stats.tensors_read += (uint64_t)ntensors;
    }
    ck->stats.read_seconds += ck_now() - t0;
    pthread_mutex_unlock(&ck->lock);
    if (e) {
        ck_err(err, "qmoe_ckpt_read_layer: layer %d: %s", layer, strerror(e));
        return -1;
    }
#define AT(i) ((const void *)(b + p.off[i]))
    memset(w, 0, sizeof(*w));
    w->router = AT(P_ROUTER);
    w->shared_gate = AT(P_SGATE);
    w->logit_bias = NULL;
    w->gate = (qmoe_q4){AT(P_GQ), AT(P_GS), AT(P_GB)};
    w->up = (qmoe_q4){AT(P_UQ), AT(P_US), AT(P_UB)};
    w->down = (qmoe_q4){AT(P_DQ), AT(P_DS), AT(P_DB)};
    w->sh_gate = (qmoe_q4){AT(P_SGQ), AT(P_SGS), AT(P_SGB)};
    w->sh_up = (qmoe_q4){AT(P_SUQ), AT(P_SUS), AT(P_SUB)};
    w->sh_down = (qmoe_q4){AT(P_SDQ), AT(P_SDS), AT(P_SDB)};
#undef AT
    return 0;
}

int qmoe_ckpt_pack_experts(qmoe_ckpt *ck, const qmoe_config *cfg, int layer, const int64_t *ids,
                           size_t n, void *slots, size_t slots_bytes, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    layer_plan p;
    qk_layout L;
    if (!ck || plan_layer(cfg, layer, &p) ||
        qk_layout_init(&L, cfg->hidden, cfg->num_experts, cfg->top_k, cfg->moe_inter, cfg->group_size)) {
        ck_err(err, "qmoe_ckpt_pack_experts: bad arguments");
        return -1;
    }
    if (!n) return 0;
    if (!ids || !slots || slots_bytes / n < L.slot_bytes) {
        ck_err(err, "qmoe_ckpt_pack_experts: %zu slots need %zu bytes", n, n * L.slot_bytes);
        return -1;
    }
    for (size_t i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= cfg->num_experts) {
            ck_err(err, "qmoe_ckpt_pack_experts: expert %lld out of range", (long long)ids[i]);
            return -1;
        }
    /* the nine rows of every expert (c/src/model.c:603-629), each tensor's
     * rows read together so contiguous experts share one pread per tensor */
    const ck_tensor *t[9];
    size_t row[9], total = 0;
    for (int j = 0; j < 9; j++) {
        if (plan_tensor(ck, &p, P_GQ + j, &t[j], err)) return -1;
        row[j] = (size_t)row_bytes_of(t[j]);
        total += row[j] * n;
    }
    uint8_t *stage = malloc(total ? total : 1);
    if (!stage) {
        ck_err(err, "qmoe_ckpt_pack_experts: out of host memory");
        return -1;
    }
    uint8_t *part[9];
    size_t o = 0;
    for (int j = 0; j < 9; j++) {
        part[j] = stage + o;
        o += row[j] * n;
        if (read_rows_t(ck, t[j], ids, n, part[j], err)) {
            free(stage);
            return -1;
        }
    }
    for (size_t i = 0; i < n; i++) {
#define R(j, T) ((const T *)(part[j] + i * row[j]))
        qk_pack_expert(&L, R(0, uint32_t), R(1, uint16_t), R(2, uint16_t), R(3, uint32_t),
                       R(4, uint16_t), R(5, uint16_t), R(6, uint32_t), R(7, uint16_t),
                       R(8, uint16_t), (uint8_t *)slots + i * L.slot_bytes);
#undef R
    }
    free(stage);
    return 0;
}

int qmoe_pack_expert(const qmoe_config *cfg, const qmoe_layer_weights *w, int expert, void *slot) {
    qk_layout L;
    if (!cfg || !w || !slot ||
        qk_layout_init(&L, cfg->hidden, cfg->num_experts, cfg->top_k, cfg->moe_inter, cfg->group_size) ||
        expert < -1 || expert >= cfg->num_experts)
        return -1;
    if (expert < 0) {
        if (!w->sh_gate.q || !w->sh_gate.scales || !w->sh_gate.biases || !w->sh_up.q ||
            !w->sh_up.scales || !w->sh_up.biases || !w->sh_down.q || !w->sh_down.scales ||
            !w->sh_down.biases)
            return -1;
        qk_pack_expert(&L, w->sh_gate.q, w->sh_gate.scales, w->sh_gate.biases, w->sh_up.q,
                       w->sh_up.scales, w->sh_up.biases, w->sh_down.q, w->sh_down.scales,
                       w->sh_down.biases, slot);
        return 0;
    }
    if (!w->gate.q || !w->gate.scales || !w->gate.biases || !w->up.q || !w->up.scales ||
        !w->up.biases || !w->down.q || !w->down.scales || !w->down.biases)
        return -1;
    const size_t d = (size_t)L.d, I = (size_t)L.I, g = (size_t)L.g, e = (size_t)expert;
    const size_t qo = e * I * (d / 8), so = e * I * (d / g), dqo = e * d * (I / 8), dso = e * d * (I / g);
    qk_pack_expert(&L, w->gate.q + qo, w->gate.scales + so, w->gate.biases + so, w->up.q + qo,
                   w->up.scales + so, w->up.biases + so, w->down.q + dqo, w->down.scales + dso,
                   w->down.biases + dso, slot);
    return 0;
}
