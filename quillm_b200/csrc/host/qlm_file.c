/* .qlm loader over a read-only private mapping (format in include/qlm_file.h).
 *
 * The header is walked with one explicit byte position and one bounds predicate (`fits`): nothing is
 * read before it is known to lie inside the buffer.  Each section has its own small parser that reports
 * success or failure; qlm_parse turns a failure into a message naming the section, the entry index and
 * the byte position, frees what it allocated and returns -1.
 *
 * What a file must satisfy to load (the reference loader's acceptance rules, src/qlm_file.c:73-150;
 * tests/test_loader.py checks acceptance and the parsed result against the compiled reference on
 * thousands of mutated headers):
 *   prelude  "QLMF", version 1, at most QLM_MAX_KV key/value entries and QLM_MAX_TENSORS tensors, and
 *            a data offset that is a multiple of QM_ALIGN and not past the end of the file;
 *   entries  a key of 1..63 bytes with no NUL; a value of type u32 or f32 (4 bytes), string (u32 length
 *            and that many bytes) or u32 array (u32 count and 4 bytes per element);
 *   tensors  a name of 1..63 bytes with no NUL; a known dtype; 1..4 dimensions, each in [1, 2^40],
 *            whose product is at most 2^40; an offset that is a multiple of QM_ALIGN; the tensor's bytes
 *            inside the data region;
 *   and the header ends at or before the data offset.
 * The messages "bad magic" and "unsupported version N" are the ones callers of the reference see and
 * test for; the others are this loader's own. */
#include "qlm_file.h"

#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define QLM_PRELUDE_BYTES 24u            /* magic, version, n_kv, n_tensors, data offset */
#define QLM_MAX_ELEMS ((uint64_t)1 << 40) /* per dimension and per tensor */

typedef struct {
    const uint8_t *base;
    size_t size; /* bytes in the buffer */
    size_t pos;  /* next unread byte */
} walk;

static int fits(const walk *w, uint64_t n) { return n <= (uint64_t)(w->size - w->pos); }

static uint32_t load_le32(const uint8_t *p) {
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}
static uint64_t load_le64(const uint8_t *p) { return (uint64_t)load_le32(p) | (uint64_t)load_le32(p + 4) << 32; }

/* each reader advances only over bytes that are there; 0 on success */
static int get_u32(walk *w, uint32_t *v) {
    if (!fits(w, 4)) return -1;
    *v = load_le32(w->base + w->pos);
    w->pos += 4;
    return 0;
}
static int get_u64(walk *w, uint64_t *v) {
    if (!fits(w, 8)) return -1;
    *v = load_le64(w->base + w->pos);
    w->pos += 8;
    return 0;
}
static int get_span(walk *w, uint64_t n, const uint8_t **p) {
    if (!fits(w, n)) return -1;
    *p = w->base + w->pos;
    w->pos += (size_t)n;
    return 0;
}
/* u32 length + bytes into dst[cap] as a C string: 1..cap-1 bytes, none of them NUL */
static int get_name(walk *w, char *dst, size_t cap) {
    uint32_t n;
    const uint8_t *s;
    if (get_u32(w, &n) || n == 0 || n >= cap || get_span(w, n, &s) || memchr(s, 0, n)) return -1;
    memcpy(dst, s, n);
    dst[n] = '\0';
    return 0;
}

static int say(char *err, size_t errlen, const char *fmt, ...) {
    if (err && errlen) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, errlen, fmt, ap);
        va_end(ap);
    }
    return -1;
}

/* one key/value entry */
static int parse_entry(walk *w, qlm_kv *kv) {
    uint32_t raw;
    if (get_name(w, kv->key, sizeof kv->key) || get_u32(w, &kv->type)) return -1;
    switch (kv->type) {
    case QLM_KV_U32: return get_u32(w, &kv->u32);
    case QLM_KV_F32:
        if (get_u32(w, &raw)) return -1;
        memcpy(&kv->f32, &raw, sizeof raw);
        return 0;
    case QLM_KV_STR: return get_u32(w, &kv->len) || get_span(w, kv->len, (const uint8_t **)&kv->str);
    case QLM_KV_ARR_U32: return get_u32(w, &kv->len) || get_span(w, (uint64_t)kv->len * 4, &kv->arr);
    default: return -1;
    }
}

/* one tensor entry up to its offset (the range check against the data region is the caller's) */
static int parse_tensor(walk *w, qm_tensor *t, uint64_t *off) {
    uint32_t dt, nd;
    if (get_name(w, t->name, sizeof t->name) || get_u32(w, &dt) || get_u32(w, &nd)) return -1;
    if (!qm_dtype_valid(dt) || nd < 1 || nd > 4) return -1;
    t->type = (qm_dtype)dt;
    t->ndim = (int)nd;
    uint64_t elems = 1;
    for (uint32_t d = 0; d < nd; d++) {
        uint64_t ne;
        if (get_u64(w, &ne) || ne == 0 || ne > QLM_MAX_ELEMS || elems > QLM_MAX_ELEMS / ne) return -1;
        elems *= ne;
        t->ne[d] = (int64_t)ne;
    }
    return get_u64(w, off) || *off % QM_ALIGN != 0 ? -1 : 0;
}

int qlm_parse(qlm_file *f, const uint8_t *buf, size_t size, char *err, size_t errlen) {
    memset(f, 0, sizeof *f);
    if (size < 4 || memcmp(buf, QLM_MAGIC, 4) != 0) return say(err, errlen, "bad magic");
    if (size < 8) return say(err, errlen, "file ends inside the %u-byte header prelude", QLM_PRELUDE_BYTES);
    const uint32_t version = load_le32(buf + 4);
    if (version != QLM_VERSION) return say(err, errlen, "unsupported version %u", version);
    if (size < QLM_PRELUDE_BYTES)
        return say(err, errlen, "file ends inside the %u-byte header prelude", QLM_PRELUDE_BYTES);
    const uint32_t n_kv = load_le32(buf + 8), n_t = load_le32(buf + 12);
    const uint64_t data_off = load_le64(buf + 16);
    if (n_kv > QLM_MAX_KV || n_t > QLM_MAX_TENSORS)
        return say(err, errlen, "header declares %u key/value entries and %u tensors (limits %d and %d)", n_kv, n_t,
                   QLM_MAX_KV, QLM_MAX_TENSORS);
    if (data_off % QM_ALIGN != 0 || data_off > size)
        return say(err, errlen, "data offset %llu is not a multiple of %d or lies past the end of the %zu-byte file",
                   (unsigned long long)data_off, QM_ALIGN, size);

    qlm_kv *kv = calloc(n_kv ? n_kv : 1, sizeof *kv);
    qm_tensor *tn = calloc(n_t ? n_t : 1, sizeof *tn);
    if (!kv || !tn) {
        free(kv);
        free(tn);
        return say(err, errlen, "out of memory for %u entries and %u tensors", n_kv, n_t);
    }
    f->kv = kv, f->tensors = tn, f->n_kv = n_kv, f->n_tensors = n_t;

    walk w = {buf, size, QLM_PRELUDE_BYTES};
    for (uint32_t i = 0; i < n_kv; i++) {
        const size_t at = w.pos;
        if (parse_entry(&w, &kv[i])) {
            qlm_close(f);
            return say(err, errlen, "key/value entry %u (at byte %zu) is malformed or truncated", i, at);
        }
    }
    const uint64_t data_bytes = size - (size_t)data_off;
    for (uint32_t i = 0; i < n_t; i++) {
        const size_t at = w.pos;
        uint64_t off = 0;
        if (parse_tensor(&w, &tn[i], &off)) {
            qlm_close(f);
            return say(err, errlen, "tensor entry %u (at byte %zu) is malformed or truncated", i, at);
        }
        const uint64_t bytes = qm_tensor_bytes(&tn[i]);
        if (off > data_bytes || bytes > data_bytes - off) {
            say(err, errlen, "tensor '%s' (%llu bytes at data offset %llu) lies outside the %llu-byte data region",
                tn[i].name, (unsigned long long)bytes, (unsigned long long)off, (unsigned long long)data_bytes);
            qlm_close(f);
            return -1;
        }
        tn[i].data = buf + data_off + off;
    }
    if (w.pos > data_off) {
        qlm_close(f);
        return say(err, errlen, "header (%zu bytes) runs into the data at byte %llu", w.pos, (unsigned long long)data_off);
    }
    return 0;
}

int qlm_open(qlm_file *f, const char *path, char *err, size_t errlen) {
    memset(f, 0, sizeof *f);
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return say(err, errlen, "cannot open %s: %s", path, strerror(errno));
    struct stat st;
    const int stat_ok = fstat(fd, &st) == 0 && st.st_size > 0;
    void *map = stat_ok ? mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    close(fd); /* the mapping keeps the file's pages */
    if (!stat_ok) return say(err, errlen, "%s is empty or cannot be inspected", path);
    if (map == MAP_FAILED) return say(err, errlen, "cannot map %s: %s", path, strerror(errno));
    if (qlm_parse(f, map, (size_t)st.st_size, err, errlen) != 0) {
        munmap(map, (size_t)st.st_size);
        return -1;
    }
    f->map = map;
    f->map_size = (size_t)st.st_size;
    return 0;
}

void qlm_close(qlm_file *f) {
    if (f->map) munmap(f->map, f->map_size);
    free(f->kv);
    free(f->tensors);
    memset(f, 0, sizeof *f);
}

const qlm_kv *qlm_find_kv(const qlm_file *f, const char *key) {
    for (uint32_t i = 0; i < f->n_kv; i++)
        if (strcmp(f->kv[i].key, key) == 0) return &f->kv[i];
    return NULL;
}

const qm_tensor *qlm_find_tensor(const qlm_file *f, const char *name) {
    for (uint32_t i = 0; i < f->n_tensors; i++)
        if (strcmp(f->tensors[i].name, name) == 0) return &f->tensors[i];
    return NULL;
}

uint32_t qlm_arr_get(const qlm_kv *kv, uint32_t i) { return load_le32(kv->arr + (size_t)i * 4); }
