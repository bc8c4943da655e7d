/* .qlm loader: bounds-checked parser over a read-only private mapping (format in include/qlm_file.h).
 * Same acceptance rules as the reference loader (src/qlm_file.c:73-150): every count, name, dtype,
 * shape, offset and size is checked against the buffer before use; a failure frees everything and
 * returns -1 with a message. */
#include "qlm_file.h"

#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef struct {
    const uint8_t *buf;
    size_t size, at;
    int broken; /* sticky: set by the first out-of-range read */
} cursor;

static const uint8_t *take(cursor *c, size_t n) {
    if (c->broken || n > c->size - c->at) {
        c->broken = 1;
        return NULL;
    }
    const uint8_t *p = c->buf + c->at;
    c->at += n;
    return p;
}

static uint32_t le32(const uint8_t *p) {
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

static uint32_t take_u32(cursor *c) {
    const uint8_t *p = take(c, 4);
    return p ? le32(p) : 0;
}

static uint64_t take_u64(cursor *c) {
    const uint64_t lo = take_u32(c), hi = take_u32(c);
    return lo | (hi << 32);
}

static int errf(char *err, size_t errlen, const char *fmt, ...) {
    if (err && errlen) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, errlen, fmt, ap);
        va_end(ap);
    }
    return -1;
}

/* length-prefixed name into dst[cap]: 1..cap-1 bytes, no embedded NUL */
static int take_name(cursor *c, char *dst, size_t cap) {
    const uint32_t n = take_u32(c);
    if (c->broken || n == 0 || n >= cap) return -1;
    const uint8_t *s = take(c, n);
    if (!s || memchr(s, 0, n)) return -1;
    memcpy(dst, s, n);
    dst[n] = 0;
    return 0;
}

int qlm_parse(qlm_file *f, const uint8_t *buf, size_t size, char *err, size_t errlen) {
    memset(f, 0, sizeof *f);
    cursor c = {buf, size, 0, 0};
    const uint8_t *magic = take(&c, 4);
    if (!magic || memcmp(magic, QLM_MAGIC, 4) != 0) return errf(err, errlen, "bad magic");
    const uint32_t version = take_u32(&c);
    if (version != QLM_VERSION) return errf(err, errlen, "unsupported version %u", version);
    const uint32_t n_kv = take_u32(&c), n_t = take_u32(&c);
    const uint64_t data_off = take_u64(&c);
    if (c.broken) return errf(err, errlen, "truncated header");
    if (n_kv > QLM_MAX_KV || n_t > QLM_MAX_TENSORS) return errf(err, errlen, "too many entries");
    if (data_off % QM_ALIGN || data_off > size) return errf(err, errlen, "bad data offset");
    f->kv = calloc(n_kv ? n_kv : 1, sizeof *f->kv);
    f->tensors = calloc(n_t ? n_t : 1, sizeof *f->tensors);
    if (!f->kv || !f->tensors) {
        qlm_close(f);
        return errf(err, errlen, "out of memory");
    }
    f->n_kv = n_kv;
    f->n_tensors = n_t;
    for (uint32_t i = 0; i < n_kv; i++) {
        qlm_kv *kv = &f->kv[i];
        if (take_name(&c, kv->key, sizeof kv->key)) goto malformed;
        kv->type = take_u32(&c);
        if (kv->type == QLM_KV_U32) {
            kv->u32 = take_u32(&c);
        } else if (kv->type == QLM_KV_F32) {
            const uint32_t b = take_u32(&c);
            memcpy(&kv->f32, &b, 4);
        } else if (kv->type == QLM_KV_STR) {
            kv->len = take_u32(&c);
            kv->str = (const char *)take(&c, kv->len);
        } else if (kv->type == QLM_KV_ARR_U32) {
            kv->len = take_u32(&c);
            if (!c.broken && kv->len > (size - c.at) / 4) goto malformed;
            kv->arr = take(&c, (size_t)kv->len * 4);
        } else {
            goto malformed;
        }
        if (c.broken) goto malformed;
    }
    const size_t data_bytes = size - (size_t)data_off;
    for (uint32_t i = 0; i < n_t; i++) {
        qm_tensor *t = &f->tensors[i];
        if (take_name(&c, t->name, sizeof t->name)) goto malformed;
        const uint32_t dt = take_u32(&c), nd = take_u32(&c);
        if (c.broken || !qm_dtype_valid(dt) || nd < 1 || nd > 4) goto malformed;
        t->type = (qm_dtype)dt;
        t->ndim = (int)nd;
        uint64_t total = 1;
        const uint64_t cap = (uint64_t)1 << 40;
        for (uint32_t d = 0; d < nd; d++) {
            const uint64_t ne = take_u64(&c);
            if (ne == 0 || ne > cap || total > cap / ne) goto malformed;
            total *= ne;
            t->ne[d] = (int64_t)ne;
        }
        const uint64_t off = take_u64(&c);
        if (c.broken || off % QM_ALIGN) goto malformed;
        const size_t bytes = qm_tensor_bytes(t);
        if (off > data_bytes || bytes > data_bytes - off) {
            errf(err, errlen, "tensor '%s' out of range", t->name);
            qlm_close(f);
            return -1;
        }
        t->data = buf + data_off + off;
    }
    if (c.at > data_off) goto malformed; /* header runs into the data */
    return 0;
malformed:
    qlm_close(f);
    return errf(err, errlen, "malformed header near byte %zu", c.at);
}

int qlm_open(qlm_file *f, const char *path, char *err, size_t errlen) {
    memset(f, 0, sizeof *f);
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return errf(err, errlen, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        return errf(err, errlen, "cannot stat %s", path);
    }
    const size_t size = (size_t)st.st_size;
    void *map = mmap(NULL, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return errf(err, errlen, "mmap failed");
    if (qlm_parse(f, map, size, err, errlen) != 0) {
        munmap(map, size);
        return -1;
    }
    f->map = map;
    f->map_size = size;
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
        if (!strcmp(f->kv[i].key, key)) return &f->kv[i];
    return NULL;
}

const qm_tensor *qlm_find_tensor(const qlm_file *f, const char *name) {
    for (uint32_t i = 0; i < f->n_tensors; i++)
        if (!strcmp(f->tensors[i].name, name)) return &f->tensors[i];
    return NULL;
}

uint32_t qlm_arr_get(const qlm_kv *kv, uint32_t i) { return le32(kv->arr + (size_t)i * 4); }
