/* Oracle GGUF reader: GgufModelFile.ReadHeader restated (Gguf.cs:143-208) over an mmap of one file.
 * Test infrastructure only (see oracle.h). */
#include "oracle.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef struct { char* key; int type, arr_type; int64_t ival; double fval; char* sval; int64_t arr_len; } kv_t;
typedef struct { char* name; int64_t dims[4]; int ndims; int type; int64_t offset, size; uint8_t* owned; } tinfo_t;

struct or_gguf {
    uint8_t* map; size_t len;
    kv_t* kv; int nkv;
    tinfo_t* t; int nt;
};

typedef struct { const uint8_t* p; const uint8_t* end; int bad; } rd_t;

static int rd(rd_t* r, void* dst, size_t n)
{
    if (r->bad || (size_t)(r->end - r->p) < n) { r->bad = 1; memset(dst, 0, n); return 0; }
    memcpy(dst, r->p, n); r->p += n; return 1;
}
static uint32_t rd_u32(rd_t* r) { uint32_t v; rd(r, &v, 4); return v; }
static uint64_t rd_u64(rd_t* r) { uint64_t v; rd(r, &v, 8); return v; }
static char* rd_str(rd_t* r)
{
    uint64_t len = rd_u64(r);
    if (r->bad || len > (uint64_t)(r->end - r->p)) { r->bad = 1; return NULL; }
    char* s = (char*)malloc(len + 1);
    memcpy(s, r->p, len); s[len] = 0; r->p += len;
    return s;
}

static int scalar_size(int t)
{
    switch (t) { case 0: case 1: case 7: return 1; case 2: case 3: return 2; case 4: case 5: case 6: return 4;
                 case 10: case 11: case 12: return 8; }
    return -1;
}

static void read_scalar(rd_t* r, kv_t* kv, int t)
{
    uint8_t b[8] = {0};
    switch (t) {
    case 0: rd(r, b, 1); kv->ival = b[0]; break;
    case 1: rd(r, b, 1); kv->ival = (int8_t)b[0]; break;
    case 2: { uint16_t v; rd(r, &v, 2); kv->ival = v; break; }
    case 3: { int16_t v; rd(r, &v, 2); kv->ival = v; break; }
    case 4: { uint32_t v; rd(r, &v, 4); kv->ival = v; break; }
    case 5: { int32_t v; rd(r, &v, 4); kv->ival = v; break; }
    case 6: { float v; rd(r, &v, 4); kv->fval = v; kv->ival = (int64_t)v; break; }
    case 7: rd(r, b, 1); kv->ival = b[0] != 0; break;
    case 8: kv->sval = rd_str(r); break;
    case 10: { uint64_t v; rd(r, &v, 8); kv->ival = (int64_t)v; break; }
    case 11: { int64_t v; rd(r, &v, 8); kv->ival = v; break; }
    case 12: { double v; rd(r, &v, 8); kv->fval = v; kv->ival = (int64_t)v; break; }
    default: r->bad = 1;
    }
    if (t == 6 || t == 12) { /* keep fval */ } else kv->fval = (double)kv->ival;
}

static void set_err(char* err, int errlen, const char* msg, const char* path)
{
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s: %s", path, msg);
}

or_gguf* or_gguf_open(const char* path, char* err, int errlen)
{
    int fd = open(path, O_RDONLY);
    if (fd < 0) { set_err(err, errlen, "cannot open", path); return NULL; }
    struct stat st; fstat(fd, &st);
    size_t len = (size_t)st.st_size;
    if (len < 24) { close(fd); set_err(err, errlen, "is not a GGUF file", path); return NULL; }
    uint8_t* map = (uint8_t*)mmap(NULL, len, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { set_err(err, errlen, "mmap failed", path); return NULL; }
    rd_t r = { map, map + len, 0 };
    or_gguf* g = (or_gguf*)calloc(1, sizeof(or_gguf));
    g->map = map; g->len = len;
    if (rd_u32(&r) != 0x46554747u) { set_err(err, errlen, "is not a GGUF file", path); or_gguf_close(g); return NULL; }
    uint32_t version = rd_u32(&r);
    if (version < 2 || version > 3) { set_err(err, errlen, "unsupported GGUF version", path); or_gguf_close(g); return NULL; }
    int64_t nt = (int64_t)rd_u64(&r), nkv = (int64_t)rd_u64(&r);
    if (nt < 0 || nkv < 0 || nt > 1000000 || nkv > 1000000) { set_err(err, errlen, "bad tensor or key count", path); or_gguf_close(g); return NULL; }
    g->kv = (kv_t*)calloc((size_t)nkv + 1, sizeof(kv_t));
    int64_t alignment = 32;
    for (int64_t i = 0; i < nkv && !r.bad; i++) {
        kv_t* kv = &g->kv[g->nkv++];
        kv->key = rd_str(&r);
        kv->type = (int)rd_u32(&r);
        if (kv->type == 9) {
            kv->arr_type = (int)rd_u32(&r);
            kv->arr_len = (int64_t)rd_u64(&r);
            if (kv->arr_len < 0) { r.bad = 1; break; }
            if (kv->arr_type == 8) { for (int64_t j = 0; j < kv->arr_len && !r.bad; j++) free(rd_str(&r)); }
            else {
                int sz = scalar_size(kv->arr_type);
                if (sz < 0 || (uint64_t)(r.end - r.p) < (uint64_t)sz * (uint64_t)kv->arr_len) { r.bad = 1; break; }
                r.p += sz * kv->arr_len;
            }
        } else read_scalar(&r, kv, kv->type);
        if (kv->key && strcmp(kv->key, "general.alignment") == 0) alignment = kv->ival;
    }
    if (r.bad) { set_err(err, errlen, "truncated or malformed header", path); or_gguf_close(g); return NULL; }
    if (alignment <= 0 || (alignment & (alignment - 1)) != 0) { set_err(err, errlen, "general.alignment must be a power of two", path); or_gguf_close(g); return NULL; }
    g->t = (tinfo_t*)calloc((size_t)nt + 1, sizeof(tinfo_t));
    for (int64_t i = 0; i < nt && !r.bad; i++) {
        tinfo_t* t = &g->t[g->nt++];
        t->name = rd_str(&r);
        uint32_t nd = rd_u32(&r);
        if (nd == 0 || nd > 4) { set_err(err, errlen, "tensor has a bad dim count", path); or_gguf_close(g); return NULL; }
        t->ndims = (int)nd;
        for (uint32_t d = 0; d < nd; d++) {
            t->dims[d] = (int64_t)rd_u64(&r);
            if (t->dims[d] <= 0) { set_err(err, errlen, "tensor has a non-positive dim", path); or_gguf_close(g); return NULL; }
        }
        for (int d = (int)nd; d < 4; d++) t->dims[d] = 1;
        t->type = (int)rd_u32(&r);
        t->offset = (int64_t)rd_u64(&r);
        for (int64_t j = 0; j + 1 < g->nt; j++)
            if (t->name && g->t[j].name && strcmp(g->t[j].name, t->name) == 0) { set_err(err, errlen, "duplicate tensor", path); or_gguf_close(g); return NULL; }
    }
    if (r.bad) { set_err(err, errlen, "truncated tensor index", path); or_gguf_close(g); return NULL; }
    int64_t data_off = ((int64_t)(r.p - map) + alignment - 1) / alignment * alignment;
    for (int i = 0; i < g->nt; i++) {
        tinfo_t* t = &g->t[i];
        int bs, ts;
        if (!or_layout(t->type, &bs, &ts)) { set_err(err, errlen, "tensor uses an unreadable type", path); or_gguf_close(g); return NULL; }
        if (t->dims[0] % bs != 0) { set_err(err, errlen, "tensor row is not a multiple of the block size", path); or_gguf_close(g); return NULL; }
        int64_t ne = t->dims[0] * t->dims[1] * t->dims[2] * t->dims[3];
        t->size = ne / bs * ts;
        t->offset += data_off;
        if (t->offset + t->size > (int64_t)len) { set_err(err, errlen, "tensor extends past the end of the file", path); or_gguf_close(g); return NULL; }
    }
    return g;
}

void or_gguf_close(or_gguf* g)
{
    if (!g) return;
    for (int i = 0; i < g->nkv; i++) { free(g->kv[i].key); free(g->kv[i].sval); }
    for (int i = 0; i < g->nt; i++) { free(g->t[i].name); free(g->t[i].owned); }
    free(g->kv); free(g->t);
    if (g->map) munmap(g->map, g->len);
    free(g);
}

int or_gguf_tensor_count(const or_gguf* g) { return g->nt; }
const char* or_gguf_tensor_name(const or_gguf* g, int i) { return g->t[i].name; }
int or_gguf_find(const or_gguf* g, const char* name)
{
    for (int i = 0; i < g->nt; i++) if (strcmp(g->t[i].name, name) == 0) return i;
    return -1;
}
int or_gguf_tensor_info(const or_gguf* g, int i, int* type, int64_t dims[4], int* ndims, int64_t* size, const uint8_t** data)
{
    if (i < 0 || i >= g->nt) return -1;
    const tinfo_t* t = &g->t[i];
    if (type) *type = t->type;
    if (dims) for (int d = 0; d < 4; d++) dims[d] = t->dims[d];
    if (ndims) *ndims = t->ndims;
    if (size) *size = t->size;
    if (data) *data = t->owned ? t->owned : g->map + t->offset;
    return 0;
}

static const kv_t* find_kv(const or_gguf* g, const char* key)
{
    for (int i = 0; i < g->nkv; i++) if (g->kv[i].key && strcmp(g->kv[i].key, key) == 0) return &g->kv[i];
    return NULL;
}
int or_gguf_has(const or_gguf* g, const char* key) { return find_kv(g, key) != NULL; }
int64_t or_gguf_get_int(const or_gguf* g, const char* key, int64_t dflt) { const kv_t* k = find_kv(g, key); return k && k->type != 8 && k->type != 9 ? k->ival : dflt; }
float or_gguf_get_float(const or_gguf* g, const char* key, float dflt) { const kv_t* k = find_kv(g, key); return k && k->type != 8 && k->type != 9 ? (float)k->fval : dflt; }
const char* or_gguf_get_string(const or_gguf* g, const char* key, const char* dflt) { const kv_t* k = find_kv(g, key); return k && k->type == 8 && k->sval ? k->sval : dflt; }
int or_gguf_get_bool(const or_gguf* g, const char* key, int dflt) { const kv_t* k = find_kv(g, key); return k && k->type != 8 && k->type != 9 ? k->ival != 0 : dflt; }

/* In-memory GGUF: the same index as a file, with tensor bytes owned by the object (used to build synthetic models
 * without writing them to disk). */
or_gguf* or_gguf_mem_new(void) { return (or_gguf*)calloc(1, sizeof(or_gguf)); }

static kv_t* mem_kv(or_gguf* g, const char* key, int type)
{
    g->kv = (kv_t*)realloc(g->kv, sizeof(kv_t) * (size_t)(g->nkv + 1));
    kv_t* k = &g->kv[g->nkv++];
    memset(k, 0, sizeof *k);
    k->key = strdup(key); k->type = type;
    return k;
}
void or_gguf_mem_set_int(or_gguf* g, const char* key, int64_t v) { kv_t* k = mem_kv(g, key, 11); k->ival = v; k->fval = (double)v; }
void or_gguf_mem_set_float(or_gguf* g, const char* key, float v) { kv_t* k = mem_kv(g, key, 6); k->fval = v; k->ival = (int64_t)v; }
void or_gguf_mem_set_string(or_gguf* g, const char* key, const char* v) { kv_t* k = mem_kv(g, key, 8); k->sval = strdup(v); }
void or_gguf_mem_add_tensor(or_gguf* g, const char* name, int type, int nd, const int64_t* dims, uint8_t* data, int64_t size)
{
    g->t = (tinfo_t*)realloc(g->t, sizeof(tinfo_t) * (size_t)(g->nt + 1));
    tinfo_t* t = &g->t[g->nt++];
    memset(t, 0, sizeof *t);
    t->name = strdup(name); t->type = type; t->ndims = nd; t->size = size; t->owned = data;
    for (int d = 0; d < 4; d++) t->dims[d] = d < nd ? dims[d] : 1;
}

/* Writes the metadata scalars and tensors of g as a GGUF v3 file (32-byte alignment). */
int or_gguf_save(const or_gguf* g, const char* path)
{
    FILE* f = fopen(path, "wb");
    if (!f) return -1;
    uint32_t magic = 0x46554747u, version = 3;
    int64_t nt = g->nt, nkv = g->nkv;
    fwrite(&magic, 4, 1, f); fwrite(&version, 4, 1, f); fwrite(&nt, 8, 1, f); fwrite(&nkv, 8, 1, f);
    for (int i = 0; i < g->nkv; i++) {
        const kv_t* k = &g->kv[i];
        uint64_t n = strlen(k->key); fwrite(&n, 8, 1, f); fwrite(k->key, 1, n, f);
        int32_t ty = k->type == 11 ? 4 : k->type;          /* ints are written as uint32 */
        fwrite(&ty, 4, 1, f);
        if (k->type == 8) { uint64_t m = strlen(k->sval); fwrite(&m, 8, 1, f); fwrite(k->sval, 1, m, f); }
        else if (k->type == 6) { float v = (float)k->fval; fwrite(&v, 4, 1, f); }
        else { uint32_t v = (uint32_t)k->ival; fwrite(&v, 4, 1, f); }
    }
    uint64_t off = 0;
    for (int i = 0; i < g->nt; i++) {
        const tinfo_t* t = &g->t[i];
        uint64_t n = strlen(t->name); fwrite(&n, 8, 1, f); fwrite(t->name, 1, n, f);
        uint32_t nd = (uint32_t)t->ndims; fwrite(&nd, 4, 1, f);
        for (int d = 0; d < t->ndims; d++) fwrite(&t->dims[d], 8, 1, f);
        int32_t ty = t->type; fwrite(&ty, 4, 1, f);
        fwrite(&off, 8, 1, f);
        off += (uint64_t)((t->size + 31) / 32 * 32);
    }
    static const uint8_t z[32] = {0};
    long p = ftell(f); if (p % 32) fwrite(z, 1, (size_t)(32 - p % 32), f);
    for (int i = 0; i < g->nt; i++) {
        const tinfo_t* t = &g->t[i];
        const uint8_t* d = t->owned ? t->owned : g->map + t->offset;
        fwrite(d, 1, (size_t)t->size, f);
        p = ftell(f); if (p % 32) fwrite(z, 1, (size_t)(32 - p % 32), f);
    }
    int bad = ferror(f);
    fclose(f);
    return bad ? -1 : 0;
}
