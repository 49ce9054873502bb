/* Small recursive-descent JSON reader: config.json and safetensors headers (the reference parses
   the same two documents with src/json.c). Numbers are doubles; strings keep \uXXXX escapes as
   UTF-8. Depth is bounded so a malformed file cannot exhaust the stack. */
#include "nb.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct { const char *p, *end, *begin; char *err; size_t errlen; int depth; } jp;

static void ws(jp *s) { while (s->p < s->end && (*s->p == ' ' || *s->p == '\n' || *s->p == '\r' || *s->p == '\t')) s->p++; }
static nbj_t *fail(jp *s, const char *msg) {
    if (s->errlen && !s->err[0]) snprintf(s->err, s->errlen, "json: %s at offset %ld", msg, (long)(s->p - s->begin));
    return NULL;
}
static void put_utf8(char **o, unsigned cp) {
    if (cp < 0x80) *(*o)++ = (char)cp;
    else if (cp < 0x800) { *(*o)++ = (char)(0xc0 | (cp >> 6)); *(*o)++ = (char)(0x80 | (cp & 0x3f)); }
    else if (cp < 0x10000) { *(*o)++ = (char)(0xe0 | (cp >> 12)); *(*o)++ = (char)(0x80 | ((cp >> 6) & 0x3f)); *(*o)++ = (char)(0x80 | (cp & 0x3f)); }
    else { *(*o)++ = (char)(0xf0 | (cp >> 18)); *(*o)++ = (char)(0x80 | ((cp >> 12) & 0x3f)); *(*o)++ = (char)(0x80 | ((cp >> 6) & 0x3f)); *(*o)++ = (char)(0x80 | (cp & 0x3f)); }
}
static int hex4(const char *p, unsigned *v) {
    *v = 0;
    for (int i = 0; i < 4; ++i) {
        char c = p[i];
        *v <<= 4;
        if (c >= '0' && c <= '9') *v |= (unsigned)(c - '0');
        else if (c >= 'a' && c <= 'f') *v |= (unsigned)(c - 'a' + 10);
        else if (c >= 'A' && c <= 'F') *v |= (unsigned)(c - 'A' + 10);
        else return -1;
    }
    return 0;
}
static char *parse_str(jp *s) {
    if (s->p >= s->end || *s->p != '"') return NULL;
    s->p++;
    const char *q = s->p;
    size_t n = 0;
    while (q < s->end && *q != '"') { if (*q == '\\') q++; q++; n++; }
    if (q >= s->end) return NULL;
    char *out = malloc(n * 4 + 1), *o = out;
    while (s->p < s->end && *s->p != '"') {
        char c = *s->p++;
        if (c != '\\') { *o++ = c; continue; }
        if (s->p >= s->end) { free(out); return NULL; }
        c = *s->p++;
        switch (c) {
        case 'n': *o++ = '\n'; break;
        case 't': *o++ = '\t'; break;
        case 'r': *o++ = '\r'; break;
        case 'b': *o++ = '\b'; break;
        case 'f': *o++ = '\f'; break;
        case 'u': {
            unsigned cp;
            if (s->end - s->p < 4 || hex4(s->p, &cp)) { free(out); return NULL; }
            s->p += 4;
            if (cp >= 0xd800 && cp < 0xdc00 && s->end - s->p >= 6 && s->p[0] == '\\' && s->p[1] == 'u') {
                unsigned lo;
                if (!hex4(s->p + 2, &lo) && lo >= 0xdc00 && lo < 0xe000) { cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00); s->p += 6; }
            }
            put_utf8(&o, cp);
            break;
        }
        default: *o++ = c;
        }
    }
    s->p++; /* closing quote */
    *o = 0;
    return out;
}
static nbj_t *parse_val(jp *s);
static nbj_t *newv(nbj_type t) { nbj_t *v = calloc(1, sizeof *v); v->type = t; return v; }
static void push(nbj_t *v, char *key, nbj_t *item, size_t *cap) {
    if (v->count == *cap) {
        *cap = *cap ? *cap * 2 : 8;
        v->items = realloc(v->items, *cap * sizeof *v->items);
        if (v->type == NBJ_OBJ) v->keys = realloc(v->keys, *cap * sizeof *v->keys);
    }
    if (v->type == NBJ_OBJ) v->keys[v->count] = key;
    v->items[v->count++] = item;
}
static nbj_t *parse_val(jp *s) {
    ws(s);
    if (s->p >= s->end) return fail(s, "unexpected end");
    if (++s->depth > 64) return fail(s, "nesting too deep");
    nbj_t *v = NULL;
    char c = *s->p;
    if (c == '{' || c == '[') {
        const int obj = c == '{';
        v = newv(obj ? NBJ_OBJ : NBJ_ARR);
        size_t cap = 0;
        s->p++;
        ws(s);
        if (s->p < s->end && *s->p == (obj ? '}' : ']')) { s->p++; s->depth--; return v; }
        for (;;) {
            char *key = NULL;
            if (obj) {
                ws(s);
                key = parse_str(s);
                if (!key) { nbj_free(v); return fail(s, "bad key"); }
                ws(s);
                if (s->p >= s->end || *s->p != ':') { free(key); nbj_free(v); return fail(s, "expected ':'"); }
                s->p++;
            }
            nbj_t *item = parse_val(s);
            if (!item) { free(key); nbj_free(v); return NULL; }
            push(v, key, item, &cap);
            ws(s);
            if (s->p < s->end && *s->p == ',') { s->p++; continue; }
            if (s->p < s->end && *s->p == (obj ? '}' : ']')) { s->p++; break; }
            nbj_free(v);
            return fail(s, "expected ',' or close");
        }
    } else if (c == '"') {
        char *str = parse_str(s);
        if (!str) return fail(s, "bad string");
        v = newv(NBJ_STR);
        v->str = str;
    } else if (c == 't' && s->end - s->p >= 4 && !strncmp(s->p, "true", 4)) {
        v = newv(NBJ_BOOL); v->num = 1; s->p += 4;
    } else if (c == 'f' && s->end - s->p >= 5 && !strncmp(s->p, "false", 5)) {
        v = newv(NBJ_BOOL); s->p += 5;
    } else if (c == 'n' && s->end - s->p >= 4 && !strncmp(s->p, "null", 4)) {
        v = newv(NBJ_NULL); s->p += 4;
    } else {
        char buf[64];
        size_t n = 0;
        while (s->p + n < s->end && n < sizeof buf - 1 && strchr("+-0123456789.eE", s->p[n])) { buf[n] = s->p[n]; n++; }
        if (!n) return fail(s, "unexpected character");
        buf[n] = 0;
        char *endp;
        double d = strtod(buf, &endp);
        if (endp != buf + n) return fail(s, "bad number");
        s->p += n;
        v = newv(NBJ_NUM);
        v->num = d;
    }
    s->depth--;
    return v;
}

nbj_t *nbj_parse(const char *text, size_t len, char *err, size_t errlen) {
    jp s = { text, text + len, text, err, errlen, 0 };
    if (errlen) err[0] = 0;
    nbj_t *v = parse_val(&s);
    if (v) {
        ws(&s);
        if (s.p != s.end) { nbj_free(v); return fail(&s, "trailing data"); }
    }
    return v;
}
void nbj_free(nbj_t *v) {
    if (!v) return;
    for (size_t i = 0; i < v->count; ++i) {
        nbj_free(v->items[i]);
        if (v->keys) free(v->keys[i]);
    }
    free(v->items);
    free(v->keys);
    free(v->str);
    free(v);
}
const nbj_t *nbj_get(const nbj_t *o, const char *key) {
    if (!o || o->type != NBJ_OBJ) return NULL;
    for (size_t i = 0; i < o->count; ++i) if (!strcmp(o->keys[i], key)) return o->items[i];
    return NULL;
}
double nbj_num(const nbj_t *v, double d) { return v && (v->type == NBJ_NUM || v->type == NBJ_BOOL) ? v->num : d; }
const char *nbj_str(const nbj_t *v, const char *d) { return v && v->type == NBJ_STR ? v->str : d; }
size_t nbj_len(const nbj_t *v) { return v && (v->type == NBJ_ARR || v->type == NBJ_OBJ) ? v->count : 0; }
const nbj_t *nbj_at(const nbj_t *a, size_t i) { return a && (a->type == NBJ_ARR || a->type == NBJ_OBJ) && i < a->count ? a->items[i] : NULL; }
