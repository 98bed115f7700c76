/* Minimal JSON reader (see json.h): recursive descent, depth-limited. */
#include "json.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    const char *p, *end;
    char *err;
    size_t errlen;
    int depth;
} jparser;

static void jfail(jparser *ps, const char *msg) {
    if (ps->err && ps->errlen && !ps->err[0])
        snprintf(ps->err, ps->errlen, "json: %s at byte %ld", msg, (long)(ps->end - ps->p));
}

static void skip_ws(jparser *ps) {
    while (ps->p < ps->end && (*ps->p == ' ' || *ps->p == '\t' || *ps->p == '\n' || *ps->p == '\r')) ps->p++;
}

static json_val *jnew(json_type t) {
    json_val *v = calloc(1, sizeof(json_val));
    if (v) v->type = t;
    return v;
}

static int push(json_val *v, json_val *item, char *key) {
    json_val **ni = realloc(v->items, sizeof(json_val *) * (size_t)(v->n + 1));
    if (!ni) return -1;
    v->items = ni;
    if (v->type == JSON_OBJ) {
        char **nk = realloc(v->keys, sizeof(char *) * (size_t)(v->n + 1));
        if (!nk) return -1;
        v->keys = nk;
        v->keys[v->n] = key;
    }
    v->items[v->n++] = item;
    return 0;
}

static int hex4(const char *s, unsigned *out) {
    unsigned v = 0;
    for (int i = 0; i < 4; i++) {
        char c = s[i];
        v <<= 4;
        if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
        else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
        else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
        else return -1;
    }
    *out = v;
    return 0;
}

static size_t put_utf8(char *o, unsigned cp) {
    if (cp < 0x80) { o[0] = (char)cp; return 1; }
    if (cp < 0x800) { o[0] = (char)(0xC0 | (cp >> 6)); o[1] = (char)(0x80 | (cp & 0x3F)); return 2; }
    if (cp < 0x10000) {
        o[0] = (char)(0xE0 | (cp >> 12)); o[1] = (char)(0x80 | ((cp >> 6) & 0x3F)); o[2] = (char)(0x80 | (cp & 0x3F));
        return 3;
    }
    o[0] = (char)(0xF0 | (cp >> 18)); o[1] = (char)(0x80 | ((cp >> 12) & 0x3F));
    o[2] = (char)(0x80 | ((cp >> 6) & 0x3F)); o[3] = (char)(0x80 | (cp & 0x3F));
    return 4;
}

/* a string starting at the opening quote; returns a malloc'd decoded copy */
static char *parse_string(jparser *ps) {
    if (ps->p >= ps->end || *ps->p != '"') { jfail(ps, "expected string"); return NULL; }
    ps->p++;
    const char *s = ps->p;
    size_t cap = 0;
    while (s < ps->end && *s != '"') { if (*s == '\\') s++; s++; cap++; }
    if (s >= ps->end) { jfail(ps, "unterminated string"); return NULL; }
    char *out = malloc(cap * 4 + 1), *o = out;
    if (!out) return NULL;
    while (ps->p < ps->end && *ps->p != '"') {
        unsigned char c = (unsigned char)*ps->p++;
        if (c < 0x20) { free(out); jfail(ps, "control character in string"); return NULL; }
        if (c != '\\') { *o++ = (char)c; continue; }
        if (ps->p >= ps->end) break;
        char e = *ps->p++;
        switch (e) {
        case '"': *o++ = '"'; break;
        case '\\': *o++ = '\\'; break;
        case '/': *o++ = '/'; break;
        case 'b': *o++ = '\b'; break;
        case 'f': *o++ = '\f'; break;
        case 'n': *o++ = '\n'; break;
        case 'r': *o++ = '\r'; break;
        case 't': *o++ = '\t'; break;
        case 'u': {
            unsigned cp;
            if (ps->end - ps->p < 4 || hex4(ps->p, &cp)) { free(out); jfail(ps, "bad \\u escape"); return NULL; }
            ps->p += 4;
            if (cp >= 0xD800 && cp < 0xDC00 && ps->end - ps->p >= 6 && ps->p[0] == '\\' && ps->p[1] == 'u') {
                unsigned lo;
                if (!hex4(ps->p + 2, &lo) && lo >= 0xDC00 && lo < 0xE000) {
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    ps->p += 6;
                }
            }
            o += put_utf8(o, cp);
            break;
        }
        default: free(out); jfail(ps, "bad escape"); return NULL;
        }
    }
    if (ps->p >= ps->end) { free(out); jfail(ps, "unterminated string"); return NULL; }
    ps->p++;   /* closing quote */
    *o = '\0';
    return out;
}

static json_val *parse_value(jparser *ps);

static json_val *parse_container(jparser *ps, int obj) {
    json_val *v = jnew(obj ? JSON_OBJ : JSON_ARR);
    if (!v) return NULL;
    ps->p++;
    skip_ws(ps);
    if (ps->p < ps->end && *ps->p == (obj ? '}' : ']')) { ps->p++; return v; }
    for (;;) {
        char *key = NULL;
        skip_ws(ps);
        if (obj) {
            key = parse_string(ps);
            if (!key) goto fail;
            skip_ws(ps);
            if (ps->p >= ps->end || *ps->p != ':') { free(key); jfail(ps, "expected ':'"); goto fail; }
            ps->p++;
        }
        json_val *item = parse_value(ps);
        if (!item || push(v, item, key)) { free(key); json_free(item); goto fail; }
        skip_ws(ps);
        if (ps->p < ps->end && *ps->p == ',') { ps->p++; continue; }
        if (ps->p < ps->end && *ps->p == (obj ? '}' : ']')) { ps->p++; return v; }
        jfail(ps, obj ? "expected ',' or '}'" : "expected ',' or ']'");
        goto fail;
    }
fail:
    json_free(v);
    return NULL;
}

static json_val *parse_value(jparser *ps) {
    skip_ws(ps);
    if (ps->p >= ps->end) { jfail(ps, "unexpected end"); return NULL; }
    if (++ps->depth > 64) { jfail(ps, "nesting too deep"); return NULL; }
    json_val *v = NULL;
    char c = *ps->p;
    if (c == '{' || c == '[') {
        v = parse_container(ps, c == '{');
    } else if (c == '"') {
        char *s = parse_string(ps);
        if (s && (v = jnew(JSON_STR))) v->str = s;
        else free(s);
    } else if (ps->end - ps->p >= 4 && !strncmp(ps->p, "true", 4)) {
        if ((v = jnew(JSON_BOOL))) v->boolean = 1;
        ps->p += 4;
    } else if (ps->end - ps->p >= 5 && !strncmp(ps->p, "false", 5)) {
        v = jnew(JSON_BOOL);
        ps->p += 5;
    } else if (ps->end - ps->p >= 4 && !strncmp(ps->p, "null", 4)) {
        v = jnew(JSON_NULL);
        ps->p += 4;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
        char buf[64];
        size_t n = 0;
        while (ps->p + n < ps->end && n < sizeof buf - 1 && strchr("+-0123456789.eE", ps->p[n])) n++;
        memcpy(buf, ps->p, n);
        buf[n] = '\0';
        char *endp = NULL;
        double d = strtod(buf, &endp);
        if (endp != buf + n) { jfail(ps, "bad number"); ps->depth--; return NULL; }
        if ((v = jnew(JSON_NUM))) v->num = d;
        ps->p += n;
    } else {
        jfail(ps, "unexpected character");
    }
    ps->depth--;
    return v;
}

json_val *json_parse(const char *text, size_t len, char *err, size_t errlen) {
    if (err && errlen) err[0] = '\0';
    jparser ps = {text, text + len, err, errlen, 0};
    json_val *v = parse_value(&ps);
    if (!v) {
        jfail(&ps, "parse error");
        return NULL;
    }
    skip_ws(&ps);
    if (ps.p != ps.end) {
        jfail(&ps, "trailing characters");
        json_free(v);
        return NULL;
    }
    return v;
}

json_val *json_parse_file(const char *path, char *err, size_t errlen) {
    FILE *f = fopen(path, "rb");
    if (!f) {
        if (err && errlen) snprintf(err, errlen, "cannot open %s", path);
        return NULL;
    }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (n < 0 || n > (1L << 30)) {
        fclose(f);
        if (err && errlen) snprintf(err, errlen, "%s: bad size", path);
        return NULL;
    }
    char *buf = malloc((size_t)n + 1);
    size_t got = buf ? fread(buf, 1, (size_t)n, f) : 0;
    fclose(f);
    if (!buf || got != (size_t)n) {
        free(buf);
        if (err && errlen) snprintf(err, errlen, "%s: read failed", path);
        return NULL;
    }
    json_val *v = json_parse(buf, (size_t)n, err, errlen);
    free(buf);
    return v;
}

void json_free(json_val *v) {
    if (!v) return;
    for (int i = 0; i < v->n; i++) {
        json_free(v->items[i]);
        if (v->keys) free(v->keys[i]);
    }
    free(v->items);
    free(v->keys);
    free(v->str);
    free(v);
}

const json_val *json_get(const json_val *obj, const char *key) {
    if (!obj || obj->type != JSON_OBJ) return NULL;
    for (int i = 0; i < obj->n; i++)
        if (!strcmp(obj->keys[i], key)) return obj->items[i];
    return NULL;
}

double json_num(const json_val *v, double def) {
    if (!v) return def;
    if (v->type == JSON_NUM) return v->num;
    if (v->type == JSON_BOOL) return v->boolean;
    return def;
}

int json_int(const json_val *obj, const char *key, int def) { return (int)json_num(json_get(obj, key), def); }
double json_double(const json_val *obj, const char *key, double def) { return json_num(json_get(obj, key), def); }
int json_bool(const json_val *obj, const char *key, int def) {
    const json_val *v = json_get(obj, key);
    return v && v->type == JSON_BOOL ? v->boolean : def;
}
const char *json_str(const json_val *obj, const char *key) {
    const json_val *v = json_get(obj, key);
    return v && v->type == JSON_STR ? v->str : NULL;
}
