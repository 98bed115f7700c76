/* Minimal JSON reader for config.json, model.safetensors.index.json and
   safetensors headers (RFC 8259: objects, arrays, strings with escapes,
   numbers, true/false/null). The whole document is parsed into a tree;
   json_free releases it. */
#ifndef MLXD_ENGINE_JSON_H
#define MLXD_ENGINE_JSON_H

#include <stddef.h>

typedef enum { JSON_NULL, JSON_BOOL, JSON_NUM, JSON_STR, JSON_ARR, JSON_OBJ } json_type;

typedef struct json_val {
    json_type type;
    int boolean;
    double num;
    char *str;                  /* JSON_STR: decoded UTF-8, NUL-terminated */
    int n;                      /* JSON_ARR / JSON_OBJ: entries */
    struct json_val **items;    /* values */
    char **keys;                /* JSON_OBJ: keys (same order as in the text) */
} json_val;

/* NULL on a syntax error (message in err) */
json_val *json_parse(const char *text, size_t len, char *err, size_t errlen);
json_val *json_parse_file(const char *path, char *err, size_t errlen);
void json_free(json_val *v);

/* member of an object (first match), NULL if absent or not an object */
const json_val *json_get(const json_val *obj, const char *key);
/* typed reads with defaults when absent, null or of another type */
double json_num(const json_val *v, double def);
int json_int(const json_val *obj, const char *key, int def);
double json_double(const json_val *obj, const char *key, double def);
int json_bool(const json_val *obj, const char *key, int def);
const char *json_str(const json_val *obj, const char *key);

#endif
