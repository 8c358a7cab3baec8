/* Declarations of the part of the jansson 2.x public C API that the
 * reference's gpt2.c uses, written from jansson's published API reference,
 * for linking against the libjansson.so.4 runtime of this image (which ships
 * no headers). Test infrastructure only. */
#ifndef ORACLE_SHIM_JANSSON_H
#define ORACLE_SHIM_JANSSON_H
#include <stddef.h>
#include <stdio.h>
#ifdef __cplusplus
extern "C" {
#endif
typedef enum {
  JSON_OBJECT, JSON_ARRAY, JSON_STRING, JSON_INTEGER, JSON_REAL, JSON_TRUE, JSON_FALSE, JSON_NULL
} json_type;
typedef struct json_t {
  json_type type;
  volatile size_t refcount;
} json_t;
typedef long long json_int_t;
#define JSON_ERROR_TEXT_LENGTH 160
#define JSON_ERROR_SOURCE_LENGTH 80
typedef struct json_error_t {
  int line;
  int column;
  int position;
  char source[JSON_ERROR_SOURCE_LENGTH];
  char text[JSON_ERROR_TEXT_LENGTH];
} json_error_t;
#define JSON_INDENT(n) ((n) & 0x1F)
#define JSON_COMPACT 0x20
#define json_typeof(json) ((json)->type)
#define json_is_string(json) ((json) && json_typeof(json) == JSON_STRING)
json_t *json_object(void);
json_t *json_array(void);
json_t *json_string(const char *value);
json_t *json_integer(json_int_t value);
json_t *json_real(double value);
int json_object_set_new(json_t *object, const char *key, json_t *value);
json_t *json_object_get(const json_t *object, const char *key);
int json_array_append_new(json_t *array, json_t *value);
const char *json_string_value(const json_t *string);
json_t *json_pack(const char *fmt, ...);
json_t *json_loads(const char *input, size_t flags, json_error_t *error);
char *json_dumps(const json_t *json, size_t flags);
int json_dumpf(const json_t *json, FILE *output, size_t flags);
void json_delete(json_t *json);
static inline void json_decref(json_t *json) {
  if (json && json->refcount != (size_t)-1 &&
      __atomic_sub_fetch(&json->refcount, 1, __ATOMIC_RELEASE) == 0)
    json_delete(json);
}
#ifdef __cplusplus
}
#endif
#endif
