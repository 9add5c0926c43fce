/*
 * A minimal Node-API host for testing gemma4_cuda.node where Node.js is not installed: it
 * implements the Node-API calls the addon makes over a small value model (numbers, booleans,
 * strings, typed arrays, arrays, objects, functions, externals, a pending exception), loads the
 * addon with dlopen, registers it through napi_register_module_v1 as Node does, and calls its
 * exports the way cudaExecutor.ts would. Test infrastructure only.
 *
 *   node_host <addon.node> exports
 *   node_host <addon.node> errors
 *   node_host <addon.node> generate key=value... -- seed new_tokens id id ...
 */
#include <dlfcn.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../gemma4-webgpu-engine_b200/napi/node_api_min.h"

typedef enum { V_UNDEF, V_NUM, V_BOOL, V_STR, V_EXT, V_TYPED, V_OBJ, V_FUNC, V_ARR } Kind;

struct napi_value__ {
  Kind k;
  double num;
  bool b;
  char *s;
  void *ext;
  napi_finalize fin;
  napi_typedarray_type tt;
  void *data;
  size_t len;
  int nprop;
  char *pname[64];
  napi_value pval[64];
  napi_callback cb;
  napi_value *el;
};
struct napi_env__ {
  int pending;
  char code[64];
  char msg[2048];
};
struct napi_callback_info__ {
  size_t argc;
  napi_value *argv;
};

static napi_value newv(Kind k) {
  napi_value v = (napi_value)calloc(1, sizeof(struct napi_value__));
  v->k = k;
  return v;
}

napi_status napi_get_cb_info(napi_env env, napi_callback_info ci, size_t *argc, napi_value *argv,
                             napi_value *this_arg, void **data) {
  for (size_t i = 0; i < *argc; i++) argv[i] = i < ci->argc ? ci->argv[i] : newv(V_UNDEF);
  *argc = ci->argc;
  if (this_arg) *this_arg = NULL;
  if (data) *data = NULL;
  return napi_ok;
}
napi_status napi_get_value_int32(napi_env env, napi_value v, int32_t *r) {
  if (!v || v->k != V_NUM) return napi_number_expected;
  *r = (int32_t)v->num;
  return napi_ok;
}
napi_status napi_get_value_double(napi_env env, napi_value v, double *r) {
  if (!v || v->k != V_NUM) return napi_number_expected;
  *r = v->num;
  return napi_ok;
}
napi_status napi_get_value_bool(napi_env env, napi_value v, bool *r) {
  if (!v || v->k != V_BOOL) return napi_boolean_expected;
  *r = v->b;
  return napi_ok;
}
napi_status napi_get_value_string_utf8(napi_env env, napi_value v, char *buf, size_t cap, size_t *r) {
  if (!v || v->k != V_STR) return napi_string_expected;
  size_t n = strlen(v->s);
  if (buf && cap) {
    size_t c = n < cap - 1 ? n : cap - 1;
    memcpy(buf, v->s, c);
    buf[c] = 0;
    n = c;
  }
  if (r) *r = n;
  return napi_ok;
}
napi_status napi_get_typedarray_info(napi_env env, napi_value v, napi_typedarray_type *t, size_t *len,
                                     void **data, napi_value *ab, size_t *off) {
  if (!v || v->k != V_TYPED) return napi_invalid_arg;
  *t = v->tt;
  *len = v->len;
  *data = v->data;
  if (ab) *ab = NULL;
  if (off) *off = 0;
  return napi_ok;
}
static int find_prop(napi_value o, const char *name) {
  for (int i = 0; i < o->nprop; i++)
    if (!strcmp(o->pname[i], name)) return i;
  return -1;
}
napi_status napi_has_named_property(napi_env env, napi_value o, const char *name, bool *r) {
  if (!o || o->k != V_OBJ) return napi_object_expected;
  *r = find_prop(o, name) >= 0;
  return napi_ok;
}
napi_status napi_get_named_property(napi_env env, napi_value o, const char *name, napi_value *r) {
  if (!o || o->k != V_OBJ) return napi_object_expected;
  int i = find_prop(o, name);
  *r = i >= 0 ? o->pval[i] : newv(V_UNDEF);
  return napi_ok;
}
napi_status napi_set_named_property(napi_env env, napi_value o, const char *name, napi_value v) {
  if (!o || o->k != V_OBJ) return napi_object_expected;
  int i = find_prop(o, name);
  if (i < 0) {
    if (o->nprop == 64) return napi_generic_failure;
    i = o->nprop++;
    o->pname[i] = strdup(name);
  }
  o->pval[i] = v;
  return napi_ok;
}
napi_status napi_create_int32(napi_env env, int32_t x, napi_value *r) {
  *r = newv(V_NUM);
  (*r)->num = x;
  return napi_ok;
}
napi_status napi_create_double(napi_env env, double x, napi_value *r) {
  *r = newv(V_NUM);
  (*r)->num = x;
  return napi_ok;
}
napi_status napi_create_string_utf8(napi_env env, const char *s, size_t n, napi_value *r) {
  *r = newv(V_STR);
  (*r)->s = n == NAPI_AUTO_LENGTH ? strdup(s) : strndup(s, n);
  return napi_ok;
}
napi_status napi_create_array_with_length(napi_env env, size_t n, napi_value *r) {
  *r = newv(V_ARR);
  (*r)->len = n;
  (*r)->el = (napi_value *)calloc(n ? n : 1, sizeof(napi_value));
  return napi_ok;
}
napi_status napi_set_element(napi_env env, napi_value o, uint32_t i, napi_value v) {
  if (!o || o->k != V_ARR || i >= o->len) return napi_array_expected;
  o->el[i] = v;
  return napi_ok;
}
static napi_value g_externals[256];
static int g_next;
napi_status napi_create_external(napi_env env, void *data, napi_finalize fin, void *hint, napi_value *r) {
  *r = newv(V_EXT);
  (*r)->ext = data;
  (*r)->fin = fin;
  if (g_next < 256) g_externals[g_next++] = *r;
  return napi_ok;
}
napi_status napi_get_value_external(napi_env env, napi_value v, void **r) {
  if (!v || v->k != V_EXT) return napi_invalid_arg;
  *r = v->ext;
  return napi_ok;
}
napi_status napi_create_function(napi_env env, const char *name, size_t n, napi_callback cb, void *data,
                                 napi_value *r) {
  *r = newv(V_FUNC);
  (*r)->cb = cb;
  return napi_ok;
}
napi_status napi_get_undefined(napi_env env, napi_value *r) {
  *r = newv(V_UNDEF);
  return napi_ok;
}
napi_status napi_throw_error(napi_env env, const char *code, const char *msg) {
  env->pending = 1;
  snprintf(env->code, sizeof env->code, "%s", code ? code : "");
  snprintf(env->msg, sizeof env->msg, "%s", msg ? msg : "");
  return napi_ok;
}
napi_status napi_is_exception_pending(napi_env env, bool *r) {
  *r = env->pending != 0;
  return napi_ok;
}

/* ---------------------------------------------------------------- the calling side */

static struct napi_env__ g_env;
static napi_value g_exports;

static napi_value num(double x) {
  napi_value v = newv(V_NUM);
  v->num = x;
  return v;
}
static napi_value boolean(bool b) {
  napi_value v = newv(V_BOOL);
  v->b = b;
  return v;
}
static napi_value str(const char *s) {
  napi_value v = newv(V_STR);
  v->s = strdup(s);
  return v;
}
static napi_value typed(napi_typedarray_type t, void *data, size_t len) {
  napi_value v = newv(V_TYPED);
  v->tt = t;
  v->data = data;
  v->len = len;
  return v;
}

/* Call exports[name](args...): NULL and the exception printed when one is thrown. */
static napi_value call(const char *name, int argc, ...) {
  napi_value f;
  napi_get_named_property(&g_env, g_exports, name, &f);
  if (f->k != V_FUNC) {
    printf("no export %s\n", name);
    exit(2);
  }
  napi_value argv[8];
  va_list ap;
  va_start(ap, argc);
  for (int i = 0; i < argc; i++) argv[i] = va_arg(ap, napi_value);
  va_end(ap);
  struct napi_callback_info__ ci = {(size_t)argc, argv};
  g_env.pending = 0;
  napi_value r = f->cb(&g_env, &ci);
  if (g_env.pending) {
    printf("threw %s: %s\n", g_env.code, g_env.msg);
    return NULL;
  }
  return r;
}

int main(int argc, char **argv) {
  if (argc < 3) {
    fprintf(stderr, "usage: node_host addon.node exports|errors|generate ...\n");
    return 2;
  }
  void *h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    printf("dlopen failed: %s\n", dlerror());
    return 1;
  }
  napi_value (*reg)(napi_env, napi_value) = (napi_value(*)(napi_env, napi_value))dlsym(h, "napi_register_module_v1");
  if (!reg) {
    printf("no napi_register_module_v1\n");
    return 1;
  }
  g_exports = newv(V_OBJ);
  if (reg(&g_env, g_exports) != g_exports) {
    printf("registration failed\n");
    return 1;
  }
  const char *mode = argv[2];
  if (!strcmp(mode, "exports")) {
    for (int i = 0; i < g_exports->nprop; i++)
      printf("export %s %s\n", g_exports->pname[i], g_exports->pval[i]->k == V_FUNC ? "function" : "other");
    napi_value v = call("version", 0);
    printf("version %s\n", v ? v->s : "?");
    return 0;
  }
  if (!strcmp(mode, "errors")) {
    napi_value opts = newv(V_OBJ);
    napi_set_named_property(&g_env, opts, "maxSeqs", num(1));
    call("createContext", 2, num(99), opts);              /* no such device */
    call("createContext", 0);                              /* missing argument */
    int32_t ids[2] = {1, 2};
    call("prefill", 5, num(0), num(0), typed(napi_int32_array, ids, 2), num(0), boolean(true));
    call("decode", 4, str("not a context"), num(0), num(1), num(0));
    return 0;
  }
  if (!strcmp(mode, "generate")) {
    napi_value opts = newv(V_OBJ);
    int i = 3;
    for (; i < argc && strcmp(argv[i], "--"); i++) {
      char key[128];
      double val;
      if (sscanf(argv[i], "%127[^=]=%lf", key, &val) == 2) napi_set_named_property(&g_env, opts, key, num(val));
    }
    if (i + 3 > argc) return 2;
    const double seed = atof(argv[i + 1]);
    const int n_new = atoi(argv[i + 2]);
    const int n = argc - (i + 3);
    int32_t *prompt = (int32_t *)calloc(n, sizeof(int32_t));
    for (int k = 0; k < n; k++) prompt[k] = atoi(argv[i + 3 + k]);
    napi_value ctx = call("createContext", 2, num(0), opts);
    if (!ctx) return 1;
    if (call("initRandom", 2, ctx, num(seed)) == NULL) return 1;
    napi_value t = call("prefill", 5, ctx, num(0), typed(napi_int32_array, prompt, n), num(0), boolean(true));
    if (!t) return 1;
    int32_t toks[256];
    toks[0] = (int32_t)t->num;
    for (int k = 1; k < n_new && k < 256; k++) {
      napi_value d = call("decodeAhead", 3, ctx, num(0), num(n + k - 1));
      if (!d) return 1;
      toks[k] = (int32_t)d->num;
    }
    printf("tokens");
    for (int k = 0; k < n_new; k++) printf(" %d", toks[k]);
    printf("\n");
    /* The verify pass over the first tokens, from the prompt's end. */
    if (call("kvTruncate", 3, ctx, num(0), num(n)) == NULL) return 1;
    int32_t vt[4];
    const int nv = n_new < 4 ? n_new : 4;
    memcpy(vt, toks, sizeof(int32_t) * nv);
    napi_value ans = call("verify", 4, ctx, num(0), typed(napi_int32_array, vt, nv), num(n));
    if (!ans) return 1;
    printf("verify");
    for (size_t k = 0; k < ans->len; k++) printf(" %d", (int32_t)ans->el[k]->num);
    printf("\n");
    call("kvTruncate", 3, ctx, num(0), num(n));
    call("decode", 4, ctx, num(0), num(-5), num(n));       /* a token outside the vocabulary */
    call("destroyContext", 1, ctx);
    call("decode", 4, ctx, num(0), num(1), num(n));         /* after destroy */
    return 0;
  }
  return 2;
}
