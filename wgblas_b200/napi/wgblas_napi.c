/* Node-API addon: the JavaScript side of wgblas's API (index.mjs, src/init.mjs,
 * src/sgemm/sgemm.mjs, src/dgemm/dgemm.mjs, src/classes/GpuMatrix.mjs) reaches
 * the CUDA library through this file, and only through the C ABI of
 * include/wgblas.h. The JavaScript shim in js/ keeps the reference's argument
 * validation and messages; this layer checks types and sizes again before any
 * pointer reaches the library.
 *
 * Asynchrony: every operation that queues GPU work returns a Promise. The work
 * (copies, kernels) is queued on the device handle's stream, followed by
 * cudaLaunchHostFunc; that host function (on a CUDA thread) hands the pending
 * operation to the device's napi_threadsafe_function, whose call_js callback
 * runs on the JavaScript thread, checks the device's error word, builds the
 * result and resolves (or rejects) the promise. Host arrays are copied into
 * page-locked staging memory before anything is queued, so the caller's typed
 * arrays are not referenced after the call returns; results come back through
 * staging into new typed arrays (the reference's sgemm returns a new C).
 *
 * Node-API (https://nodejs.org/api/n-api.html) is a stable C ABI exported by the
 * node binary. node_api.h is not part of this build's toolchain, so the types,
 * enum values and functions used here are declared below as documented; the
 * addon's undefined napi_* symbols resolve against the node process at load.
 * Build: gcc -shared -fPIC -O2 -Iinclude -I<cuda>/include wgblas_napi.c
 *        -Lwgblas_b200 -lwgblas_b200 -L<cuda>/lib64 -lcudart -o wgblas_napi.node
 * (wgblas_b200/build.py does this). */
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "wgblas.h"

/* ---- Node-API declarations (js_native_api.h / node_api.h, NAPI_VERSION 8) ---- */

typedef struct napi_env__ *napi_env;
typedef struct napi_value__ *napi_value;
typedef struct napi_ref__ *napi_ref;
typedef struct napi_callback_info__ *napi_callback_info;
typedef struct napi_deferred__ *napi_deferred;
typedef struct napi_threadsafe_function__ *napi_threadsafe_function;

typedef enum {
  napi_ok,
  napi_invalid_arg,
  napi_object_expected,
  napi_string_expected,
  napi_name_expected,
  napi_function_expected,
  napi_number_expected,
  napi_boolean_expected,
  napi_array_expected,
  napi_generic_failure,
  napi_pending_exception,
  napi_cancelled,
  napi_escape_called_twice,
  napi_handle_scope_mismatch,
  napi_callback_scope_mismatch,
  napi_queue_full,
  napi_closing,
  napi_bigint_expected,
  napi_date_expected,
  napi_arraybuffer_expected,
  napi_detachable_arraybuffer_expected,
  napi_would_deadlock
} napi_status;

typedef enum {
  napi_undefined,
  napi_null,
  napi_boolean,
  napi_number,
  napi_string,
  napi_symbol,
  napi_object,
  napi_function,
  napi_external,
  napi_bigint
} napi_valuetype;

typedef enum {
  napi_int8_array,
  napi_uint8_array,
  napi_uint8_clamped_array,
  napi_int16_array,
  napi_uint16_array,
  napi_int32_array,
  napi_uint32_array,
  napi_float32_array,
  napi_float64_array,
  napi_bigint64_array,
  napi_biguint64_array
} napi_typedarray_type;

typedef enum { napi_tsfn_release, napi_tsfn_abort } napi_threadsafe_function_release_mode;
typedef enum { napi_tsfn_nonblocking, napi_tsfn_blocking } napi_threadsafe_function_call_mode;

typedef napi_value (*napi_callback)(napi_env env, napi_callback_info info);
typedef void (*napi_finalize)(napi_env env, void *finalize_data, void *finalize_hint);
typedef void (*napi_threadsafe_function_call_js)(napi_env env, napi_value js_callback, void *context, void *data);

typedef struct {
  const char *error_message;
  void *engine_reserved;
  uint32_t engine_error_code;
  napi_status error_code;
} napi_extended_error_info;

napi_status napi_get_cb_info(napi_env env, napi_callback_info cbinfo, size_t *argc, napi_value *argv,
                             napi_value *this_arg, void **data);
napi_status napi_create_function(napi_env env, const char *utf8name, size_t length, napi_callback cb, void *data,
                                 napi_value *result);
napi_status napi_set_named_property(napi_env env, napi_value object, const char *utf8name, napi_value value);
napi_status napi_create_object(napi_env env, napi_value *result);
napi_status napi_get_undefined(napi_env env, napi_value *result);
napi_status napi_get_null(napi_env env, napi_value *result);
napi_status napi_typeof(napi_env env, napi_value value, napi_valuetype *result);
napi_status napi_get_value_double(napi_env env, napi_value value, double *result);
napi_status napi_get_value_int32(napi_env env, napi_value value, int32_t *result);
napi_status napi_get_value_int64(napi_env env, napi_value value, int64_t *result);
napi_status napi_get_value_bool(napi_env env, napi_value value, bool *result);
napi_status napi_create_double(napi_env env, double value, napi_value *result);
napi_status napi_create_int32(napi_env env, int32_t value, napi_value *result);
napi_status napi_create_int64(napi_env env, int64_t value, napi_value *result);
napi_status napi_create_string_utf8(napi_env env, const char *str, size_t length, napi_value *result);
napi_status napi_create_external(napi_env env, void *data, napi_finalize finalize_cb, void *finalize_hint,
                                 napi_value *result);
napi_status napi_get_value_external(napi_env env, napi_value value, void **result);
napi_status napi_is_typedarray(napi_env env, napi_value value, bool *result);
napi_status napi_get_typedarray_info(napi_env env, napi_value typedarray, napi_typedarray_type *type, size_t *length,
                                     void **data, napi_value *arraybuffer, size_t *byte_offset);
napi_status napi_is_arraybuffer(napi_env env, napi_value value, bool *result);
napi_status napi_get_arraybuffer_info(napi_env env, napi_value arraybuffer, void **data, size_t *byte_length);
napi_status napi_create_arraybuffer(napi_env env, size_t byte_length, void **data, napi_value *result);
napi_status napi_create_typedarray(napi_env env, napi_typedarray_type type, size_t length, napi_value arraybuffer,
                                   size_t byte_offset, napi_value *result);
napi_status napi_create_promise(napi_env env, napi_deferred *deferred, napi_value *promise);
napi_status napi_resolve_deferred(napi_env env, napi_deferred deferred, napi_value resolution);
napi_status napi_reject_deferred(napi_env env, napi_deferred deferred, napi_value rejection);
napi_status napi_create_error(napi_env env, napi_value code, napi_value msg, napi_value *result);
napi_status napi_throw_error(napi_env env, const char *code, const char *msg);
napi_status napi_throw_type_error(napi_env env, const char *code, const char *msg);
napi_status napi_is_exception_pending(napi_env env, bool *result);
napi_status napi_get_last_error_info(napi_env env, const napi_extended_error_info **result);
napi_status napi_create_threadsafe_function(napi_env env, napi_value func, napi_value async_resource,
                                            napi_value async_resource_name, size_t max_queue_size,
                                            size_t initial_thread_count, void *thread_finalize_data,
                                            napi_finalize thread_finalize_cb, void *context,
                                            napi_threadsafe_function_call_js call_js_cb,
                                            napi_threadsafe_function *result);
napi_status napi_call_threadsafe_function(napi_threadsafe_function func, void *data,
                                          napi_threadsafe_function_call_mode is_blocking);
napi_status napi_release_threadsafe_function(napi_threadsafe_function func,
                                             napi_threadsafe_function_release_mode mode);
napi_status napi_ref_threadsafe_function(napi_env env, napi_threadsafe_function func);
napi_status napi_unref_threadsafe_function(napi_env env, napi_threadsafe_function func);

/* ---- status plumbing ---------------------------------------------------------- */

/* Throws a JavaScript Error for a failed Node-API call unless one is pending. */
static void throw_napi(napi_env env, napi_status st, const char *what) {
  bool pending = false;
  if (napi_is_exception_pending(env, &pending) == napi_ok && pending) return;
  const napi_extended_error_info *info = NULL;
  char msg[256];
  if (napi_get_last_error_info(env, &info) == napi_ok && info && info->error_message)
    snprintf(msg, sizeof msg, "wgblas addon: %s failed: %s", what, info->error_message);
  else
    snprintf(msg, sizeof msg, "wgblas addon: %s failed (napi_status %d)", what, (int)st);
  napi_throw_error(env, NULL, msg);
}

#define NAPI_CALL(env, call)                    \
  do {                                          \
    napi_status st_ = (call);                   \
    if (st_ != napi_ok) {                       \
      throw_napi((env), st_, #call);            \
      return NULL;                              \
    }                                           \
  } while (0)

/* Throws the library's message for a failed C-ABI call. */
static napi_value throw_wg(napi_env env, wg_status st, const char *what) {
  char msg[1200];
  snprintf(msg, sizeof msg, "%s: %s (wg_status %d)", what, wg_last_error(), (int)st);
  napi_throw_error(env, NULL, msg);
  return NULL;
}

#define WG_CALL(env, call)                                   \
  do {                                                       \
    wg_status wst_ = (call);                                 \
    if (wst_ != WG_OK) return throw_wg((env), wst_, #call); \
  } while (0)

static napi_value undefined_value(napi_env env) {
  napi_value u = NULL;
  if (napi_get_undefined(env, &u) != napi_ok) return NULL;
  return u;
}

/* ---- argument readers (each throws a TypeError and returns false on a bad value) ---- */

static bool arg_int64(napi_env env, napi_value v, const char *name, int64_t *out) {
  napi_valuetype t;
  double d;
  char msg[128];
  if (napi_typeof(env, v, &t) != napi_ok || t != napi_number || napi_get_value_double(env, v, &d) != napi_ok ||
      d != d || d < -9007199254740991.0 || d > 9007199254740991.0 || (double)(int64_t)d != d) {
    snprintf(msg, sizeof msg, "%s must be an integer.", name);
    napi_throw_type_error(env, NULL, msg);
    return false;
  }
  *out = (int64_t)d;
  return true;
}

static bool arg_double(napi_env env, napi_value v, const char *name, double *out) {
  napi_valuetype t;
  char msg[128];
  if (napi_typeof(env, v, &t) != napi_ok || t != napi_number || napi_get_value_double(env, v, out) != napi_ok) {
    snprintf(msg, sizeof msg, "%s must be a number.", name);
    napi_throw_type_error(env, NULL, msg);
    return false;
  }
  return true;
}

static bool arg_bool(napi_env env, napi_value v, const char *name, bool *out) {
  napi_valuetype t;
  char msg[128];
  if (napi_typeof(env, v, &t) != napi_ok || t != napi_boolean || napi_get_value_bool(env, v, out) != napi_ok) {
    snprintf(msg, sizeof msg, "%s must be a boolean.", name);
    napi_throw_type_error(env, NULL, msg);
    return false;
  }
  return true;
}

/* A typed array of the given element type: its data pointer and length in elements. */
static bool arg_typed(napi_env env, napi_value v, const char *name, napi_typedarray_type want, void **data,
                      size_t *length) {
  bool is = false;
  napi_typedarray_type t;
  napi_value ab;
  size_t off;
  char msg[128];
  if (napi_is_typedarray(env, v, &is) != napi_ok || !is ||
      napi_get_typedarray_info(env, v, &t, length, data, &ab, &off) != napi_ok || t != want) {
    snprintf(msg, sizeof msg, "%s must be a %s.", name, want == napi_float64_array ? "Float64Array" : "Float32Array");
    napi_throw_type_error(env, NULL, msg);
    return false;
  }
  return true;
}

/* ---- handles ------------------------------------------------------------------- */

/* One device handle and the threadsafe function its completions go through. */
typedef struct Device {
  uint32_t magic;
  wg_device *dev;
  cudaStream_t stream;
  napi_threadsafe_function tsfn;
  int64_t pending;  /* operations queued and not yet completed (keeps the event loop alive) */
  bool closed;
} Device;

typedef struct Buffer {
  uint32_t magic;
  wg_buffer *buf;
  size_t bytes;
  Device *owner;
} Buffer;

typedef struct Comm {
  uint32_t magic;
  wg_comm *comm;
  Device *owner;
} Comm;

enum { MAGIC_DEVICE = 0x57474456u, MAGIC_BUFFER = 0x57474246u, MAGIC_COMM = 0x5747434du };

static bool arg_device(napi_env env, napi_value v, Device **out) {
  void *p = NULL;
  if (napi_get_value_external(env, v, &p) != napi_ok || !p || ((Device *)p)->magic != MAGIC_DEVICE) {
    napi_throw_type_error(env, NULL, "device must be a GPUDevice.");
    return false;
  }
  if (((Device *)p)->closed) {
    napi_throw_error(env, NULL, "device has been destroyed — call init() again.");
    return false;
  }
  *out = (Device *)p;
  return true;
}

static bool arg_buffer(napi_env env, napi_value v, const char *name, Buffer **out) {
  void *p = NULL;
  char msg[128];
  if (napi_get_value_external(env, v, &p) != napi_ok || !p || ((Buffer *)p)->magic != MAGIC_BUFFER) {
    snprintf(msg, sizeof msg, "%s must be a device buffer.", name);
    napi_throw_type_error(env, NULL, msg);
    return false;
  }
  if (!((Buffer *)p)->buf) {
    snprintf(msg, sizeof msg, "%s has been destroyed.", name);
    napi_throw_error(env, NULL, msg);
    return false;
  }
  *out = (Buffer *)p;
  return true;
}

/* ---- pending operations -------------------------------------------------------- */

typedef enum { OP_VOID, OP_TYPED, OP_GEMM } OpKind;

/* An operation queued on a device stream, completed on the JavaScript thread. */
typedef struct Op {
  Device *d;
  napi_deferred deferred;
  OpKind kind;
  /* staging (page-locked) host memory and device temporaries freed on completion */
  void *stage_in[3];
  void *stage_out;
  size_t out_bytes;
  napi_typedarray_type out_type;
  size_t out_length;
  wg_buffer *temps[3];
  /* timing (benchmark devices) */
  cudaEvent_t ev0, ev1;
  bool timed;
  char error[512];  /* set when queuing failed after the promise was created */
} Op;

static void op_free(Op *op) {
  for (int i = 0; i < 3; i++) {
    if (op->stage_in[i]) wg_host_free(op->stage_in[i]);
    if (op->temps[i]) wg_buffer_free(op->temps[i]);
  }
  if (op->stage_out) wg_host_free(op->stage_out);
  if (op->ev0) cudaEventDestroy(op->ev0);
  if (op->ev1) cudaEventDestroy(op->ev1);
  free(op);
}

static void reject_with(napi_env env, napi_deferred deferred, const char *message) {
  napi_value msg, err;
  if (napi_create_string_utf8(env, message, strlen(message), &msg) == napi_ok &&
      napi_create_error(env, NULL, msg, &err) == napi_ok)
    napi_reject_deferred(env, deferred, err);
}

/* Runs on the JavaScript thread: settles the operation's promise. */
static void call_js(napi_env env, napi_value js_cb, void *context, void *data) {
  (void)js_cb;
  (void)context;
  Op *op = (Op *)data;
  if (!env) {  /* the threadsafe function is being torn down: nothing to settle */
    op_free(op);
    return;
  }
  Device *d = op->d;
  if (--d->pending == 0) napi_unref_threadsafe_function(env, d->tsfn);
  wg_status st = op->error[0] ? WG_ERR_CUDA : wg_device_check(d->dev);
  if (st != WG_OK) {
    char msg[1200];
    snprintf(msg, sizeof msg, "%s", op->error[0] ? op->error : wg_last_error());
    reject_with(env, op->deferred, msg);
    op_free(op);
    return;
  }
  napi_value result = NULL, obj = NULL;
  bool ok = true;
  if (op->kind == OP_TYPED || op->kind == OP_GEMM) {
    ok = napi_create_object(env, &obj) == napi_ok;
    if (ok && op->stage_out) {
      void *data_out = NULL;
      napi_value ab, ta;
      ok = napi_create_arraybuffer(env, op->out_bytes, &data_out, &ab) == napi_ok &&
           napi_create_typedarray(env, op->out_type, op->out_length, ab, 0, &ta) == napi_ok;
      if (ok) {
        memcpy(data_out, op->stage_out, op->out_bytes);
        ok = napi_set_named_property(env, obj, op->kind == OP_GEMM ? "C" : "data", ta) == napi_ok;
      }
    }
    if (ok && op->timed) {
      float ms = 0.0f;
      napi_value v;
      ok = cudaEventElapsedTime(&ms, op->ev0, op->ev1) == cudaSuccess &&
           napi_create_double(env, (double)ms, &v) == napi_ok &&
           napi_set_named_property(env, obj, "gpuTimeMs", v) == napi_ok;
    }
    result = obj;
  } else {
    ok = napi_get_undefined(env, &result) == napi_ok;
  }
  if (ok)
    napi_resolve_deferred(env, op->deferred, result);
  else
    reject_with(env, op->deferred, "wgblas addon: building the result failed");
  op_free(op);
}

/* Runs on a CUDA thread once the work queued before it has finished. Makes no
 * CUDA call (a host function may not). */
static void CUDART_CB on_stream_done(void *data) {
  Op *op = (Op *)data;
  napi_call_threadsafe_function(op->d->tsfn, op, napi_tsfn_nonblocking);
}

/* A new operation with its promise (returned through *promise). */
static Op *op_new(napi_env env, Device *d, OpKind kind, napi_value *promise) {
  Op *op = (Op *)calloc(1, sizeof(Op));
  if (!op) {
    napi_throw_error(env, NULL, "wgblas addon: out of host memory");
    return NULL;
  }
  op->d = d;
  op->kind = kind;
  if (napi_create_promise(env, &op->deferred, promise) != napi_ok) {
    free(op);
    throw_napi(env, napi_generic_failure, "napi_create_promise");
    return NULL;
  }
  return op;
}

/* Queues the completion behind everything on the device stream. If queuing
 * failed (error set), the promise is rejected on the next turn of the loop. */
static napi_value op_submit(napi_env env, Op *op, napi_value promise, const char *error) {
  Device *d = op->d;
  if (d->pending++ == 0 && napi_ref_threadsafe_function(env, d->tsfn) != napi_ok) {
    d->pending--;
    reject_with(env, op->deferred, "wgblas addon: napi_ref_threadsafe_function failed");
    op_free(op);
    return promise;
  }
  if (error) snprintf(op->error, sizeof op->error, "%s", error);
  if (op->timed && !error) cudaEventRecord(op->ev1, d->stream);
  if (error || cudaLaunchHostFunc(d->stream, on_stream_done, op) != cudaSuccess) {
    if (!op->error[0]) snprintf(op->error, sizeof op->error, "wgblas addon: cudaLaunchHostFunc failed");
    /* settle through the same path, from this thread */
    if (napi_call_threadsafe_function(d->tsfn, op, napi_tsfn_nonblocking) != napi_ok) {
      d->pending--;
      reject_with(env, op->deferred, op->error);
      op_free(op);
    }
  }
  return promise;
}

/* ---- devices: src/init.mjs:31-143 ------------------------------------------------ */

static napi_value js_device_count(napi_env env, napi_callback_info info) {
  (void)info;
  int n = 0;
  WG_CALL(env, wg_device_count(&n));
  napi_value v;
  NAPI_CALL(env, napi_create_int32(env, n, &v));
  return v;
}

static void finalize_device(napi_env env, void *data, void *hint) {
  (void)env;
  (void)hint;
  Device *d = (Device *)data;
  if (!d->closed) {
    d->closed = true;
    wg_device_close(d->dev);
    napi_release_threadsafe_function(d->tsfn, napi_tsfn_release);
  }
  d->magic = 0;
  free(d);
}

/* deviceOpen(ordinal, benchmark) -> device */
static napi_value js_device_open(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  int64_t ordinal;
  bool bench;
  if (argc < 2 || !arg_int64(env, argv[0], "ordinal", &ordinal) || !arg_bool(env, argv[1], "benchmark", &bench))
    return NULL;
  Device *d = (Device *)calloc(1, sizeof(Device));
  if (!d) {
    napi_throw_error(env, NULL, "wgblas addon: out of host memory");
    return NULL;
  }
  wg_status st = wg_device_open((int)ordinal, bench ? WG_DEVICE_TIMING : 0u, &d->dev);
  if (st != WG_OK) {
    free(d);
    return throw_wg(env, st, "wg_device_open");
  }
  void *stream = NULL;
  if ((st = wg_device_stream(d->dev, &stream)) != WG_OK) {
    wg_device_close(d->dev);
    free(d);
    return throw_wg(env, st, "wg_device_stream");
  }
  d->stream = (cudaStream_t)stream;
  napi_value name;
  napi_status ns = napi_create_string_utf8(env, "wgblas-completion", 17, &name);
  if (ns == napi_ok)
    ns = napi_create_threadsafe_function(env, NULL, NULL, name, 0, 1, NULL, NULL, NULL, call_js, &d->tsfn);
  if (ns == napi_ok) ns = napi_unref_threadsafe_function(env, d->tsfn);  /* idle devices do not keep node alive */
  if (ns != napi_ok) {
    wg_device_close(d->dev);
    free(d);
    throw_napi(env, ns, "creating the device's threadsafe function");
    return NULL;
  }
  d->magic = MAGIC_DEVICE;
  napi_value ext;
  ns = napi_create_external(env, d, finalize_device, NULL, &ext);
  if (ns != napi_ok) {
    napi_release_threadsafe_function(d->tsfn, napi_tsfn_release);
    wg_device_close(d->dev);
    free(d);
    throw_napi(env, ns, "napi_create_external");
    return NULL;
  }
  return ext;
}

/* deviceClose(device): waits for its work, releases the handle (cleanup()). */
static napi_value js_device_close(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  void *p = NULL;
  if (argc < 1 || napi_get_value_external(env, argv[0], &p) != napi_ok || !p ||
      ((Device *)p)->magic != MAGIC_DEVICE) {
    napi_throw_type_error(env, NULL, "device must be a GPUDevice.");
    return NULL;
  }
  Device *d = (Device *)p;
  if (!d->closed) {
    d->closed = true;
    wg_device_sync(d->dev);
    wg_device_close(d->dev);
    NAPI_CALL(env, napi_release_threadsafe_function(d->tsfn, napi_tsfn_release));
  }
  return undefined_value(env);
}

/* deviceInfo(device) -> {name, ordinal, smCount, architecture, totalMemory, benchmark} (gpuName/getAdapter). */
static napi_value js_device_info(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  if (argc < 1 || !arg_device(env, argv[0], &d)) return NULL;
  char name[256];
  WG_CALL(env, wg_device_name(d->dev, name, sizeof name));
  wg_device_props p;
  WG_CALL(env, wg_device_props_get(d->dev, &p));
  char arch[32];
  snprintf(arch, sizeof arch, "sm_%d%d", p.cc_major, p.cc_minor);
  napi_value obj, v;
  NAPI_CALL(env, napi_create_object(env, &obj));
  NAPI_CALL(env, napi_create_string_utf8(env, name, strlen(name), &v));
  NAPI_CALL(env, napi_set_named_property(env, obj, "name", v));
  NAPI_CALL(env, napi_create_int32(env, p.ordinal, &v));
  NAPI_CALL(env, napi_set_named_property(env, obj, "ordinal", v));
  NAPI_CALL(env, napi_create_int32(env, p.sm_count, &v));
  NAPI_CALL(env, napi_set_named_property(env, obj, "smCount", v));
  NAPI_CALL(env, napi_create_string_utf8(env, arch, strlen(arch), &v));
  NAPI_CALL(env, napi_set_named_property(env, obj, "architecture", v));
  NAPI_CALL(env, napi_create_double(env, (double)p.total_mem, &v));
  NAPI_CALL(env, napi_set_named_property(env, obj, "totalMemory", v));
  NAPI_CALL(env, napi_create_int32(env, (int32_t)((p.flags & WG_DEVICE_TIMING) != 0), &v));
  NAPI_CALL(env, napi_set_named_property(env, obj, "benchmark", v));
  return obj;
}

/* ---- buffers: the storage of GpuMatrix / GpuVector (src/classes/GpuMatrix.mjs:43-207) ---- */

static void finalize_buffer(napi_env env, void *data, void *hint) {
  (void)env;
  (void)hint;
  Buffer *b = (Buffer *)data;
  /* a buffer the program dropped without destroy(): free it if its device lives */
  if (b->buf && b->owner && !b->owner->closed) wg_buffer_free(b->buf);
  b->magic = 0;
  free(b);
}

/* bufferAlloc(device, bytes) -> buffer */
static napi_value js_buffer_alloc(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  int64_t bytes;
  if (argc < 2 || !arg_device(env, argv[0], &d) || !arg_int64(env, argv[1], "bytes", &bytes)) return NULL;
  if (bytes <= 0) {
    napi_throw_error(env, NULL, "bytes must be positive.");
    return NULL;
  }
  Buffer *b = (Buffer *)calloc(1, sizeof(Buffer));
  if (!b) {
    napi_throw_error(env, NULL, "wgblas addon: out of host memory");
    return NULL;
  }
  wg_status st = wg_buffer_alloc(d->dev, (size_t)bytes, &b->buf);
  if (st != WG_OK) {
    free(b);
    return throw_wg(env, st, "wg_buffer_alloc");
  }
  b->magic = MAGIC_BUFFER;
  b->bytes = (size_t)bytes;
  b->owner = d;
  napi_value ext;
  napi_status ns = napi_create_external(env, b, finalize_buffer, NULL, &ext);
  if (ns != napi_ok) {
    wg_buffer_free(b->buf);
    free(b);
    throw_napi(env, ns, "napi_create_external");
    return NULL;
  }
  return ext;
}

/* bufferFree(buffer): GpuMatrix.destroy(). */
static napi_value js_buffer_free(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  void *p = NULL;
  if (argc < 1 || napi_get_value_external(env, argv[0], &p) != napi_ok || !p ||
      ((Buffer *)p)->magic != MAGIC_BUFFER) {
    napi_throw_type_error(env, NULL, "buffer must be a device buffer.");
    return NULL;
  }
  Buffer *b = (Buffer *)p;
  if (b->buf) {
    wg_buffer *buf = b->buf;
    b->buf = NULL;
    WG_CALL(env, wg_buffer_free(buf));
  }
  return undefined_value(env);
}

/* bufferUpload(device, buffer, typedArray, byteOffset) -> Promise<void>. The array
 * is copied into page-locked staging first and may be reused as soon as this returns. */
static napi_value js_buffer_upload(napi_env env, napi_callback_info info) {
  size_t argc = 4;
  napi_value argv[4];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  Buffer *b;
  int64_t off;
  bool is = false;
  if (argc < 4 || !arg_device(env, argv[0], &d) || !arg_buffer(env, argv[1], "buffer", &b) ||
      !arg_int64(env, argv[3], "byteOffset", &off))
    return NULL;
  napi_typedarray_type t;
  size_t len = 0, aoff = 0;
  void *src = NULL;
  napi_value ab;
  NAPI_CALL(env, napi_is_typedarray(env, argv[2], &is));
  if (!is) {
    napi_throw_type_error(env, NULL, "data must be a Float32Array or Float64Array.");
    return NULL;
  }
  NAPI_CALL(env, napi_get_typedarray_info(env, argv[2], &t, &len, &src, &ab, &aoff));
  if (t != napi_float32_array && t != napi_float64_array) {
    napi_throw_type_error(env, NULL, "data must be a Float32Array or Float64Array.");
    return NULL;
  }
  const size_t bytes = len * (t == napi_float64_array ? 8 : 4);
  if (off < 0 || (size_t)off > b->bytes || bytes > b->bytes - (size_t)off) {
    napi_throw_error(env, NULL, "upload exceeds the buffer.");
    return NULL;
  }
  napi_value promise;
  Op *op = op_new(env, d, OP_VOID, &promise);
  if (!op) return NULL;
  const char *error = NULL;
  void *dptr = NULL;
  if (bytes) {
    if (wg_host_alloc(bytes, &op->stage_in[0]) != WG_OK || wg_buffer_device_ptr(b->buf, &dptr) != WG_OK)
      error = wg_last_error();
    else {
      memcpy(op->stage_in[0], src, bytes);
      if (cudaMemcpyAsync((char *)dptr + off, op->stage_in[0], bytes, cudaMemcpyHostToDevice, d->stream) !=
          cudaSuccess)
        error = "cudaMemcpyAsync (upload) failed";
    }
  }
  return op_submit(env, op, promise, error);
}

/* bufferRead(device, buffer, byteOffset, elementBytes, rows, cols, ld) -> Promise<{data}>:
 * the `rows` runs of `cols` elements, `ld` elements apart, as one dense typed
 * array (GpuMatrix.read() strips lda padding this way; elementBytes 4 or 8). */
static napi_value js_buffer_read(napi_env env, napi_callback_info info) {
  size_t argc = 7;
  napi_value argv[7];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  Buffer *b;
  int64_t off, eb, rows, cols, ld;
  if (argc < 7 || !arg_device(env, argv[0], &d) || !arg_buffer(env, argv[1], "buffer", &b) ||
      !arg_int64(env, argv[2], "byteOffset", &off) || !arg_int64(env, argv[3], "elementBytes", &eb) ||
      !arg_int64(env, argv[4], "rows", &rows) || !arg_int64(env, argv[5], "cols", &cols) ||
      !arg_int64(env, argv[6], "ld", &ld))
    return NULL;
  if ((eb != 4 && eb != 8) || rows < 1 || cols < 1 || ld < cols || off < 0) {
    napi_throw_error(env, NULL, "bufferRead: invalid shape.");
    return NULL;
  }
  const size_t need = (size_t)off + ((size_t)(rows - 1) * (size_t)ld + (size_t)cols) * (size_t)eb;
  if (need > b->bytes) {
    napi_throw_error(env, NULL, "read exceeds the buffer.");
    return NULL;
  }
  napi_value promise;
  Op *op = op_new(env, d, OP_TYPED, &promise);
  if (!op) return NULL;
  op->out_bytes = (size_t)rows * (size_t)cols * (size_t)eb;
  op->out_type = eb == 8 ? napi_float64_array : napi_float32_array;
  op->out_length = (size_t)rows * (size_t)cols;
  const char *error = NULL;
  void *dptr = NULL;
  if (wg_host_alloc(op->out_bytes, &op->stage_out) != WG_OK || wg_buffer_device_ptr(b->buf, &dptr) != WG_OK)
    error = wg_last_error();
  else if (cudaMemcpy2DAsync(op->stage_out, (size_t)cols * eb, (char *)dptr + off, (size_t)ld * eb,
                             (size_t)cols * eb, (size_t)rows, cudaMemcpyDeviceToHost, d->stream) != cudaSuccess)
    error = "cudaMemcpy2DAsync (read) failed";
  return op_submit(env, op, promise, error);
}

/* ---- GEMM: src/sgemm/sgemm.mjs:151-262, src/dgemm/dgemm.mjs (column-major frame) ---- */

typedef struct GemmArgs {
  int transA, transB;
  int64_t m, n, k, lda, ldb, ldc;
  double alpha, beta;
} GemmArgs;

/* transA, transB, m, n, k, alpha at argv[1..6]; lda, ldb, beta, ldc at the given slots. */
static bool read_gemm_args(napi_env env, napi_value *argv, int ilda, int ildb, int ibeta, int ildc, GemmArgs *g) {
  int64_t ta, tb;
  if (!arg_int64(env, argv[1], "transA", &ta) || !arg_int64(env, argv[2], "transB", &tb) ||
      !arg_int64(env, argv[3], "m", &g->m) || !arg_int64(env, argv[4], "n", &g->n) ||
      !arg_int64(env, argv[5], "k", &g->k) || !arg_double(env, argv[6], "alpha", &g->alpha) ||
      !arg_int64(env, argv[ilda], "lda", &g->lda) || !arg_int64(env, argv[ildb], "ldb", &g->ldb) ||
      !arg_double(env, argv[ibeta], "beta", &g->beta) || !arg_int64(env, argv[ildc], "ldc", &g->ldc))
    return false;
  g->transA = (int)ta;
  g->transB = (int)tb;
  return true;
}

static bool timing_start(Device *d, Op *op) {
  wg_device_props p;
  if (wg_device_props_get(d->dev, &p) != WG_OK || !(p.flags & WG_DEVICE_TIMING)) return true;
  if (cudaEventCreate(&op->ev0) != cudaSuccess || cudaEventCreate(&op->ev1) != cudaSuccess) return false;
  op->timed = cudaEventRecord(op->ev0, d->stream) == cudaSuccess;
  return op->timed;
}

/* gemm(device, transA, transB, m, n, k, alpha, A, offA, lda, B, offB, ldb, beta, C, offC, ldc, f64)
 * on device buffers (offsets in elements) -> Promise<{gpuTimeMs?}>; C is updated in place. */
static napi_value js_gemm(napi_env env, napi_callback_info info) {
  size_t argc = 18;
  napi_value argv[18];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  Buffer *A, *B, *C;
  GemmArgs g;
  int64_t oa, ob, oc;
  bool f64;
  if (argc < 18 || !arg_device(env, argv[0], &d) || !read_gemm_args(env, argv, 9, 12, 13, 16, &g) ||
      !arg_buffer(env, argv[7], "A", &A) || !arg_int64(env, argv[8], "offA", &oa) ||
      !arg_buffer(env, argv[10], "B", &B) || !arg_int64(env, argv[11], "offB", &ob) ||
      !arg_buffer(env, argv[14], "C", &C) || !arg_int64(env, argv[15], "offC", &oc) ||
      !arg_bool(env, argv[17], "f64", &f64))
    return NULL;
  napi_value promise;
  Op *op = op_new(env, d, OP_GEMM, &promise);
  if (!op) return NULL;
  const char *error = NULL;
  if (!timing_start(d, op)) error = "cudaEventRecord failed";
  wg_status st = WG_OK;
  if (!error)
    st = f64 ? wg_dgemm(d->dev, g.transA, g.transB, g.m, g.n, g.k, g.alpha, A->buf, oa, g.lda, B->buf, ob, g.ldb,
                        g.beta, C->buf, oc, g.ldc, NULL)
             : wg_sgemm(d->dev, g.transA, g.transB, g.m, g.n, g.k, (float)g.alpha, A->buf, oa, g.lda, B->buf, ob,
                        g.ldb, (float)g.beta, C->buf, oc, g.ldc, NULL);
  if (st != WG_OK) error = wg_last_error();
  return op_submit(env, op, promise, error);
}

/* Rows x cols of a column-major matrix stored with leading dimension ld. */
static size_t span_elems(int64_t rows, int64_t cols, int64_t ld) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)((cols - 1) * ld + rows);
}

/* gemmHost(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, f64)
 * on typed arrays -> Promise<{C, gpuTimeMs?}>: a new C (the input C is not
 * modified). Operands go through page-locked staging into stream-ordered device
 * temporaries; the kernels, the read-back and the completion follow on the
 * device stream. */
static napi_value js_gemm_host(napi_env env, napi_callback_info info) {
  size_t argc = 15;
  napi_value argv[15];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  GemmArgs g;
  bool f64;
  if (argc < 15 || !arg_device(env, argv[0], &d) || !read_gemm_args(env, argv, 8, 10, 11, 13, &g) ||
      !arg_bool(env, argv[14], "f64", &f64))
    return NULL;
  const napi_typedarray_type tt = f64 ? napi_float64_array : napi_float32_array;
  const size_t es = f64 ? 8 : 4;
  void *hA, *hB, *hC;
  size_t nA, nB, nC;
  if (!arg_typed(env, argv[7], "A", tt, &hA, &nA) || !arg_typed(env, argv[9], "B", tt, &hB, &nB) ||
      !arg_typed(env, argv[12], "C", tt, &hC, &nC))
    return NULL;
  if (g.m < 0 || g.n < 0 || g.k < 0 || g.lda <= 0 || g.ldb <= 0 || g.ldc <= 0 || g.ldc < g.m ||
      g.lda < (g.transA ? g.k : g.m) || g.ldb < (g.transB ? g.n : g.k)) {
    napi_throw_error(env, NULL, "gemmHost: invalid dimensions.");
    return NULL;
  }
  const size_t sa = g.transA ? span_elems(g.k, g.m, g.lda) : span_elems(g.m, g.k, g.lda);
  const size_t sb = g.transB ? span_elems(g.n, g.k, g.ldb) : span_elems(g.k, g.n, g.ldb);
  const size_t sc = span_elems(g.m, g.n, g.ldc);
  if (nA < sa || nB < sb || nC < sc) {
    napi_throw_error(env, NULL, "gemmHost: an operand does not have enough elements.");
    return NULL;
  }
  napi_value promise;
  Op *op = op_new(env, d, OP_GEMM, &promise);
  if (!op) return NULL;
  op->out_type = tt;
  op->out_length = nC;
  op->out_bytes = nC * es;
  const char *error = NULL;
  /* the whole of C comes back (its padding as it was), A and B as far as they are read */
  const size_t bytes[3] = {(sa ? sa : 1) * es, (sb ? sb : 1) * es, (nC ? nC : 1) * es};
  const void *src[3] = {hA, hB, hC};
  const size_t used[3] = {sa * es, sb * es, nC * es};
  void *dp[3] = {NULL, NULL, NULL};
  for (int i = 0; i < 3 && !error; i++) {
    if (wg_host_alloc(bytes[i], &op->stage_in[i]) != WG_OK || wg_buffer_alloc_async(d->dev, bytes[i], &op->temps[i]) != WG_OK ||
        wg_buffer_device_ptr(op->temps[i], &dp[i]) != WG_OK) {
      error = wg_last_error();
      break;
    }
    memcpy(op->stage_in[i], src[i], used[i]);
    if (used[i] && cudaMemcpyAsync(dp[i], op->stage_in[i], used[i], cudaMemcpyHostToDevice, d->stream) != cudaSuccess)
      error = "cudaMemcpyAsync (operands) failed";
  }
  if (!error && wg_host_alloc(op->out_bytes ? op->out_bytes : 1, &op->stage_out) != WG_OK) error = wg_last_error();
  if (!error && !timing_start(d, op)) error = "cudaEventRecord failed";
  if (!error) {
    wg_status st = f64 ? wg_dgemm(d->dev, g.transA, g.transB, g.m, g.n, g.k, g.alpha, op->temps[0], 0, g.lda,
                                  op->temps[1], 0, g.ldb, g.beta, op->temps[2], 0, g.ldc, NULL)
                       : wg_sgemm(d->dev, g.transA, g.transB, g.m, g.n, g.k, (float)g.alpha, op->temps[0], 0, g.lda,
                                  op->temps[1], 0, g.ldb, (float)g.beta, op->temps[2], 0, g.ldc, NULL);
    if (st != WG_OK) error = wg_last_error();
  }
  if (!error && op->out_bytes &&
      cudaMemcpyAsync(op->stage_out, dp[2], op->out_bytes, cudaMemcpyDeviceToHost, d->stream) != cudaSuccess)
    error = "cudaMemcpyAsync (result) failed";
  return op_submit(env, op, promise, error);
}

/* ---- multi-GPU: wg_comm_* and the sharded GEMM ------------------------------------ */

/* commUniqueId() -> ArrayBuffer of WG_COMM_ID_BYTES bytes (made on rank 0, shared out of band). */
static napi_value js_comm_unique_id(napi_env env, napi_callback_info info) {
  (void)info;
  void *data = NULL;
  napi_value ab;
  NAPI_CALL(env, napi_create_arraybuffer(env, WG_COMM_ID_BYTES, &data, &ab));
  WG_CALL(env, wg_comm_unique_id((unsigned char *)data, WG_COMM_ID_BYTES));
  return ab;
}

static void finalize_comm(napi_env env, void *data, void *hint) {
  (void)env;
  (void)hint;
  Comm *c = (Comm *)data;
  if (c->comm && c->owner && !c->owner->closed) wg_comm_destroy(c->comm);
  c->magic = 0;
  free(c);
}

/* commInitRank(device, nranks, rank, idArrayBuffer, timeoutMs) -> communicator */
static napi_value js_comm_init_rank(napi_env env, napi_callback_info info) {
  size_t argc = 5;
  napi_value argv[5];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Device *d;
  int64_t nranks, rank, timeout;
  bool is = false;
  if (argc < 5 || !arg_device(env, argv[0], &d) || !arg_int64(env, argv[1], "nranks", &nranks) ||
      !arg_int64(env, argv[2], "rank", &rank) || !arg_int64(env, argv[4], "timeoutMs", &timeout))
    return NULL;
  void *id = NULL;
  size_t idlen = 0;
  NAPI_CALL(env, napi_is_arraybuffer(env, argv[3], &is));
  if (!is) {
    napi_throw_type_error(env, NULL, "id must be an ArrayBuffer from commUniqueId().");
    return NULL;
  }
  NAPI_CALL(env, napi_get_arraybuffer_info(env, argv[3], &id, &idlen));
  Comm *c = (Comm *)calloc(1, sizeof(Comm));
  if (!c) {
    napi_throw_error(env, NULL, "wgblas addon: out of host memory");
    return NULL;
  }
  wg_status st = wg_comm_init_rank(d->dev, (int)nranks, (int)rank, (const unsigned char *)id, idlen, (int)timeout,
                                   &c->comm);
  if (st != WG_OK) {
    free(c);
    return throw_wg(env, st, "wg_comm_init_rank");
  }
  c->magic = MAGIC_COMM;
  c->owner = d;
  napi_value ext;
  napi_status ns = napi_create_external(env, c, finalize_comm, NULL, &ext);
  if (ns != napi_ok) {
    wg_comm_destroy(c->comm);
    free(c);
    throw_napi(env, ns, "napi_create_external");
    return NULL;
  }
  return ext;
}

static bool arg_comm(napi_env env, napi_value v, Comm **out) {
  void *p = NULL;
  if (napi_get_value_external(env, v, &p) != napi_ok || !p || ((Comm *)p)->magic != MAGIC_COMM || !((Comm *)p)->comm) {
    napi_throw_type_error(env, NULL, "comm must be a live communicator.");
    return false;
  }
  *out = (Comm *)p;
  return true;
}

/* commDestroy(comm) */
static napi_value js_comm_destroy(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Comm *c;
  if (argc < 1 || !arg_comm(env, argv[0], &c)) return NULL;
  wg_comm *cm = c->comm;
  c->comm = NULL;
  WG_CALL(env, wg_comm_destroy(cm));
  return undefined_value(env);
}

/* gemmSharded(comm, transA, transB, mLocal, n, k, alpha, A, lda, B|null, ldb, root, beta, C, ldc,
 * panelCols, f64) on this rank's device buffers -> Promise<void> (every rank calls it). */
static napi_value js_gemm_sharded(napi_env env, napi_callback_info info) {
  size_t argc = 17;
  napi_value argv[17];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  Comm *c;
  Buffer *A, *C, *B = NULL;
  int64_t ta, tb, ml, n, k, lda, ldb, root, ldc, panel;
  double alpha, beta;
  bool f64;
  napi_valuetype bt;
  if (argc < 17 || !arg_comm(env, argv[0], &c) || !arg_int64(env, argv[1], "transA", &ta) ||
      !arg_int64(env, argv[2], "transB", &tb) || !arg_int64(env, argv[3], "mLocal", &ml) ||
      !arg_int64(env, argv[4], "n", &n) || !arg_int64(env, argv[5], "k", &k) ||
      !arg_double(env, argv[6], "alpha", &alpha) || !arg_buffer(env, argv[7], "A", &A) ||
      !arg_int64(env, argv[8], "lda", &lda) || !arg_int64(env, argv[10], "ldb", &ldb) ||
      !arg_int64(env, argv[11], "root", &root) || !arg_double(env, argv[12], "beta", &beta) ||
      !arg_buffer(env, argv[13], "C", &C) || !arg_int64(env, argv[14], "ldc", &ldc) ||
      !arg_int64(env, argv[15], "panelCols", &panel) || !arg_bool(env, argv[16], "f64", &f64))
    return NULL;
  NAPI_CALL(env, napi_typeof(env, argv[9], &bt));
  if (bt != napi_null && bt != napi_undefined && !arg_buffer(env, argv[9], "B", &B)) return NULL;
  void *pa = NULL, *pb = NULL, *pc = NULL;
  WG_CALL(env, wg_buffer_device_ptr(A->buf, &pa));
  WG_CALL(env, wg_buffer_device_ptr(C->buf, &pc));
  if (B) WG_CALL(env, wg_buffer_device_ptr(B->buf, &pb));
  napi_value promise;
  Op *op = op_new(env, c->owner, OP_VOID, &promise);
  if (!op) return NULL;
  wg_status st = f64 ? wg_dgemm_sharded(c->comm, (int)ta, (int)tb, ml, n, k, alpha, (const double *)pa, lda,
                                        (double *)pb, ldb, (int)root, beta, (double *)pc, ldc, panel)
                     : wg_sgemm_sharded(c->comm, (int)ta, (int)tb, ml, n, k, (float)alpha, (const float *)pa, lda,
                                        (float *)pb, ldb, (int)root, (float)beta, (float *)pc, ldc, panel);
  return op_submit(env, op, promise, st == WG_OK ? NULL : wg_last_error());
}

/* ---- seeded inputs: src/random/random.mjs:4-26 ---------------------------------- */

/* randomArray(n, low, high, seed, f64) -> Float32Array | Float64Array (mulberry32) */
static napi_value js_random_array(napi_env env, napi_callback_info info) {
  size_t argc = 5;
  napi_value argv[5];
  NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  int64_t n, seed;
  double low, high;
  bool f64;
  if (argc < 5 || !arg_int64(env, argv[0], "n", &n) || !arg_double(env, argv[1], "low", &low) ||
      !arg_double(env, argv[2], "high", &high) || !arg_int64(env, argv[3], "seed", &seed) ||
      !arg_bool(env, argv[4], "f64", &f64))
    return NULL;
  if (n < 0) {
    napi_throw_error(env, NULL, "n must be non-negative.");
    return NULL;
  }
  void *data = NULL;
  napi_value ab, ta;
  NAPI_CALL(env, napi_create_arraybuffer(env, (size_t)n * (f64 ? 8 : 4), &data, &ab));
  if (f64)
    wg_random_f64((double *)data, n, low, high, (uint32_t)seed);
  else
    wg_random_f32((float *)data, n, low, high, (uint32_t)seed);
  NAPI_CALL(env, napi_create_typedarray(env, f64 ? napi_float64_array : napi_float32_array, (size_t)n, ab, 0, &ta));
  return ta;
}

/* ---- module registration ----------------------------------------------------------- */

typedef struct {
  const char *name;
  napi_callback fn;
} Export;

static const Export kExports[] = {
    {"deviceCount", js_device_count},     {"deviceOpen", js_device_open},
    {"deviceClose", js_device_close},     {"deviceInfo", js_device_info},
    {"bufferAlloc", js_buffer_alloc},     {"bufferFree", js_buffer_free},
    {"bufferUpload", js_buffer_upload},   {"bufferRead", js_buffer_read},
    {"gemm", js_gemm},                    {"gemmHost", js_gemm_host},
    {"commUniqueId", js_comm_unique_id},  {"commInitRank", js_comm_init_rank},
    {"commDestroy", js_comm_destroy},     {"gemmSharded", js_gemm_sharded},
    {"randomArray", js_random_array},
};

__attribute__((visibility("default"))) napi_value napi_register_module_v1(napi_env env, napi_value exports) {
  for (size_t i = 0; i < sizeof kExports / sizeof kExports[0]; i++) {
    napi_value fn;
    NAPI_CALL(env, napi_create_function(env, kExports[i].name, strlen(kExports[i].name), kExports[i].fn, NULL, &fn));
    NAPI_CALL(env, napi_set_named_property(env, exports, kExports[i].name, fn));
  }
  napi_value v;
  NAPI_CALL(env, napi_create_int32(env, wg_abi_version(), &v));
  NAPI_CALL(env, napi_set_named_property(env, exports, "abiVersion", v));
  return exports;
}

/* The Node-API version this addon was written against (Node reads it at load). */
__attribute__((visibility("default"))) int32_t node_api_module_get_api_version_v1(void) { return 8; }
