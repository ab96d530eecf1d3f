// Compile-check stub for the N-API shim (test infrastructure): the subset of
// Node's public N-API declarations that nemotron-webgpu-decode_b200/napi/nwd_napi.cc
// uses, so that tests/test_napi_shim.py can compile the shim with g++ where no
// Node.js headers are installed.  Not a working N-API.
#pragma once
#include <cstddef>
#include <cstdint>
typedef struct napi_env__* napi_env;
typedef struct napi_value__* napi_value;
typedef struct napi_callback_info__* napi_callback_info;
typedef enum { napi_ok } napi_status;
typedef enum { napi_int8_array, napi_uint8_array, napi_uint8_clamped_array, napi_int16_array, napi_uint16_array, napi_int32_array, napi_uint32_array, napi_float32_array } napi_typedarray_type;
typedef enum { napi_default = 0 } napi_property_attributes;
typedef napi_value (*napi_callback)(napi_env, napi_callback_info);
typedef void (*napi_finalize)(napi_env, void*, void*);
typedef struct { const char* utf8name; napi_value name; napi_callback method; napi_callback getter; napi_callback setter; napi_value value; napi_property_attributes attributes; void* data; } napi_property_descriptor;
napi_status napi_throw_error(napi_env, const char*, const char*);
napi_status napi_throw_type_error(napi_env, const char*, const char*);
napi_status napi_throw_range_error(napi_env, const char*, const char*);
napi_status napi_get_value_external(napi_env, napi_value, void**);
napi_status napi_has_named_property(napi_env, napi_value, const char*, bool*);
napi_status napi_get_named_property(napi_env, napi_value, const char*, napi_value*);
napi_status napi_get_value_uint32(napi_env, napi_value, uint32_t*);
napi_status napi_get_value_int64(napi_env, napi_value, int64_t*);
napi_status napi_get_cb_info(napi_env, napi_callback_info, size_t*, napi_value*, napi_value*, void**);
napi_status napi_create_external(napi_env, void*, napi_finalize, void*, napi_value*);
napi_status napi_get_typedarray_info(napi_env, napi_value, napi_typedarray_type*, size_t*, void**, napi_value*, size_t*);
napi_status napi_create_buffer_copy(napi_env, size_t, const void*, void**, napi_value*);
napi_status napi_get_buffer_info(napi_env, napi_value, void**, size_t*);
napi_status napi_define_properties(napi_env, napi_value, size_t, const napi_property_descriptor*);
#define NODE_GYP_MODULE_NAME nwd
#define NAPI_MODULE(name, init) extern "C" napi_value nwd_napi_init(napi_env e, napi_value x) { return init(e, x); }
