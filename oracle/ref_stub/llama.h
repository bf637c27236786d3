/* Minimal declarations so the reference's host-side headers (backend.h)
 * compile without llama.cpp; none of these types is used by the functions the
 * oracle shim calls.  Test infrastructure only. */
#pragma once
#include <stdint.h>
struct llama_context;
struct llama_model;
struct llama_vocab;
struct llama_model_params { int32_t unused; };
typedef int32_t llama_token;
typedef int32_t llama_pos;
