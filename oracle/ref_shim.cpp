// C entry points over the reference's own host-side code (compiled from its
// sources by oracle/Makefile into oracle/_ref/).  Test infrastructure only: the
// tests compare the product's ChunkScheduler / FfnSkipController mirror with
// these.  Return values are edge_prefill::ErrorCode numbers.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "edge_prefill/chunk_scheduler.h"
#include "edge_prefill/ffn_skip.h"
#include "edge_prefill/status.h"

using namespace edge_prefill;

extern "C" {

int32_t ref_chunk_plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                       uint32_t* ranges, int32_t cap, int32_t* n_out) {
    std::vector<Range> out;
    Status st = ChunkScheduler::plan(n_tokens, chunk_size, n_ubatch, &out);
    if (!st.ok()) return static_cast<int32_t>(st.code);
    *n_out = static_cast<int32_t>(out.size());
    for (size_t i = 0; i < out.size() && static_cast<int32_t>(i) < cap; ++i) {
        ranges[2 * i] = out[i].begin;
        ranges[2 * i + 1] = out[i].end;
    }
    return 0;
}

int32_t ref_ffn_auto_mask(int32_t n_layer, double ratio, uint64_t* out) {
    return static_cast<int32_t>(FfnSkipController::auto_mask(n_layer, ratio, out).code);
}

int32_t ref_ffn_parse(const char* spec, int32_t n_layer, uint64_t* out, char* warning, int32_t cap) {
    std::string w;
    Status st = FfnSkipController::parse(spec ? std::string(spec) : std::string(), n_layer, out, &w);
    if (warning && cap > 0) {
        std::strncpy(warning, w.c_str(), static_cast<size_t>(cap - 1));
        warning[cap - 1] = 0;
    }
    return static_cast<int32_t>(st.code);
}

const char* ref_error_code_name(int32_t code) {
    return error_code_name(static_cast<ErrorCode>(code));
}

}  // extern "C"
