// planning.cpp -- host-side planning that needs no device: error names, the
// ubatch partition, the FFN skip mask and the bound-gating config keys.
#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "epsp_host.h"

namespace edge_prefill_b200 {

// Same names and numbering as edge_prefill::error_code_name (src/status.cpp:5-22).
const char* error_code_name(ErrorCode code) {
    switch (code) {
        case ErrorCode::Ok: return "Ok";
        case ErrorCode::InvalidArgument: return "InvalidArgument";
        case ErrorCode::ModelLoad: return "ModelLoad";
        case ErrorCode::Tokenize: return "Tokenize";
        case ErrorCode::ContextInit: return "ContextInit";
        case ErrorCode::Prefill: return "Prefill";
        case ErrorCode::Decode: return "Decode";
        case ErrorCode::Cache: return "Cache";
        case ErrorCode::Unsupported: return "Unsupported";
        case ErrorCode::OutOfMemory: return "OutOfMemory";
        case ErrorCode::Io: return "Io";
        case ErrorCode::Internal: return "Internal";
        case ErrorCode::Unavailable: return "Unavailable";
    }
    return "Unknown";
}

void log_warn(const std::string& msg) {
    if (std::getenv("EPSP_QUIET") == nullptr) std::fprintf(stderr, "[epsp] warn: %s\n", msg.c_str());
}

// src/chunk_scheduler.cpp:9-45: chunk 0 = one n_ubatch-aligned range per
// ubatch; an explicit chunk >= n_tokens is a single range; otherwise the
// chunk is clamped to n_ubatch.
Status ChunkScheduler::plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch, std::vector<Range>* out) {
    if (!out) return Status::error(ErrorCode::InvalidArgument, "null chunk output");
    if (n_tokens == 0) return Status::error(ErrorCode::InvalidArgument, "n_tokens must be > 0");
    if (n_ubatch == 0) return Status::error(ErrorCode::InvalidArgument, "n_ubatch must be > 0");
    out->clear();
    if (chunk_size != 0 && chunk_size >= n_tokens) {
        out->push_back(Range{0, n_tokens});
        return Status::success();
    }
    uint32_t step = chunk_size == 0 ? n_ubatch : chunk_size;
    if (step > n_ubatch) {
        log_warn("chunk_size " + std::to_string(step) + " exceeds n_ubatch " + std::to_string(n_ubatch) +
                 "; clamping to n_ubatch");
        step = n_ubatch;
    }
    step = std::max<uint32_t>(1, std::min(step, n_tokens));
    for (uint32_t b = 0; b < n_tokens; b += step) out->push_back(Range{b, std::min(n_tokens, b + step)});
    return Status::success();
}

namespace {

bool parse_i32_strict(const std::string& text, int32_t* out) {
    if (text.empty()) return false;
    char* end = nullptr;
    errno = 0;
    const long v = std::strtol(text.c_str(), &end, 10);
    if (errno != 0 || end != text.c_str() + text.size()) return false;
    *out = static_cast<int32_t>(v);
    return true;
}

std::string strip_spaces(const std::string& s) {
    std::string r;
    for (char c : s)
        if (!std::isspace(static_cast<unsigned char>(c))) r.push_back(c);
    return r;
}

}  // namespace

// src/ffn_skip.cpp:41-60: round(ratio * n_layer) layers spread evenly,
// layer i * (n_layer / count).
Status FfnSkipController::auto_mask(int32_t n_layer, double ratio, uint64_t* out) {
    if (!out) return Status::error(ErrorCode::InvalidArgument, "null mask output");
    if (n_layer <= 0 || n_layer > 64) return Status::error(ErrorCode::InvalidArgument, "n_layer must be in (0,64]");
    if (!(ratio >= 0.0 && ratio <= 1.0)) return Status::error(ErrorCode::InvalidArgument, "ratio must be in [0,1]");
    const int32_t count = static_cast<int32_t>(std::llround(ratio * n_layer));
    uint64_t mask = 0;
    if (count > 0) {
        const double step = static_cast<double>(n_layer) / count;
        for (int32_t i = 0; i < count; ++i) {
            const int32_t layer = std::min(n_layer - 1, static_cast<int32_t>(i * step));
            mask |= uint64_t(1) << layer;
        }
    }
    *out = mask;
    return Status::success();
}

// src/ffn_skip.cpp:62-117: "N%" delegates to auto_mask; otherwise a comma list
// of layers and inclusive ranges (reversed ranges are swapped); whitespace is
// ignored; layers >= n_layer are dropped with the warning
// "mask-bit-out-of-range".
Status FfnSkipController::parse(const std::string& spec, int32_t n_layer, uint64_t* out, std::string* warning) {
    if (!out) return Status::error(ErrorCode::InvalidArgument, "null mask output");
    if (n_layer <= 0 || n_layer > 64) return Status::error(ErrorCode::InvalidArgument, "n_layer must be in (0,64]");
    if (spec.empty()) return Status::error(ErrorCode::InvalidArgument, "empty mask spec");
    if (warning) warning->clear();
    if (spec.back() == '%') {
        const std::string num = spec.substr(0, spec.size() - 1);
        char* end = nullptr;
        const double pct = std::strtod(num.c_str(), &end);
        if (num.empty() || end == num.c_str()) return Status::error(ErrorCode::InvalidArgument, "invalid percentage mask");
        return auto_mask(n_layer, pct / 100.0, out);
    }
    uint64_t mask = 0;
    size_t start = 0;
    while (true) {
        const size_t comma = spec.find(',', start);
        const std::string part = strip_spaces(spec.substr(start, comma == std::string::npos ? std::string::npos : comma - start));
        if (part.empty()) return Status::error(ErrorCode::InvalidArgument, "empty mask component");
        const size_t dash = part.find('-');
        int32_t lo = 0, hi = 0;
        if (dash == std::string::npos) {
            if (!parse_i32_strict(part, &lo)) return Status::error(ErrorCode::InvalidArgument, "invalid mask token: " + part);
            hi = lo;
        } else {
            if (!parse_i32_strict(part.substr(0, dash), &lo) || !parse_i32_strict(part.substr(dash + 1), &hi))
                return Status::error(ErrorCode::InvalidArgument, "invalid mask range: " + part);
            if (hi < lo) std::swap(lo, hi);
        }
        if (lo < 0) return Status::error(ErrorCode::InvalidArgument, "negative layer index");
        for (int32_t layer = lo; layer <= hi; ++layer) {
            if (layer >= n_layer || layer >= 64) {
                if (warning) *warning = "mask-bit-out-of-range";
                continue;
            }
            mask |= uint64_t(1) << layer;
        }
        if (comma == std::string::npos) break;
        start = comma + 1;
    }
    *out = mask;
    return Status::success();
}

}  // namespace edge_prefill_b200

using namespace edge_prefill_b200;

namespace {

std::string trim(const std::string& s) {
    size_t a = 0, b = s.size();
    while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
    while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
    return s.substr(a, b - a);
}

bool parse_bool_value(const std::string& v, int32_t* out) {
    if (v == "1" || v == "true" || v == "yes" || v == "on") {
        *out = 1;
        return true;
    }
    if (v == "0" || v == "false" || v == "no" || v == "off") {
        *out = 0;
        return true;
    }
    return false;
}

bool parse_u64_value(const std::string& v, uint64_t* out) {
    if (v.empty() || v[0] == '-' || v[0] == '+') return false;
    char* end = nullptr;
    errno = 0;
    const unsigned long long x = std::strtoull(v.c_str(), &end, 10);
    if (errno != 0 || end != v.c_str() + v.size()) return false;
    *out = x;
    return true;
}

}  // namespace

extern "C" {

const char* ep_sp_error_name(int32_t code) { return error_code_name(static_cast<ErrorCode>(code)); }

int32_t ep_sp_chunk_plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch, uint32_t* ranges, int32_t cap,
                         int32_t* n_out) {
    std::vector<Range> r;
    const Status st = ChunkScheduler::plan(n_tokens, chunk_size, n_ubatch, &r);
    if (!st.ok()) return static_cast<int32_t>(st.code);
    if (n_out) *n_out = static_cast<int32_t>(r.size());
    for (size_t i = 0; ranges && i < r.size() && static_cast<int32_t>(i) < cap; ++i) {
        ranges[2 * i] = r[i].begin;
        ranges[2 * i + 1] = r[i].end;
    }
    return 0;
}

int32_t ep_sp_ffn_auto_mask(int32_t n_layer, double ratio, uint64_t* out) {
    return static_cast<int32_t>(FfnSkipController::auto_mask(n_layer, ratio, out).code);
}

int32_t ep_sp_ffn_parse(const char* spec, int32_t n_layer, uint64_t* out, char* warning, int32_t cap) {
    std::string w;
    const Status st = FfnSkipController::parse(spec ? std::string(spec) : std::string(), n_layer, out, &w);
    if (warning && cap > 0) {
        std::strncpy(warning, w.c_str(), static_cast<size_t>(cap - 1));
        warning[cap - 1] = 0;
    }
    return static_cast<int32_t>(st.code);
}

// src/config.cpp:173-215 line grammar ('#' comments, "key = value", a line
// without '=' is an error) and :527-538 for the four bound-gating keys.
int32_t ep_sp_parse_config(const char* path, ep_sp_prefill_options* out) {
    if (!path || !out) return static_cast<int32_t>(ErrorCode::InvalidArgument);
    std::ifstream f(path);
    if (!f) return static_cast<int32_t>(ErrorCode::Io);
    ep_sp_prefill_options o = *out;
    std::string line;
    while (std::getline(f, line)) {
        const size_t hash = line.find('#');
        if (hash != std::string::npos) line = line.substr(0, hash);
        line = trim(line);
        if (line.empty()) continue;
        const size_t eq = line.find('=');
        if (eq == std::string::npos) return static_cast<int32_t>(ErrorCode::InvalidArgument);
        const std::string key = trim(line.substr(0, eq));
        const std::string value = trim(line.substr(eq + 1));
        uint64_t u = 0;
        int32_t b = 0;
        if (key == "qg_bound") {
            if (!parse_bool_value(value, &b)) return static_cast<int32_t>(ErrorCode::InvalidArgument);
            o.enable_qg_bound = b;
        } else if (key == "qg_sel_pages") {
            if (!parse_u64_value(value, &u) || u > 128) return static_cast<int32_t>(ErrorCode::InvalidArgument);
            o.qg_sel_pages = static_cast<uint32_t>(u);
        } else if (key == "qg_local_rows") {
            if (!parse_u64_value(value, &u) || u > 32768) return static_cast<int32_t>(ErrorCode::InvalidArgument);
            o.qg_local_rows = static_cast<uint32_t>(u);
        } else if (key == "qg_pool_pages") {
            if (!parse_u64_value(value, &u) || u > 4096) return static_cast<int32_t>(ErrorCode::InvalidArgument);
            o.qg_pool_pages = static_cast<uint32_t>(u);
        }
    }
    *out = o;
    return 0;
}

}  // extern "C"
