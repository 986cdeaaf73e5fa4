// czm_parse.h -- minimal safetensors (.czm) header parser for the engine.
//
// Layout read by the reference at rust/src/safetensors.rs:287-376: an 8-byte
// little-endian header length, a JSON object mapping tensor names to
// {"dtype", "shape", "data_offsets"} plus an optional "__metadata__" object of
// strings, then the raw tensor bytes.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace czg {

struct TensorRef {
    std::string dtype;            // "I8", "I16", "I32", "U8", "U16", "U32", ...
    std::vector<int64_t> shape;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t s : shape) n *= s;
        return n;
    }
};

struct CzmFile {
    std::map<std::string, TensorRef> tensors;
    std::map<std::string, std::string> metadata;
};

// Returns an empty string on success, else the reason the bytes were rejected.
std::string parse_czm(const uint8_t *data, size_t len, CzmFile &out);

}  // namespace czg
