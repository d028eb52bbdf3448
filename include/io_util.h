// io_util.h — the on-disk KV exchange format shared by the decode drivers:
// a directory holding meta.json (integer keys B, H, D, S, ...) and raw
// little-endian tensors Q.bin, K.bin, V.bin (fp16), Kq.bin / Vq.bin (int8),
// K_scales.bin / V_scales.bin (fp16), O_cuda.bin (fp16).
//
// Same three helpers, names and failure behaviour (message on stderr, exit
// code 2) as the reference (reference include/io_util.h:14-64), so its
// tqkv_decode / tqkv_bench sources compile against this include directory.
#pragma once

#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <string>

// Whole file as a string; exits with status 2 if it cannot be opened.
inline std::string tqkv_slurp(const std::string& path) {
    std::ifstream in(path, std::ios::in | std::ios::binary);
    if (!in.is_open()) {
        std::fprintf(stderr, "could not open %s\n", path.c_str());
        std::exit(2);
    }
    return std::string(std::istreambuf_iterator<char>(in),
                       std::istreambuf_iterator<char>());
}

// Integer value of `"key": <int>` in a flat JSON text.  Exits with status 2
// when the key is missing, has no ':' after it, or its value is not an
// (optionally negative) decimal integer.
inline int tqkv_read_meta_int(const std::string& json, const char* key) {
    const std::string quoted = "\"" + std::string(key) + "\"";
    const size_t at = json.find(quoted);
    if (at == std::string::npos) {
        std::fprintf(stderr, "meta.json: missing key \"%s\"\n", key);
        std::exit(2);
    }
    size_t pos = json.find(':', at + quoted.size());
    if (pos == std::string::npos) {
        std::fprintf(stderr, "meta.json: malformed near \"%s\"\n", key);
        std::exit(2);
    }
    ++pos;
    while (pos < json.size() && std::isspace(static_cast<unsigned char>(json[pos]))) ++pos;
    bool negative = false;
    if (pos < json.size() && json[pos] == '-') {
        negative = true;
        ++pos;
    }
    if (pos >= json.size() || !std::isdigit(static_cast<unsigned char>(json[pos]))) {
        std::fprintf(stderr, "meta.json: non-integer value for \"%s\"\n", key);
        std::exit(2);
    }
    int value = 0;
    for (; pos < json.size() && std::isdigit(static_cast<unsigned char>(json[pos])); ++pos) {
        value = value * 10 + (json[pos] - '0');
    }
    return negative ? -value : value;
}

// Reads exactly `bytes` bytes of `path` into `dst`; exits with status 2 if the
// file cannot be opened or is shorter.
inline void tqkv_read_bin(const std::string& path, void* dst, size_t bytes) {
    std::ifstream in(path, std::ios::in | std::ios::binary);
    if (!in.is_open()) {
        std::fprintf(stderr, "could not open %s for reading\n", path.c_str());
        std::exit(2);
    }
    in.read(static_cast<char*>(dst), static_cast<std::streamsize>(bytes));
    if (static_cast<size_t>(in.gcount()) != bytes) {
        std::fprintf(stderr, "could not read %zu bytes from %s\n", bytes, path.c_str());
        std::exit(2);
    }
}
