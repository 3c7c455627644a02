// Safetensors checkpoints straight into device memory: the file format of src/files/safetensors_file.cpp (an 8-byte
// little-endian header length, a JSON header mapping tensor names to {dtype, shape, data_offsets}, optional
// "__metadata__" of string values, then the tensor bytes), parsed with the same checks and messages, and each
// tensor the model uses copied from the memory-mapped file to its device slot -- no host copy of the whole file.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "cppinf_b200.h"
#include "decoder.h"
#include "runtime.h"

namespace rt = cppinf::runtime;

namespace {

// A JSON value of the subset a safetensors header uses (objects, arrays, strings, numbers, literals).
struct Json {
    enum class Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = Kind::kNull;
    bool integer = false;
    long long int_value = 0;
    std::string text;
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> members;
};

class JsonParser {
  public:
    JsonParser(const char* data, std::size_t size) : p_(data), end_(data + size) {}

    bool parse(Json* out, std::string* error) {
        if (!value(out, 0)) {
            *error = error_.empty() ? "unexpected character" : error_;
            return false;
        }
        skip();
        if (p_ != end_) {
            *error = "trailing characters after the header object";
            return false;
        }
        return true;
    }

  private:
    void skip() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) {
            ++p_;
        }
    }

    bool value(Json* out, int depth) {
        if (depth > 64) {
            error_ = "nesting too deep";
            return false;
        }
        skip();
        if (p_ >= end_) {
            error_ = "unexpected end of input";
            return false;
        }
        const char c = *p_;
        if (c == '{') {
            return object(out, depth);
        }
        if (c == '[') {
            return array(out, depth);
        }
        if (c == '"') {
            out->kind = Json::Kind::kString;
            return string(&out->text);
        }
        if (c == '-' || (c >= '0' && c <= '9')) {
            return number(out);
        }
        return literal(out);
    }

    bool object(Json* out, int depth) {
        out->kind = Json::Kind::kObject;
        ++p_;
        skip();
        if (p_ < end_ && *p_ == '}') {
            ++p_;
            return true;
        }
        while (true) {
            skip();
            std::string key;
            if (p_ >= end_ || *p_ != '"' || !string(&key)) {
                error_ = error_.empty() ? "expected a string key" : error_;
                return false;
            }
            skip();
            if (p_ >= end_ || *p_ != ':') {
                error_ = "expected ':'";
                return false;
            }
            ++p_;
            Json v;
            if (!value(&v, depth + 1)) {
                return false;
            }
            out->members.emplace_back(std::move(key), std::move(v));
            skip();
            if (p_ < end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            error_ = "expected ',' or '}'";
            return false;
        }
    }

    bool array(Json* out, int depth) {
        out->kind = Json::Kind::kArray;
        ++p_;
        skip();
        if (p_ < end_ && *p_ == ']') {
            ++p_;
            return true;
        }
        while (true) {
            Json v;
            if (!value(&v, depth + 1)) {
                return false;
            }
            out->items.push_back(std::move(v));
            skip();
            if (p_ < end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            error_ = "expected ',' or ']'";
            return false;
        }
    }

    bool string(std::string* out) {
        ++p_;  // opening quote
        while (p_ < end_ && *p_ != '"') {
            if (*p_ == '\\') {
                ++p_;
                if (p_ >= end_) {
                    break;
                }
                switch (*p_) {
                case '"':
                case '\\':
                case '/':
                    out->push_back(*p_);
                    break;
                case 'b':
                    out->push_back('\b');
                    break;
                case 'f':
                    out->push_back('\f');
                    break;
                case 'n':
                    out->push_back('\n');
                    break;
                case 'r':
                    out->push_back('\r');
                    break;
                case 't':
                    out->push_back('\t');
                    break;
                case 'u': {
                    if (end_ - p_ < 5) {
                        error_ = "truncated \\u escape";
                        return false;
                    }
                    unsigned cp = 0;
                    for (int i = 1; i <= 4; ++i) {
                        const char h = p_[i];
                        cp <<= 4;
                        if (h >= '0' && h <= '9') {
                            cp |= static_cast<unsigned>(h - '0');
                        } else if (h >= 'a' && h <= 'f') {
                            cp |= static_cast<unsigned>(h - 'a' + 10);
                        } else if (h >= 'A' && h <= 'F') {
                            cp |= static_cast<unsigned>(h - 'A' + 10);
                        } else {
                            error_ = "bad \\u escape";
                            return false;
                        }
                    }
                    p_ += 4;
                    // UTF-8 of a basic-plane code point (surrogate pairs are kept as two 3-byte sequences).
                    if (cp < 0x80) {
                        out->push_back(static_cast<char>(cp));
                    } else if (cp < 0x800) {
                        out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
                        out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
                    } else {
                        out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
                        out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
                        out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
                    }
                    break;
                }
                default:
                    error_ = "bad escape";
                    return false;
                }
                ++p_;
                continue;
            }
            out->push_back(*p_++);
        }
        if (p_ >= end_) {
            error_ = "unterminated string";
            return false;
        }
        ++p_;  // closing quote
        return true;
    }

    bool number(Json* out) {
        out->kind = Json::Kind::kNumber;
        const char* start = p_;
        if (*p_ == '-') {
            ++p_;
        }
        bool digits = false;
        while (p_ < end_ && *p_ >= '0' && *p_ <= '9') {
            ++p_;
            digits = true;
        }
        bool fraction = false;
        if (p_ < end_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) {
            fraction = true;
            while (p_ < end_ && (std::strchr("0123456789.eE+-", *p_) != nullptr)) {
                ++p_;
            }
        }
        if (!digits) {
            error_ = "bad number";
            return false;
        }
        const std::string text(start, p_);
        out->text = text;
        if (!fraction) {
            errno = 0;
            char* endp = nullptr;
            const long long v = std::strtoll(text.c_str(), &endp, 10);
            out->integer = errno == 0 && endp != nullptr && *endp == '\0';
            out->int_value = v;
        }
        return true;
    }

    bool literal(Json* out) {
        auto match = [&](const char* word) {
            const std::size_t n = std::strlen(word);
            if (static_cast<std::size_t>(end_ - p_) >= n && std::memcmp(p_, word, n) == 0) {
                p_ += n;
                return true;
            }
            return false;
        };
        if (match("true") || match("false")) {
            out->kind = Json::Kind::kBool;
            return true;
        }
        if (match("null")) {
            out->kind = Json::Kind::kNull;
            return true;
        }
        error_ = "unexpected character";
        return false;
    }

    const char* p_;
    const char* end_;
    std::string error_;
};

struct TensorEntry {
    std::string name;
    int dtype;  // cppinf_dtype
    std::vector<int64_t> shape;
    uint64_t begin;
    uint64_t end;
};

// A read-only memory mapping of a whole file.
class MappedFile {
  public:
    ~MappedFile() {
        if (data_ != nullptr) {
            munmap(data_, size_);
        }
        if (fd_ >= 0) {
            close(fd_);
        }
    }

    int open_file(const char* path) {
        fd_ = open(path, O_RDONLY);
        if (fd_ < 0) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, std::string("Failed to open safetensors file: ") + path);
        }
        struct stat st {};
        if (fstat(fd_, &st) != 0) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, std::string("Failed to read safetensors file: ") + path);
        }
        size_ = static_cast<std::size_t>(st.st_size);
        if (size_ > 0) {
            void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
            if (m == MAP_FAILED) {
                return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, std::string("Failed to map safetensors file: ") + path);
            }
            data_ = m;
        }
        return CPPINF_OK;
    }

    const unsigned char* bytes() const { return static_cast<const unsigned char*>(data_); }
    std::size_t size() const { return size_; }

  private:
    int fd_ = -1;
    void* data_ = nullptr;
    std::size_t size_ = 0;
};

// parse_header, src/files/safetensors_file.cpp:93-157 (same checks and messages).
int parse_header(const MappedFile& file, std::vector<TensorEntry>* entries, uint64_t* data_offset) {
    if (file.size() < 8) {
        return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Safetensors files must start with an 8-byte header length.");
    }
    uint64_t header_size = 0;
    for (int i = 0; i < 8; ++i) {
        header_size |= static_cast<uint64_t>(file.bytes()[i]) << (8 * i);
    }
    if (header_size > file.size() - 8) {
        return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Safetensors header extends beyond the file size.");
    }
    *data_offset = 8 + header_size;
    Json header;
    std::string error;
    JsonParser parser(reinterpret_cast<const char*>(file.bytes() + 8), static_cast<std::size_t>(header_size));
    if (!parser.parse(&header, &error)) {
        return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Failed to parse safetensors header: " + error);
    }
    if (header.kind != Json::Kind::kObject) {
        return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Safetensors header must be a JSON object.");
    }
    const uint64_t data_size = file.size() - *data_offset;
    std::map<std::string, int> seen;
    for (const auto& [key, value] : header.members) {
        if (key == "__metadata__") {
            if (value.kind != Json::Kind::kObject) {
                return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "__metadata__ must be an object.");
            }
            for (const auto& m : value.members) {
                if (m.second.kind != Json::Kind::kString) {
                    return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "__metadata__ values must be strings.");
                }
            }
            continue;
        }
        if (value.kind != Json::Kind::kObject) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Tensor entries must be JSON objects.");
        }
        const Json* dtype = nullptr;
        const Json* shape = nullptr;
        const Json* offsets = nullptr;
        for (const auto& m : value.members) {
            if (m.first == "dtype") {
                dtype = &m.second;
            } else if (m.first == "shape") {
                shape = &m.second;
            } else if (m.first == "data_offsets") {
                offsets = &m.second;
            }
        }
        if (dtype == nullptr || shape == nullptr || offsets == nullptr) {
            return rt::fail(CPPINF_ERR_OUT_OF_RANGE, "Tensor entry '" + key + "' lacks dtype, shape or data_offsets.");
        }
        TensorEntry e{key, -1, {}, 0, 0};
        // tensors::parse_dtype accepts the two dtypes the library supports.
        if (dtype->kind == Json::Kind::kString && dtype->text == "BF16") {
            e.dtype = CPPINF_DTYPE_BF16;
        } else if (dtype->kind == Json::Kind::kString && dtype->text == "F32") {
            e.dtype = CPPINF_DTYPE_F32;
        } else {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT,
                            "Unsupported dtype: " + (dtype->kind == Json::Kind::kString ? dtype->text : "?"));
        }
        if (shape->kind != Json::Kind::kArray) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "shape must be an array.");
        }
        uint64_t elements = 1;
        for (const auto& d : shape->items) {
            if (d.kind != Json::Kind::kNumber || !d.integer) {
                return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "shape dimension must be an integer.");
            }
            if (d.int_value < 0) {
                return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Shape dimensions must be non-negative.");
            }
            e.shape.push_back(d.int_value);
            const auto dim = static_cast<uint64_t>(d.int_value);
            if (dim != 0 && elements > (UINT64_MAX / 8) / dim) {
                return rt::fail(CPPINF_ERR_OVERFLOW, "Tensor element count overflows.");
            }
            elements *= dim;
        }
        if (offsets->kind != Json::Kind::kArray || offsets->items.size() != 2 ||
            offsets->items[0].kind != Json::Kind::kNumber || !offsets->items[0].integer ||
            offsets->items[1].kind != Json::Kind::kNumber || !offsets->items[1].integer) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "data_offsets must contain exactly two integers.");
        }
        const long long b = offsets->items[0].int_value;
        const long long f = offsets->items[1].int_value;
        if (b < 0 || f < b) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "data_offsets must be non-negative and ordered.");
        }
        e.begin = static_cast<uint64_t>(b);
        e.end = static_cast<uint64_t>(f);
        const uint64_t bytes = elements * (e.dtype == CPPINF_DTYPE_BF16 ? 2 : 4);
        if (bytes != e.end - e.begin) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Tensor byte range does not match dtype and shape.");
        }
        if (e.begin > data_size || bytes > data_size - e.begin) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Tensor byte range extends beyond the file data.");
        }
        if (!seen.emplace(key, 1).second) {
            return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Duplicate tensor names are not allowed.");
        }
        entries->push_back(std::move(e));
    }
    return CPPINF_OK;
}

}  // namespace

extern "C" {

int cppinf_safetensors_info(const char* path, int64_t* tensor_count, int64_t* data_offset) {
    CPPINF_REQUIRE(path, CPPINF_ERR_INVALID_ARGUMENT, "safetensors_info received a null path.");
    MappedFile file;
    int st = file.open_file(path);
    if (st != CPPINF_OK) {
        return st;
    }
    std::vector<TensorEntry> entries;
    uint64_t offset = 0;
    st = parse_header(file, &entries, &offset);
    if (st != CPPINF_OK) {
        return st;
    }
    if (tensor_count != nullptr) {
        *tensor_count = static_cast<int64_t>(entries.size());
    }
    if (data_offset != nullptr) {
        *data_offset = static_cast<int64_t>(offset);
    }
    return rt::ok();
}

int cppinf_qwen3_load_safetensors(cppinf_qwen3* model, const char* path, int64_t* loaded) {
    CPPINF_REQUIRE(model && path, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_load_safetensors received a null pointer.");
    MappedFile file;
    int st = file.open_file(path);
    if (st != CPPINF_OK) {
        return st;
    }
    std::vector<TensorEntry> entries;
    uint64_t offset = 0;
    st = parse_header(file, &entries, &offset);
    if (st != CPPINF_OK) {
        return st;
    }
    // Every tensor the model uses must be present (validate_required_tensors, src/models/qwen3/qwen3_model.cpp:63-
    // 90); others (e.g. a tied checkpoint's lm_head.weight) are skipped.
    const int64_t required = cppinf::device::qwen3_tensor_count(model);
    int64_t count = 0;
    for (const auto& e : entries) {
        std::vector<int64_t> want;
        if (!cppinf::device::qwen3_tensor_shape(model, e.name, &want)) {
            continue;
        }
        CPPINF_REQUIRE(e.dtype == CPPINF_DTYPE_BF16, CPPINF_ERR_INVALID_ARGUMENT,
                       "Qwen3Model tensor '" + e.name + "' must be bf16.");
        // The shape checks the reference's layers apply to their weights: validate_projection_weight
        // (src/nn/qwen_common.cpp:38-49) for matrices, ops::rms_norm's weight checks (src/ops/nn_ops.cpp:150-159)
        // for norm vectors. A transposed matrix has the right byte count, so the shape itself is compared.
        if (want.size() == 2) {
            CPPINF_REQUIRE(e.shape.size() == 2, CPPINF_ERR_INVALID_ARGUMENT, e.name + " must be rank-2.");
            CPPINF_REQUIRE(e.shape == want, CPPINF_ERR_INVALID_ARGUMENT, e.name + " has an unexpected shape.");
        } else {
            CPPINF_REQUIRE(e.shape.size() == 1, CPPINF_ERR_INVALID_ARGUMENT,
                           "rms_norm requires a rank-1 weight tensor.");
            CPPINF_REQUIRE(e.shape == want, CPPINF_ERR_INVALID_ARGUMENT,
                           "rms_norm weight size must match the input last dimension.");
        }
        st = cppinf_qwen3_set_weight(model, e.name.c_str(), file.bytes() + offset + e.begin,
                                     static_cast<int64_t>(e.end - e.begin), 0);
        if (st != CPPINF_OK) {
            return st;
        }
        ++count;
    }
    if (loaded != nullptr) {
        *loaded = count;
    }
    CPPINF_REQUIRE(count == required, CPPINF_ERR_OUT_OF_RANGE, "Tensor was not found in safetensors file.");
    return rt::ok();
}

}  // extern "C"
