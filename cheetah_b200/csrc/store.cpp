// Prepared-model store (see store.h). A small JSON reader covers the units
// manifest grammar written by `cheetah_init.c:1668-1716` (an array of flat
// objects with string, integer and integer-array fields).
#include "store.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

namespace cheetah {

MappedFile::~MappedFile() {
    if (data_ != nullptr) munmap(const_cast<uint8_t *>(data_), size_);
}

bool MappedFile::open(const std::string &path, std::string *error) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        *error = "Failed to open " + path + ": " + std::strerror(errno);
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        *error = "Failed to stat " + path;
        ::close(fd);
        return false;
    }
    size_ = static_cast<size_t>(st.st_size);
    if (size_ == 0) {
        ::close(fd);
        data_ = nullptr;
        return true;
    }
    void *map = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map == MAP_FAILED) {
        *error = "Failed to map " + path;
        size_ = 0;
        return false;
    }
    data_ = static_cast<const uint8_t *>(map);
    return true;
}

namespace {

class Json {
  public:
    explicit Json(const std::string &text) : s_(text), i_(0) {}

    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    bool eat(char c) {
        ws();
        if (i_ < s_.size() && s_[i_] == c) {
            ++i_;
            return true;
        }
        return false;
    }
    bool peek(char c) {
        ws();
        return i_ < s_.size() && s_[i_] == c;
    }
    bool string(std::string *out) {
        ws();
        if (i_ >= s_.size() || s_[i_] != '"') return false;
        ++i_;
        out->clear();
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\' && i_ < s_.size()) {
                char e = s_[i_++];
                switch (e) {
                case 'n': out->push_back('\n'); break;
                case 't': out->push_back('\t'); break;
                case 'r': out->push_back('\r'); break;
                case 'b': out->push_back('\b'); break;
                case 'f': out->push_back('\f'); break;
                case 'u':
                    if (i_ + 4 <= s_.size()) {
                        unsigned code = std::strtoul(s_.substr(i_, 4).c_str(), nullptr, 16);
                        i_ += 4;
                        if (code < 0x80) out->push_back(static_cast<char>(code));
                        else out->push_back('?');
                    }
                    break;
                default: out->push_back(e);
                }
            } else {
                out->push_back(c);
            }
        }
        if (i_ >= s_.size()) return false;
        ++i_;
        return true;
    }
    bool number(double *out) {
        ws();
        const char *start = s_.c_str() + i_;
        char *end = nullptr;
        *out = std::strtod(start, &end);
        if (end == start) return false;
        i_ += static_cast<size_t>(end - start);
        return true;
    }
    // Skip any JSON value.
    bool skip() {
        ws();
        if (i_ >= s_.size()) return false;
        char c = s_[i_];
        if (c == '"') {
            std::string tmp;
            return string(&tmp);
        }
        if (c == '{' || c == '[') {
            char close = c == '{' ? '}' : ']';
            ++i_;
            if (eat(close)) return true;
            for (;;) {
                if (c == '{') {
                    std::string key;
                    if (!string(&key) || !eat(':')) return false;
                }
                if (!skip()) return false;
                if (eat(',')) continue;
                return eat(close);
            }
        }
        if (std::strncmp(s_.c_str() + i_, "true", 4) == 0) { i_ += 4; return true; }
        if (std::strncmp(s_.c_str() + i_, "false", 5) == 0) { i_ += 5; return true; }
        if (std::strncmp(s_.c_str() + i_, "null", 4) == 0) { i_ += 4; return true; }
        double d;
        return number(&d);
    }

  private:
    const std::string &s_;
    size_t i_;
};

bool parse_unit(Json &j, UnitRecord *unit) {
    if (!j.eat('{')) return false;
    if (j.eat('}')) return true;
    for (;;) {
        std::string key;
        if (!j.string(&key) || !j.eat(':')) return false;
        if (key == "unit_id") {
            if (!j.string(&unit->unit_id)) return false;
        } else if (key == "dtype") {
            if (!j.string(&unit->dtype)) return false;
        } else if (key == "source_file") {
            if (!j.string(&unit->source_file)) return false;
        } else if (key == "bytes" || key == "source_offset" || key == "layer_id") {
            double v;
            if (!j.number(&v)) return false;
            if (key == "bytes") unit->bytes = static_cast<uint64_t>(v);
            else if (key == "source_offset") unit->source_offset = static_cast<uint64_t>(v);
            else unit->layer_id = static_cast<int>(v);
        } else if (key == "shape") {
            if (!j.eat('[')) return false;
            if (!j.eat(']')) {
                for (;;) {
                    double v;
                    if (!j.number(&v)) return false;
                    unit->shape.push_back(static_cast<uint64_t>(v));
                    if (j.eat(',')) continue;
                    if (!j.eat(']')) return false;
                    break;
                }
            }
        } else {
            if (!j.skip()) return false;
        }
        if (j.eat(',')) continue;
        return j.eat('}');
    }
}

}  // namespace

bool PreparedStore::open(const std::string &root, std::string *error) {
    const std::string manifest_path = root + "/cheetah_units.json";
    std::ifstream in(manifest_path, std::ios::binary);
    if (!in) {
        *error = "Failed to read " + manifest_path;
        return false;
    }
    std::stringstream buffer;
    buffer << in.rdbuf();
    const std::string text = buffer.str();
    Json j(text);
    std::vector<UnitRecord> records;
    if (!j.eat('[')) {
        *error = "Invalid Ant units manifest: expected an array";
        return false;
    }
    if (!j.eat(']')) {
        for (;;) {
            UnitRecord unit;
            if (!parse_unit(j, &unit)) {
                *error = "Invalid Ant units manifest: malformed unit record";
                return false;
            }
            records.push_back(std::move(unit));
            if (j.eat(',')) continue;
            if (!j.eat(']')) {
                *error = "Invalid Ant units manifest: unterminated array";
                return false;
            }
            break;
        }
    }
    if (records.empty()) {
        *error = "Ant units manifest is empty; run `cheetah init` first.";
        return false;
    }
    const std::string weights = root + "/.cheetah/weights/";
    for (UnitRecord &unit : records) {
        if (unit.unit_id.empty() || unit.source_file.empty()) continue;
        auto it = shards_.find(unit.source_file);
        if (it == shards_.end()) {
            Shard shard;
            shard.file = std::make_unique<MappedFile>();
            if (!shard.file->open(weights + unit.source_file, error)) return false;
            if (shard.file->size() < 8) {
                *error = "Shard " + unit.source_file + " is too small for a header.";
                return false;
            }
            uint64_t header_len = 0;
            std::memcpy(&header_len, shard.file->data(), 8);
            shard.data_start = 8 + static_cast<size_t>(header_len);
            if (shard.data_start > shard.file->size()) {
                *error = "Shard " + unit.source_file + " header exceeds the file size.";
                return false;
            }
            it = shards_.emplace(unit.source_file, std::move(shard)).first;
        }
        if (unit.source_offset + unit.bytes > it->second.file->size()) {
            *error = "Unit " + unit.unit_id + " exceeds the bounds of shard " + unit.source_file + ".";
            return false;
        }
        units_[unit.unit_id] = unit;
    }
    return true;
}

const UnitRecord *PreparedStore::record(const std::string &unit_id) const {
    auto it = units_.find(unit_id);
    return it == units_.end() ? nullptr : &it->second;
}

const uint8_t *PreparedStore::slice(const std::string &unit_id, std::string *error) const {
    auto it = units_.find(unit_id);
    if (it == units_.end()) {
        *error = "Native backend: unknown unit '" + unit_id + "'.";
        return nullptr;
    }
    const UnitRecord &unit = it->second;
    const Shard &shard = shards_.at(unit.source_file);
    const size_t start = shard.data_start + unit.source_offset;
    if (start + unit.bytes > shard.file->size()) {
        *error = "Native backend: unit '" + unit_id + "' is out of bounds.";
        return nullptr;
    }
    return shard.file->data() + start;
}

}  // namespace cheetah
