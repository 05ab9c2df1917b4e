// Prepared-model store: the read side of the `cheetah init` layout.
//
// Mirrors `MmapWeightStore::open` / `slice` (`src/chat/native/store.rs:74-213`):
// cheetah_units.json lists each unit's dtype, shape, byte count, shard file
// and payload offset (relative to the shard's data section, which starts at
// 8 + the little-endian u64 header length). Shards are memory-mapped once.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace cheetah {

struct UnitRecord {
    std::string unit_id;
    std::string dtype;            // "BF16", "F16", "F32", ...
    std::vector<uint64_t> shape;
    uint64_t bytes = 0;
    std::string source_file;
    uint64_t source_offset = 0;
    int layer_id = 0;
};

class MappedFile {
  public:
    ~MappedFile();
    bool open(const std::string &path, std::string *error);
    const uint8_t *data() const { return data_; }
    size_t size() const { return size_; }

  private:
    const uint8_t *data_ = nullptr;
    size_t size_ = 0;
};

class PreparedStore {
  public:
    // Returns false and fills *error on a missing/invalid manifest or shard.
    bool open(const std::string &root, std::string *error);
    bool contains(const std::string &unit_id) const { return units_.count(unit_id) != 0; }
    const UnitRecord *record(const std::string &unit_id) const;
    std::vector<std::string> unit_ids() const {
        std::vector<std::string> ids;
        for (const auto &kv : units_) ids.push_back(kv.first);
        return ids;
    }
    // Byte view of one unit inside its shard mapping (nullptr + error if absent).
    const uint8_t *slice(const std::string &unit_id, std::string *error) const;

  private:
    struct Shard {
        std::unique_ptr<MappedFile> file;
        size_t data_start = 0;
    };
    std::map<std::string, UnitRecord> units_;
    std::map<std::string, Shard> shards_;
};

}  // namespace cheetah
