// Minimal stand-in for Gufo core's GGUF reader (the Gufo host runtime is not
// part of the reference repository). It declares only what config.cpp and
// weights.cpp call, so those files compile unmodified for the CPU oracle in
// oracle/_ref. TEST INFRASTRUCTURE ONLY.
#ifndef LFM3_ORACLE_STUB_GGUF_READER_HPP_
#define LFM3_ORACLE_STUB_GGUF_READER_HPP_
#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <optional>
#include <string>
#include <variant>
#include <vector>
namespace gufo::core {
// The GGML type codes the reference binds (weights.cpp:30-38).
enum class GgmlType : std::uint32_t {
  kF32 = 0,
  kF16 = 1,
  kQ8_0 = 8,
  kBF16 = 30,
};
struct GgufMetadataValue {
  std::variant<std::monostate, std::uint64_t, float, bool, std::string,
               std::vector<std::uint64_t>, std::vector<std::int64_t>,
               std::vector<std::string>>
      value;
};
struct GgufTensorInfo {
  std::vector<std::uint64_t> dimensions;
  GgmlType type{};
  std::size_t size_bytes{};
  const void* data{};
};
class GgufReader {
public:
  std::map<std::string, GgufMetadataValue> metadata;
  std::map<std::string, GgufTensorInfo> tensors;

  // Maps a GGUF file (declared for the engine drop-in's link check,
  // tests/shim/engine_shim_check.cpp, which defines a stand-in).
  static std::unique_ptr<GgufReader> OpenFile(const std::string& path,
                                              std::string* error);

  const GgufMetadataValue* FindMetadata(const std::string& key) const {
    auto it = metadata.find(key);
    return it == metadata.end() ? nullptr : &it->second;
  }
  const GgufTensorInfo* FindTensor(const std::string& name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
  }
  std::optional<std::string> GetMetadataString(const std::string& key) const {
    const auto* m = FindMetadata(key);
    if (const auto* s = m ? std::get_if<std::string>(&m->value) : nullptr)
      return *s;
    return std::nullopt;
  }
  std::optional<std::uint32_t> GetMetadataUint32(const std::string& key) const {
    const auto* m = FindMetadata(key);
    if (const auto* v = m ? std::get_if<std::uint64_t>(&m->value) : nullptr)
      return std::uint32_t(*v);
    return std::nullopt;
  }
  std::optional<float> GetMetadataFloat32(const std::string& key) const {
    const auto* m = FindMetadata(key);
    if (const auto* v = m ? std::get_if<float>(&m->value) : nullptr)
      return *v;
    return std::nullopt;
  }
  std::optional<bool> GetMetadataBool(const std::string& key) const {
    const auto* m = FindMetadata(key);
    if (const auto* v = m ? std::get_if<bool>(&m->value) : nullptr)
      return *v;
    return std::nullopt;
  }
  std::vector<std::string> GetMetadataStringArray(const std::string& key) const {
    const auto* m = FindMetadata(key);
    if (const auto* v =
            m ? std::get_if<std::vector<std::string>>(&m->value) : nullptr)
      return *v;
    return {};
  }
};
}  // namespace gufo::core
#endif
