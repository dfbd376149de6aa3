// TinyLlama-family model config and the FP16 weight archive manifest.
//
// The manifest is the reference's text format (src/model/weight_manifest.cpp
// :461-600): `key=value` lines plus `tensor=name|offset|bytes|d0[,d1]|sha256`
// records; a data file holds the raw FP16 tensors. Validation checks the exact
// tensor set for the config (always including a separate lm_head.weight),
// shapes, byte ranges (2-byte aligned, in bounds, non-overlapping) and, for
// the data file, its length and every tensor's SHA-256. Error codes and their
// precedence follow the reference so loaders report the same failure.
#pragma once

#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

namespace kimkvcache {

struct TinyLlamaConfig final {
    std::uint32_t hidden_size{0};
    std::uint32_t intermediate_size{0};
    std::uint32_t layer_count{0};
    std::uint32_t attention_head_count{0};
    std::uint32_t kv_head_count{0};
    std::uint32_t head_dimension{0};
    std::uint32_t vocabulary_size{0};
    std::uint32_t max_position_embeddings{0};
    std::uint32_t bos_token_id{0};
    std::uint32_t eos_token_id{0};
    float rms_norm_epsilon{0.0F};
    float rope_theta{0.0F};
    bool tied_word_embeddings{false};

    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return hidden_size != 0 && intermediate_size != 0 && layer_count != 0
            && attention_head_count != 0 && kv_head_count != 0 && head_dimension != 0
            && hidden_size == attention_head_count * head_dimension
            && attention_head_count >= kv_head_count
            && attention_head_count % kv_head_count == 0 && head_dimension % 2 == 0
            && vocabulary_size != 0 && max_position_embeddings != 0
            && bos_token_id < vocabulary_size && eos_token_id < vocabulary_size
            && rms_norm_epsilon > 0.0F && rope_theta > 0.0F;
    }
};

[[nodiscard]] constexpr TinyLlamaConfig tinyLlama11bChatConfig() noexcept
{
    return TinyLlamaConfig{2048, 5632, 22, 32, 4, 64, 32000, 2048, 1, 2, 1.0e-5F, 10000.0F, false};
}

enum class WeightManifestError : std::uint8_t {
    None,
    InvalidArgument,
    FileOpenFailed,
    ParseFailed,
    UnsupportedVersion,
    UnsupportedDataType,
    InvalidConfig,
    InvalidTensor,
    DuplicateTensor,
    MissingTensor,
    UnexpectedTensor,
    DataFileMismatch,
    ChecksumMismatch,
};

struct WeightManifestStatus final {
    WeightManifestError error{WeightManifestError::None};
    std::string detail{};
    [[nodiscard]] bool ok() const noexcept { return error == WeightManifestError::None; }
    [[nodiscard]] explicit operator bool() const noexcept { return ok(); }
};

struct WeightTensorDescriptor final {
    std::string name{};
    std::uint64_t offset{0};
    std::uint64_t byte_size{0};
    std::vector<std::uint32_t> shape{};
    std::string sha256{};
};

struct WeightManifest final {
    std::uint32_t version{0};
    std::string checkpoint{};
    std::string checkpoint_revision{};
    std::string tokenizer_revision{};
    std::string config_sha256{};
    std::string data_type{};
    std::string data_file{};
    std::uint64_t data_bytes{0};
    TinyLlamaConfig config{};
    std::vector<WeightTensorDescriptor> tensors{};

    [[nodiscard]] WeightTensorDescriptor const* find(std::string_view name) const noexcept;
};

struct WeightManifestLoadResult final {
    WeightManifestStatus status{};
    WeightManifest manifest{};
    [[nodiscard]] bool ok() const noexcept { return status.ok(); }
};

[[nodiscard]] WeightManifestLoadResult loadWeightManifest(std::string const& manifest_path);
[[nodiscard]] WeightManifestStatus validateWeightManifest(WeightManifest const& manifest);
[[nodiscard]] WeightManifestStatus validateWeightDataFile(WeightManifest const& manifest,
    std::string const& data_path);
[[nodiscard]] WeightManifestStatus computeWeightDataSha256(std::string const& data_path,
    std::uint64_t offset, std::uint64_t byte_size, std::string& sha256);

} // namespace kimkvcache
