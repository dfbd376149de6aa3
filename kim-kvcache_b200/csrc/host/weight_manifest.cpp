// Weight manifest parsing and validation (semantics: reference
// src/model/weight_manifest.cpp:361-684; the SHA-256 is this library's own).
#include "weight_manifest.h"

#include "sha256.h"

#include <algorithm>
#include <charconv>
#include <fstream>
#include <limits>
#include <map>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace kimkvcache {
namespace {

WeightManifestStatus fail(WeightManifestError e, std::string detail)
{
    return WeightManifestStatus{e, std::move(detail)};
}

bool parseU64(std::string_view s, std::uint64_t& v)
{
    if (s.empty()) {
        return false;
    }
    auto const r = std::from_chars(s.data(), s.data() + s.size(), v);
    return r.ec == std::errc{} && r.ptr == s.data() + s.size();
}

bool parseF32(std::string const& s, float& v)
{
    try {
        std::size_t used = 0;
        v = std::stof(s, &used);
        return used == s.size();
    } catch (...) {
        return false;
    }
}

bool isHexDigest(std::string const& s)
{
    return s.size() == 64 && std::all_of(s.begin(), s.end(), [](char c) {
        return (c >= '0' && c <= '9') || (c >= 'a' && c <= 'f');
    });
}

std::vector<std::string> splitOn(std::string const& s, char sep)
{
    std::vector<std::string> parts;
    std::size_t begin = 0;
    for (;;) {
        std::size_t const end = s.find(sep, begin);
        parts.push_back(s.substr(begin, end == std::string::npos ? std::string::npos : end - begin));
        if (end == std::string::npos) {
            return parts;
        }
        begin = end + 1;
    }
}

std::map<std::string, std::vector<std::uint32_t>> expectedTensors(TinyLlamaConfig const& c)
{
    std::map<std::string, std::vector<std::uint32_t>> out;
    out["model.embed_tokens.weight"] = {c.vocabulary_size, c.hidden_size};
    out["model.norm.weight"] = {c.hidden_size};
    out["lm_head.weight"] = {c.vocabulary_size, c.hidden_size};
    std::uint32_t const kv = c.kv_head_count * c.head_dimension;
    for (std::uint32_t l = 0; l < c.layer_count; ++l) {
        std::string const p = "model.layers." + std::to_string(l) + ".";
        out[p + "input_layernorm.weight"] = {c.hidden_size};
        out[p + "post_attention_layernorm.weight"] = {c.hidden_size};
        out[p + "self_attn.q_proj.weight"] = {c.hidden_size, c.hidden_size};
        out[p + "self_attn.k_proj.weight"] = {kv, c.hidden_size};
        out[p + "self_attn.v_proj.weight"] = {kv, c.hidden_size};
        out[p + "self_attn.o_proj.weight"] = {c.hidden_size, c.hidden_size};
        out[p + "mlp.gate_proj.weight"] = {c.intermediate_size, c.hidden_size};
        out[p + "mlp.up_proj.weight"] = {c.intermediate_size, c.hidden_size};
        out[p + "mlp.down_proj.weight"] = {c.hidden_size, c.intermediate_size};
    }
    return out;
}

} // namespace

WeightTensorDescriptor const* WeightManifest::find(std::string_view name) const noexcept
{
    for (WeightTensorDescriptor const& t : tensors) {
        if (t.name == name) {
            return &t;
        }
    }
    return nullptr;
}

WeightManifestStatus validateWeightManifest(WeightManifest const& m)
{
    if (m.version != 1) {
        return fail(WeightManifestError::UnsupportedVersion, "manifest version must be 1");
    }
    if (m.data_type != "fp16") {
        return fail(WeightManifestError::UnsupportedDataType, "only fp16 archives are supported");
    }
    if (!m.config.valid()) {
        return fail(WeightManifestError::InvalidConfig, "model dimensions are inconsistent");
    }
    if (m.checkpoint.empty() || m.checkpoint_revision.empty() || m.tokenizer_revision.empty()
        || !isHexDigest(m.config_sha256) || m.data_file.empty() || m.data_bytes == 0) {
        return fail(WeightManifestError::InvalidConfig, "model identity or archive metadata incomplete");
    }
    auto expected = expectedTensors(m.config);
    std::unordered_set<std::string> seen;
    struct Range {
        std::uint64_t begin, end;
        std::string const* name;
    };
    std::vector<Range> ranges;
    for (WeightTensorDescriptor const& t : m.tensors) {
        if (!seen.insert(t.name).second) {
            return fail(WeightManifestError::DuplicateTensor, "duplicate tensor: " + t.name);
        }
        auto const want = expected.find(t.name);
        if (want == expected.end()) {
            return fail(WeightManifestError::UnexpectedTensor, "unexpected tensor: " + t.name);
        }
        if (t.shape != want->second || !isHexDigest(t.sha256)) {
            return fail(WeightManifestError::InvalidTensor, "shape or checksum mismatch: " + t.name);
        }
        std::uint64_t elements = 1;
        bool shape_ok = !t.shape.empty() && t.shape.size() <= 2;
        for (std::uint32_t d : t.shape) {
            if (d == 0 || elements > std::numeric_limits<std::uint64_t>::max() / d) {
                shape_ok = false;
                break;
            }
            elements *= d;
        }
        if (!shape_ok || t.offset % 2 != 0 || elements > std::numeric_limits<std::uint64_t>::max() / 2
            || t.byte_size != elements * 2 || t.offset > m.data_bytes
            || t.byte_size > m.data_bytes - t.offset) {
            return fail(WeightManifestError::InvalidTensor, "invalid byte range: " + t.name);
        }
        ranges.push_back(Range{t.offset, t.offset + t.byte_size, &t.name});
        expected.erase(want);
    }
    if (!expected.empty()) {
        return fail(WeightManifestError::MissingTensor, "missing tensor: " + expected.begin()->first);
    }
    std::sort(ranges.begin(), ranges.end(), [](Range const& a, Range const& b) { return a.begin < b.begin; });
    for (std::size_t i = 1; i < ranges.size(); ++i) {
        if (ranges[i].begin < ranges[i - 1].end) {
            return fail(WeightManifestError::InvalidTensor, "overlapping tensor ranges: " + *ranges[i].name);
        }
    }
    return {};
}

WeightManifestLoadResult loadWeightManifest(std::string const& path)
{
    WeightManifestLoadResult result;
    std::ifstream in(path);
    if (!in) {
        result.status = fail(WeightManifestError::FileOpenFailed, path);
        return result;
    }
    std::unordered_map<std::string, std::string> kv;
    std::vector<std::string> records;
    std::string line;
    std::size_t number = 0;
    while (std::getline(in, line)) {
        ++number;
        if (line.empty() || line[0] == '#') {
            continue;
        }
        std::size_t const eq = line.find('=');
        if (eq == std::string::npos || eq == 0) {
            result.status = fail(WeightManifestError::ParseFailed, "invalid line " + std::to_string(number));
            return result;
        }
        std::string key = line.substr(0, eq);
        std::string value = line.substr(eq + 1);
        if (key == "tensor") {
            records.push_back(std::move(value));
        } else if (!kv.emplace(key, std::move(value)).second) {
            result.status = fail(WeightManifestError::ParseFailed, "duplicate key: " + key);
            return result;
        }
    }
    WeightManifest& m = result.manifest;
    auto str = [&](char const* key, std::string& out) {
        auto const f = kv.find(key);
        if (f == kv.end() || f->second.empty()) {
            return false;
        }
        out = f->second;
        return true;
    };
    auto u32 = [&](char const* key, std::uint32_t& out) {
        auto const f = kv.find(key);
        std::uint64_t v = 0;
        if (f == kv.end() || !parseU64(f->second, v) || v > std::numeric_limits<std::uint32_t>::max()) {
            return false;
        }
        out = static_cast<std::uint32_t>(v);
        return true;
    };
    TinyLlamaConfig& c = m.config;
    std::uint32_t tensor_count = 0;
    bool ok = u32("version", m.version) && str("checkpoint", m.checkpoint)
        && str("checkpoint_revision", m.checkpoint_revision)
        && str("tokenizer_revision", m.tokenizer_revision) && str("config_sha256", m.config_sha256)
        && str("dtype", m.data_type) && str("data_file", m.data_file)
        && u32("hidden_size", c.hidden_size) && u32("intermediate_size", c.intermediate_size)
        && u32("layer_count", c.layer_count) && u32("attention_head_count", c.attention_head_count)
        && u32("kv_head_count", c.kv_head_count) && u32("head_dimension", c.head_dimension)
        && u32("vocabulary_size", c.vocabulary_size)
        && u32("max_position_embeddings", c.max_position_embeddings)
        && u32("bos_token_id", c.bos_token_id) && u32("eos_token_id", c.eos_token_id)
        && u32("tensor_count", tensor_count);
    auto const bytes = kv.find("data_bytes");
    ok = ok && bytes != kv.end() && parseU64(bytes->second, m.data_bytes);
    auto const eps = kv.find("rms_norm_epsilon");
    auto const theta = kv.find("rope_theta");
    ok = ok && eps != kv.end() && theta != kv.end() && parseF32(eps->second, c.rms_norm_epsilon)
        && parseF32(theta->second, c.rope_theta);
    auto const tied = kv.find("tied_word_embeddings");
    ok = ok && tied != kv.end() && (tied->second == "0" || tied->second == "1");
    if (tied != kv.end()) {
        c.tied_word_embeddings = tied->second == "1";
    }
    if (!ok || tensor_count != records.size()) {
        result.status = fail(WeightManifestError::ParseFailed, "missing field or tensor_count mismatch");
        return result;
    }
    for (std::string const& record : records) {
        std::vector<std::string> const f = splitOn(record, '|');
        if (f.size() != 5) {
            result.status = fail(WeightManifestError::ParseFailed, "tensor record must contain five fields");
            return result;
        }
        WeightTensorDescriptor t;
        t.name = f[0];
        t.sha256 = f[4];
        if (!parseU64(f[1], t.offset) || !parseU64(f[2], t.byte_size)) {
            result.status = fail(WeightManifestError::ParseFailed, "invalid tensor range: " + t.name);
            return result;
        }
        for (std::string const& dim : splitOn(f[3], ',')) {
            std::uint64_t d = 0;
            if (!parseU64(dim, d) || d > std::numeric_limits<std::uint32_t>::max()) {
                result.status = fail(WeightManifestError::ParseFailed, "invalid tensor shape: " + t.name);
                return result;
            }
            t.shape.push_back(static_cast<std::uint32_t>(d));
        }
        m.tensors.push_back(std::move(t));
    }
    result.status = validateWeightManifest(m);
    return result;
}

WeightManifestStatus computeWeightDataSha256(std::string const& path, std::uint64_t offset,
    std::uint64_t bytes, std::string& digest)
{
    digest.clear();
    if (path.empty() || bytes == 0
        || offset > static_cast<std::uint64_t>(std::numeric_limits<std::streamoff>::max())) {
        return fail(WeightManifestError::InvalidArgument, "invalid checksum range");
    }
    std::ifstream in(path, std::ios::binary);
    if (!in) {
        return fail(WeightManifestError::FileOpenFailed, path);
    }
    in.seekg(static_cast<std::streamoff>(offset));
    std::vector<char> buffer(4u << 20);
    Sha256 sha;
    while (bytes != 0) {
        std::size_t const want = static_cast<std::size_t>(std::min<std::uint64_t>(bytes, buffer.size()));
        in.read(buffer.data(), static_cast<std::streamsize>(want));
        if (in.gcount() != static_cast<std::streamsize>(want)) {
            return fail(WeightManifestError::DataFileMismatch, "checksum range exceeds data file");
        }
        sha.update(buffer.data(), want);
        bytes -= want;
    }
    digest = sha.hexDigest();
    return {};
}

WeightManifestStatus validateWeightDataFile(WeightManifest const& m, std::string const& path)
{
    WeightManifestStatus const meta = validateWeightManifest(m);
    if (!meta.ok()) {
        return meta;
    }
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) {
        return fail(WeightManifestError::FileOpenFailed, path);
    }
    std::streamoff const size = in.tellg();
    if (size < 0 || static_cast<std::uint64_t>(size) != m.data_bytes) {
        return fail(WeightManifestError::DataFileMismatch, "archive size differs from manifest");
    }
    for (WeightTensorDescriptor const& t : m.tensors) {
        std::string actual;
        WeightManifestStatus const s = computeWeightDataSha256(path, t.offset, t.byte_size, actual);
        if (!s.ok()) {
            return s;
        }
        if (actual != t.sha256) {
            return fail(WeightManifestError::ChecksumMismatch, t.name);
        }
    }
    return {};
}

} // namespace kimkvcache
