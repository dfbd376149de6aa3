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

bool toU64(std::string_view s, std::uint64_t& v)
{
    auto const r = std::from_chars(s.data(), s.data() + s.size(), v);
    return !s.empty() && r.ec == std::errc{} && r.ptr == s.data() + s.size();
}

bool isSha256Hex(std::string_view s)
{
    return s.size() == 64
        && std::all_of(s.begin(), s.end(), [](char c) { return (c >= '0' && c <= '9') || (c >= 'a' && c <= 'f'); });
}

std::vector<std::string_view> fields(std::string_view s, char sep)
{
    std::vector<std::string_view> out;
    for (std::size_t at = 0;;) {
        std::size_t const next = s.find(sep, at);
        out.push_back(s.substr(at, next == std::string_view::npos ? std::string_view::npos : next - at));
        if (next == std::string_view::npos) {
            return out;
        }
        at = next + 1;
    }
}

// ---- header schema ----------------------------------------------------------------------------
//
// Every required key of the manifest header, its type and where it lands.
// The manifest format is the reference's (src/model/weight_manifest.cpp);
// the table is this loader's own.
enum class Kind : std::uint8_t { Text, U32, U64, F32, Flag };

struct Field {
    char const* key;
    Kind kind;
    void* (*target)(WeightManifest&);
};

template <auto Member>
void* at(WeightManifest& m)
{
    return &(m.*Member);
}

template <auto Member>
void* atConfig(WeightManifest& m)
{
    return &(m.config.*Member);
}

constexpr Field kHeader[] = {
    {"version", Kind::U32, &at<&WeightManifest::version>},
    {"checkpoint", Kind::Text, &at<&WeightManifest::checkpoint>},
    {"checkpoint_revision", Kind::Text, &at<&WeightManifest::checkpoint_revision>},
    {"tokenizer_revision", Kind::Text, &at<&WeightManifest::tokenizer_revision>},
    {"config_sha256", Kind::Text, &at<&WeightManifest::config_sha256>},
    {"dtype", Kind::Text, &at<&WeightManifest::data_type>},
    {"data_file", Kind::Text, &at<&WeightManifest::data_file>},
    {"data_bytes", Kind::U64, &at<&WeightManifest::data_bytes>},
    {"hidden_size", Kind::U32, &atConfig<&TinyLlamaConfig::hidden_size>},
    {"intermediate_size", Kind::U32, &atConfig<&TinyLlamaConfig::intermediate_size>},
    {"layer_count", Kind::U32, &atConfig<&TinyLlamaConfig::layer_count>},
    {"attention_head_count", Kind::U32, &atConfig<&TinyLlamaConfig::attention_head_count>},
    {"kv_head_count", Kind::U32, &atConfig<&TinyLlamaConfig::kv_head_count>},
    {"head_dimension", Kind::U32, &atConfig<&TinyLlamaConfig::head_dimension>},
    {"vocabulary_size", Kind::U32, &atConfig<&TinyLlamaConfig::vocabulary_size>},
    {"max_position_embeddings", Kind::U32, &atConfig<&TinyLlamaConfig::max_position_embeddings>},
    {"bos_token_id", Kind::U32, &atConfig<&TinyLlamaConfig::bos_token_id>},
    {"eos_token_id", Kind::U32, &atConfig<&TinyLlamaConfig::eos_token_id>},
    {"rms_norm_epsilon", Kind::F32, &atConfig<&TinyLlamaConfig::rms_norm_epsilon>},
    {"rope_theta", Kind::F32, &atConfig<&TinyLlamaConfig::rope_theta>},
    {"tied_word_embeddings", Kind::Flag, &atConfig<&TinyLlamaConfig::tied_word_embeddings>},
};

bool store(Field const& f, std::string const& text, WeightManifest& m)
{
    void* dst = f.target(m);
    std::uint64_t v = 0;
    switch (f.kind) {
    case Kind::Text:
        *static_cast<std::string*>(dst) = text;
        return !text.empty();
    case Kind::U32:
        if (!toU64(text, v) || v > std::numeric_limits<std::uint32_t>::max()) {
            return false;
        }
        *static_cast<std::uint32_t*>(dst) = static_cast<std::uint32_t>(v);
        return true;
    case Kind::U64:
        return toU64(text, *static_cast<std::uint64_t*>(dst));
    case Kind::F32:
        try {
            std::size_t used = 0;
            *static_cast<float*>(dst) = std::stof(text, &used);
            return used == text.size();
        } catch (...) {
            return false;
        }
    case Kind::Flag:
        *static_cast<bool*>(dst) = text == "1";
        return text == "0" || text == "1";
    }
    return false;
}

// ---- tensor schema ------------------------------------------------------------------------------

// Shape of each tensor of a decoder layer, by name suffix.
struct LayerTensor {
    char const* suffix;
    std::vector<std::uint32_t> (*shape)(TinyLlamaConfig const&);
};

std::uint32_t kvWidth(TinyLlamaConfig const& c) { return c.kv_head_count * c.head_dimension; }

constexpr LayerTensor kLayerTensors[] = {
    {"input_layernorm.weight", [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.hidden_size}; }},
    {"post_attention_layernorm.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.hidden_size}; }},
    {"self_attn.q_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.hidden_size, c.hidden_size}; }},
    {"self_attn.k_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{kvWidth(c), c.hidden_size}; }},
    {"self_attn.v_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{kvWidth(c), c.hidden_size}; }},
    {"self_attn.o_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.hidden_size, c.hidden_size}; }},
    {"mlp.gate_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.intermediate_size, c.hidden_size}; }},
    {"mlp.up_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.intermediate_size, c.hidden_size}; }},
    {"mlp.down_proj.weight",
        [](TinyLlamaConfig const& c) { return std::vector<std::uint32_t>{c.hidden_size, c.intermediate_size}; }},
};

// Every tensor a config needs, name -> shape, in name order (the first
// missing one reported is the smallest name).
std::map<std::string, std::vector<std::uint32_t>> requiredTensors(TinyLlamaConfig const& c)
{
    std::map<std::string, std::vector<std::uint32_t>> out{
        {"model.embed_tokens.weight", {c.vocabulary_size, c.hidden_size}},
        {"lm_head.weight", {c.vocabulary_size, c.hidden_size}},
        {"model.norm.weight", {c.hidden_size}},
    };
    for (std::uint32_t layer = 0; layer < c.layer_count; ++layer) {
        std::string const prefix = "model.layers." + std::to_string(layer) + ".";
        for (LayerTensor const& t : kLayerTensors) {
            out.emplace(prefix + t.suffix, t.shape(c));
        }
    }
    return out;
}

// Bytes of an FP16 tensor of this shape (0 for an unusable shape).
std::uint64_t fp16Bytes(std::vector<std::uint32_t> const& shape)
{
    if (shape.empty() || shape.size() > 2) {
        return 0;
    }
    std::uint64_t n = 1;
    for (std::uint32_t d : shape) {
        if (d == 0 || n > std::numeric_limits<std::uint64_t>::max() / 2 / d) {
            return 0;
        }
        n *= d;
    }
    return n * 2;
}

} // namespace

WeightTensorDescriptor const* WeightManifest::find(std::string_view name) const noexcept
{
    auto const it = std::find_if(tensors.begin(), tensors.end(),
        [name](WeightTensorDescriptor const& t) { return t.name == name; });
    return it == tensors.end() ? nullptr : &*it;
}

WeightManifestStatus validateWeightManifest(WeightManifest const& m)
{
    if (m.version != 1) {
        return fail(WeightManifestError::UnsupportedVersion, "unsupported manifest version");
    }
    if (m.data_type != "fp16") {
        return fail(WeightManifestError::UnsupportedDataType, "archives must be fp16");
    }
    if (!m.config.valid()) {
        return fail(WeightManifestError::InvalidConfig, "inconsistent model dimensions");
    }
    bool const identified = !m.checkpoint.empty() && !m.checkpoint_revision.empty() && !m.tokenizer_revision.empty()
        && isSha256Hex(m.config_sha256) && !m.data_file.empty() && m.data_bytes != 0;
    if (!identified) {
        return fail(WeightManifestError::InvalidConfig, "checkpoint identity or data file fields are incomplete");
    }
    std::map<std::string, std::vector<std::uint32_t>> required = requiredTensors(m.config);
    std::unordered_set<std::string_view> listed;
    std::vector<std::pair<std::uint64_t, std::uint64_t>> extents;  // [begin, end) per tensor
    for (WeightTensorDescriptor const& t : m.tensors) {
        if (!listed.insert(t.name).second) {
            return fail(WeightManifestError::DuplicateTensor, "listed twice: " + t.name);
        }
        auto const need = required.find(t.name);
        if (need == required.end()) {
            return fail(WeightManifestError::UnexpectedTensor, "not a tensor of this model: " + t.name);
        }
        if (t.shape != need->second || !isSha256Hex(t.sha256)) {
            return fail(WeightManifestError::InvalidTensor, "wrong shape or digest: " + t.name);
        }
        std::uint64_t const bytes = fp16Bytes(t.shape);
        if (bytes == 0 || t.byte_size != bytes || t.offset % 2 != 0 || t.offset > m.data_bytes
            || t.byte_size > m.data_bytes - t.offset) {
            return fail(WeightManifestError::InvalidTensor, "byte range does not fit: " + t.name);
        }
        extents.emplace_back(t.offset, t.offset + t.byte_size);
        required.erase(need);
    }
    if (!required.empty()) {
        return fail(WeightManifestError::MissingTensor, "not listed: " + required.begin()->first);
    }
    std::sort(extents.begin(), extents.end());
    auto const overlap = std::adjacent_find(extents.begin(), extents.end(),
        [](auto const& a, auto const& b) { return b.first < a.second; });
    if (overlap != extents.end()) {
        return fail(WeightManifestError::InvalidTensor, "tensor byte ranges overlap");
    }
    return {};
}

WeightManifestLoadResult loadWeightManifest(std::string const& path)
{
    WeightManifestLoadResult result;
    auto parse_error = [&result](std::string why) {
        result.status = fail(WeightManifestError::ParseFailed, std::move(why));
        return result;
    };
    std::ifstream in(path);
    if (!in) {
        result.status = fail(WeightManifestError::FileOpenFailed, path);
        return result;
    }
    // key=value lines ('#' comments and blank lines skipped); "tensor" may
    // repeat, every other key appears once.
    std::unordered_map<std::string, std::string> header;
    std::vector<std::string> tensor_lines;
    std::string line;
    for (std::size_t number = 1; std::getline(in, line); ++number) {
        if (line.empty() || line.front() == '#') {
            continue;
        }
        std::size_t const eq = line.find('=');
        if (eq == 0 || eq == std::string::npos) {
            return parse_error("line " + std::to_string(number) + " is not key=value");
        }
        std::string key = line.substr(0, eq);
        if (key == "tensor") {
            tensor_lines.push_back(line.substr(eq + 1));
        } else if (!header.emplace(key, line.substr(eq + 1)).second) {
            return parse_error("key given twice: " + key);
        }
    }
    WeightManifest& m = result.manifest;
    for (Field const& f : kHeader) {
        auto const v = header.find(f.key);
        if (v == header.end() || !store(f, v->second, m)) {
            return parse_error(std::string("missing or malformed field: ") + f.key);
        }
    }
    std::uint32_t declared = 0;
    auto const count = header.find("tensor_count");
    std::uint64_t n = 0;
    if (count == header.end() || !toU64(count->second, n) || n > std::numeric_limits<std::uint32_t>::max()
        || (declared = static_cast<std::uint32_t>(n)) != tensor_lines.size()) {
        return parse_error("tensor_count is missing or does not match the tensor lines");
    }
    // tensor=name|offset|bytes|d0[,d1]|sha256
    for (std::string const& text : tensor_lines) {
        std::vector<std::string_view> const part = fields(text, '|');
        if (part.size() != 5) {
            return parse_error("a tensor line needs five fields");
        }
        WeightTensorDescriptor t;
        t.name = std::string(part[0]);
        t.sha256 = std::string(part[4]);
        if (!toU64(part[1], t.offset) || !toU64(part[2], t.byte_size)) {
            return parse_error("bad offset or size: " + t.name);
        }
        for (std::string_view d : fields(part[3], ',')) {
            std::uint64_t dim = 0;
            if (!toU64(d, dim) || dim > std::numeric_limits<std::uint32_t>::max()) {
                return parse_error("bad shape: " + t.name);
            }
            t.shape.push_back(static_cast<std::uint32_t>(dim));
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
