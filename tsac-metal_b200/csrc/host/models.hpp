// Model packages: seeded Bellard-format sources, the packer that turns them
// into the reference's 20-file `.weights` package, and the runtime loader that
// reads a package directory (ours or one written by the reference packer).
#pragma once
#include "common.hpp"

#include <array>
#include <filesystem>
#include <string>

namespace tsacb
{
// libnc storage codes (src/weights/source_model.hpp:12-18).
enum class Storage : std::uint32_t
{
    f32 = 0,
    bf16 = 1,
    bf8 = 0x8000b,
    bf8l = 0x8000e
};

struct SourceTensor
{
    std::string name;
    Storage storage = Storage::f32;
    std::vector<std::size_t> dims; // axis 0 fastest
    std::size_t elements = 0;
    std::size_t data_plane_bytes = 0;
    Bytes payload;
};

// One original `.bin` model (libnc container, src/weights/source_model.cpp:104-178).
struct SourceModel
{
    std::string metadata = "{}";
    std::vector<SourceTensor> tensors;

    const SourceTensor& tensor(const std::string& name) const;
    std::vector<float> dequantize(const std::string& name) const;
    Bytes serialize() const;
    static SourceModel parse(ByteView bytes, const Limits& limits = {});
};

// Seeded random-init sources with the DAC-44kHz / TSAC geometry. `channels`
// is 1 (mono: 9 books) or 2 (joint stereo: 12 books).
SourceModel seeded_dac(unsigned channels, std::uint64_t seed);
SourceModel seeded_transformer(unsigned channels, std::uint64_t seed);
// Writes dac_{mono,stereo}_q8.bin and tsac_{mono,stereo}_q8.bin.
void write_seeded_sources(const std::filesystem::path& directory, std::uint64_t seed);
// Same contract as the reference packer's command line
// (src/weights/pack_main.cpp:733-787): four `.bin` inputs -> 20 `.weights`
// files plus adapter_offsets.hpp in `output`.
void pack_models(const std::filesystem::path& input, const std::filesystem::path& output,
                 const std::string& pack_id, bool include_transformer);

// File roles in the order of the reference's ModelFile enum
// (src/weights/model_directory.hpp:9-32), mono roles first.
enum Role : unsigned
{
    dac_analysis_source,
    dac_analysis_shared,
    dac_synthesis_source,
    dac_synthesis_shared,
    rvq_shared,
    rvq_encode_shared,
    rvq_encode_apple,
    rvq_encode_metal,
    transformer_source,
    transformer_shared,
    role_count
};

struct Range
{
    std::size_t offset = 0, bytes = 0;
};

struct DacLayout
{
    std::vector<Range> values, gains, biases, alphas;
};

struct VariantLayout
{
    DacLayout analysis, synthesis;
    std::vector<std::array<Range, 7>> books;
    std::vector<std::array<Range, 3>> projections;
    std::vector<std::array<Range, 2>> norms;
    std::array<Range, 2> constants{};
    Range embeddings{};
};

// Parsed adapter_offsets.hpp: file names and byte ranges per entry point.
struct PackageLayout
{
    std::string generation_id;
    bool has_transformer = false;
    std::array<std::string, 20> filenames{};
    VariantLayout variants[2]; // [0] mono, [1] stereo

    static PackageLayout parse(const std::string& header_text);
};

// A package directory: the 20 `.weights` files and adapter_offsets.hpp.
class Package
{
public:
    explicit Package(std::filesystem::path directory, const Limits& limits = {});
    const PackageLayout& layout() const
    {
        return layout_;
    }
    const std::filesystem::path& path() const
    {
        return directory_;
    }
    // Reads one stored range of a role file (channels 1 or 2).
    Bytes read(unsigned channels, Role role, Range range) const;

private:
    std::filesystem::path directory_;
    Limits limits_;
    PackageLayout layout_;
};

// --- prepared tensors (host copies, device-ready layouts) -------------------

struct Conv1dSpec
{
    unsigned input_channels = 0, output_channels = 0, kernel = 0;
    unsigned stride = 1, padding = 0, dilation = 1;
    bool transposed = false;
};

struct PreparedConv
{
    Conv1dSpec spec;
    // Folded FP32 weights in the reference's stored order: ordinary
    // [out][tap][in] (in fastest), transposed [in][tap][out] (out fastest).
    std::vector<float> weights;
    std::vector<float> bias;
};

// DAC graph in evaluation order (src/common/analysis.tpp:114-155,
// src/common/synthesis.tpp:113-157): convolutions 0..29 and Snake alphas 0..28
// in the model contract's numbering (src/models/contract.cpp:144-177).
struct PreparedDac
{
    unsigned channels = 0;
    bool synthesis = false;
    std::vector<PreparedConv> convs;       // 30
    std::vector<std::vector<float>> alphas; // 29
};

struct PreparedRvqBook
{
    std::vector<float> input_weights;   // [8][1024] (in fastest)
    std::vector<float> input_bias;      // [8]
    std::vector<float> search;          // [1024][8] normalized search vectors
    std::vector<float> codebook;        // [1024][8]
    std::vector<float> output_weights;  // [1024][8]
    std::vector<float> output_bias;     // [1024]
};

struct PreparedLinear
{
    unsigned input = 0, output = 0;
    std::vector<std::int8_t> weights; // canonical [output][input]
    std::vector<float> scales;        // [input/256][output]
    std::vector<float> bias;          // [output]
};

struct PreparedNorm
{
    std::vector<std::uint16_t> gain, bias; // bf16 [512]
};

struct PreparedTransformer
{
    unsigned channels = 0, books = 0;
    // Projection index order of the model contract (src/models/contract.cpp:185-189):
    // temporal layers 0..11 x {qkv, attn_out, mlp_in, mlp_out} = 0..47,
    // codebook layers = 48..59, 60 temporal cb_proj, 61 codebook cb_proj, 62 proj_f.
    std::vector<PreparedLinear> projections; // 63
    // normalization_index order: temporal 0..23 (ln_1, ln_2 per layer), 24 ln_f,
    // codebook 25..30, 31 ln_f.
    std::vector<PreparedNorm> norms; // 32
    std::vector<std::uint16_t> positions;  // [books][512]
    std::vector<std::uint16_t> rotations;  // [1024][128]
    std::vector<std::uint16_t> embeddings; // [books][1024][1024]
};

PreparedDac prepare_dac(const Package& package, unsigned channels, bool synthesis,
                        const Limits& limits = {});
std::vector<PreparedRvqBook> prepare_rvq(const Package& package, unsigned channels,
                                         unsigned books);
PreparedTransformer prepare_transformer(const Package& package, unsigned channels,
                                        unsigned books);

// Shared preparation arithmetic (also used by the packer).
// BF8 expansion of a contract-shaped tensor (src/weights/preparation.cpp:17-67).
std::vector<float> expand_bf8(ByteView payload, std::array<std::size_t, 3> axes);
// DAC weight-norm folding (src/weights/normalization.cpp:50-94).
void fold_dac_weight_norm(std::span<float> values, std::span<const float> gain,
                          std::size_t fan_in);
// RVQ search normalisation (src/weights/preparation.cpp:69-93).
void normalize_search(const float* input, float* output);
// Fused codebook projection (src/weights/preparation.cpp:95-114).
void project_codebook(unsigned index, std::span<const float> codebook,
                      std::span<const float> weights, std::span<const float> bias, float* output);
} // namespace tsacb
