// Seeded sources, packer, package loader and load-time preparation.
//
// The on-disk formats and the preparation arithmetic have to be identical to
// the reference's so that one package feeds both implementations:
//   * libnc `.bin` container: src/weights/source_model.cpp:104-178
//   * package roles/alignment: src/weights/pack_main.cpp:61-338, WEIGHTS.md:45-69
//   * adapter_offsets.hpp text: src/weights/pack_main.cpp:471-704
//   * contract shapes/encodings: src/models/contract.cpp:51-177
//   * BF8 expansion, DAC weight-norm folding, RVQ search normalisation and the
//     fused codebook projection: src/weights/preparation.cpp:17-114,
//     src/weights/normalization.cpp:50-94.
// Everything here is written from those descriptions; none of it is on the
// GPU hot path (it runs once per model load).
#include "models.hpp"

#include <algorithm>
#include <cstdio>
#include <fcntl.h>
#include <fstream>
#include <map>
#include <sstream>
#include <unistd.h>

namespace tsacb
{
namespace
{
constexpr std::size_t region_alignment = 16384, tensor_alignment = 256;

// ---------------------------------------------------------------- seeding --
// splitmix64 stream per (seed, tensor name): stable across platforms.
struct Rng
{
    std::uint64_t state;

    Rng(std::uint64_t seed, const std::string& name)
    {
        std::uint64_t h = 0xcbf29ce484222325ull;
        for (unsigned char c : name)
        {
            h = (h ^ c) * 0x100000001b3ull;
        }
        state = seed * 0x9e3779b97f4a7c15ull ^ h;
    }
    std::uint64_t next()
    {
        std::uint64_t z = (state += 0x9e3779b97f4a7c15ull);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        return z ^ (z >> 31);
    }
    double uniform() // [0, 1)
    {
        return double(next() >> 11) * 0x1p-53;
    }
    double uniform(double lo, double hi)
    {
        return lo + (hi - lo) * uniform();
    }
    double normal()
    {
        const double u1 = 1.0 - uniform(), u2 = uniform();
        return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
    }
    int int8() // uniform in [-127, 127]
    {
        return int(next() % 255u) - 127;
    }
};

std::size_t elements_of(const std::vector<std::size_t>& dims)
{
    std::size_t n = 1;
    for (auto d : dims)
    {
        n = checked_mul(n, d);
    }
    return n;
}

void put_f32(Bytes& out, float v)
{
    const auto bits = std::bit_cast<std::uint32_t>(v);
    for (unsigned j = 0; j < 4; ++j)
    {
        out.push_back(static_cast<std::uint8_t>(bits >> (j * 8)));
    }
}

SourceTensor f32_tensor(std::string name, std::vector<std::size_t> dims,
                        const std::vector<float>& values)
{
    SourceTensor t;
    t.name = std::move(name);
    t.storage = Storage::f32;
    t.dims = std::move(dims);
    t.elements = elements_of(t.dims);
    require(values.size() == t.elements, "seeded tensor size mismatch");
    t.payload.reserve(t.elements * 4);
    for (float v : values)
    {
        put_f32(t.payload, v);
    }
    t.data_plane_bytes = t.payload.size();
    return t;
}

std::vector<float> normal_values(Rng& rng, std::size_t n, double mean, double sd)
{
    std::vector<float> v(n);
    for (auto& x : v)
    {
        x = static_cast<float>(mean + sd * rng.normal());
    }
    return v;
}

std::vector<float> uniform_values(Rng& rng, std::size_t n, double lo, double hi)
{
    std::vector<float> v(n);
    for (auto& x : v)
    {
        x = static_cast<float>(rng.uniform(lo, hi));
    }
    return v;
}

// BF8 (32-row blocks) or BF8L (256-row blocks) payload: int8 data plane then a
// bf16 scale plane [outer][rows/block][ceil8(columns)], each 256-aligned.
SourceTensor quantized_tensor(std::string name, Storage storage, std::vector<std::size_t> dims,
                              Rng& rng, double scale_lo, double scale_hi)
{
    SourceTensor t;
    t.name = std::move(name);
    t.storage = storage;
    t.dims = std::move(dims);
    t.elements = elements_of(t.dims);
    const std::size_t block = storage == Storage::bf8 ? 32 : 256;
    const auto rows = t.dims[0], columns = t.dims[1];
    require(rows % block == 0, "seeded quantized shape");
    const auto outer = t.elements / rows / columns;
    const auto padded = align_up(columns, 8);
    t.data_plane_bytes = align_up(t.elements, 256);
    const auto scale_count = outer * (rows / block) * padded;
    t.payload.assign(t.data_plane_bytes + align_up(scale_count * 2, 256), 0);
    for (std::size_t i = 0; i < t.elements; ++i)
    {
        t.payload[i] = static_cast<std::uint8_t>(static_cast<std::int8_t>(rng.int8()));
    }
    for (std::size_t o = 0; o < outer; ++o)
    {
        for (std::size_t b = 0; b < rows / block; ++b)
        {
            for (std::size_t c = 0; c < columns; ++c)
            {
                const auto s = to_bf16(static_cast<float>(rng.uniform(scale_lo, scale_hi)));
                const auto at = t.data_plane_bytes + ((o * (rows / block) + b) * padded + c) * 2;
                t.payload[at] = static_cast<std::uint8_t>(s);
                t.payload[at + 1] = static_cast<std::uint8_t>(s >> 8);
            }
        }
    }
    return t;
}

struct DacBuilder
{
    SourceModel model;
    std::uint64_t seed;

    void conv(const std::string& stem, std::vector<std::size_t> dims, bool f32, double gain_lo,
              double gain_hi, std::size_t bias_width, std::size_t gain_width)
    {
        Rng rng(seed, stem + ".weight_v");
        if (f32)
        {
            model.tensors.push_back(f32_tensor(stem + ".weight_v", dims,
                                               normal_values(rng, elements_of(dims), 0.0, 1.0)));
        }
        else
        {
            model.tensors.push_back(
                quantized_tensor(stem + ".weight_v", Storage::bf8, dims, rng, 0.004, 0.012));
        }
        Rng g(seed, stem + ".weight_g"), b(seed, stem + ".bias");
        model.tensors.push_back(f32_tensor(stem + ".weight_g", {1, 1, gain_width},
                                           uniform_values(g, gain_width, gain_lo, gain_hi)));
        model.tensors.push_back(
            f32_tensor(stem + ".bias", {bias_width}, normal_values(b, bias_width, 0.0, 0.01)));
    }

    void alpha(const std::string& stem, std::size_t width)
    {
        Rng rng(seed, stem + ".alpha");
        model.tensors.push_back(
            f32_tensor(stem + ".alpha", {width, 1, 1}, uniform_values(rng, width, 0.5, 1.5)));
    }
};
} // namespace

SourceModel seeded_dac(unsigned channels, std::uint64_t seed)
{
    require(channels == 1 || channels == 2, "seeded DAC channels");
    DacBuilder d{{}, seed};
    // Encoder (graph order, src/weights/pack_main.cpp:419-445 names/shapes).
    d.conv("encoder.block.0", {channels, 7, 64}, true, 0.8, 1.2, 64, 64);
    std::size_t width = 64;
    for (unsigned s = 0; s < 4; ++s)
    {
        const unsigned stride = std::array<unsigned, 4>{2, 4, 8, 8}[s];
        const auto stem = "encoder.block." + std::to_string(s + 1) + ".block.";
        for (unsigned r = 0; r < 3; ++r)
        {
            const auto unit = stem + std::to_string(r) + ".block.";
            d.alpha(unit + "0", width);
            d.conv(unit + "1", {width, 7, width}, false, 0.8, 1.2, width, width);
            d.alpha(unit + "2", width);
            d.conv(unit + "3", {width, 1, width}, false, 0.3, 0.6, width, width);
        }
        d.alpha(stem + "3", width);
        d.conv(stem + "4", {width, 2u * stride, width * 2}, false, 0.8, 1.2, width * 2, width * 2);
        width *= 2;
    }
    d.alpha("encoder.block.5", 1024);
    d.conv("encoder.block.6", {1024, 3, 1024}, false, 0.8, 1.2, 1024, 1024);
    // Decoder: convolutions >= 22 are FP32 (src/models/contract.cpp:80-86).
    unsigned index = 0;
    d.conv("decoder.model.0", {1024, 7, 1536}, false, 0.8, 1.2, 1536, 1536);
    ++index;
    width = 1536;
    for (unsigned s = 0; s < 4; ++s)
    {
        const unsigned stride = std::array<unsigned, 4>{8, 8, 4, 2}[s];
        const auto stem = "decoder.model." + std::to_string(s + 1) + ".block.";
        d.alpha(stem + "0", width);
        // Transposed weights are stored [out, kernel, in]; gain is per input.
        d.conv(stem + "1", {width / 2, 2u * stride, width}, index >= 22, 0.8, 1.2, width / 2,
               width);
        ++index;
        width /= 2;
        for (unsigned r = 0; r < 3; ++r)
        {
            const auto unit = stem + std::to_string(r + 2) + ".block.";
            d.alpha(unit + "0", width);
            d.conv(unit + "1", {width, 7, width}, index >= 22, 0.8, 1.2, width, width);
            ++index;
            d.alpha(unit + "2", width);
            d.conv(unit + "3", {width, 1, width}, index >= 22, 0.3, 0.6, width, width);
            ++index;
        }
    }
    d.alpha("decoder.model.5", 96);
    // Exit gain keeps decoded PCM near the -12 dBFS input level.
    d.conv("decoder.model.6", {96, 7, channels}, true, 0.08, 0.12, channels, channels);
    // Residual quantizers (src/weights/source_model.cpp:262-270).
    const unsigned books = channels == 1 ? 9 : 12;
    for (unsigned b = 0; b < books; ++b)
    {
        const auto p = "quantizer.quantizers." + std::to_string(b) + ".";
        Rng cb(seed, p + "codebook.weight"), iv(seed, p + "in_proj.weight_v"),
            ig(seed, p + "in_proj.weight_g"), ib(seed, p + "in_proj.bias"),
            ov(seed, p + "out_proj.weight_v"), og(seed, p + "out_proj.weight_g"),
            ob(seed, p + "out_proj.bias");
        d.model.tensors.push_back(
            f32_tensor(p + "codebook.weight", {8, 1024}, normal_values(cb, 8192, 0.0, 1.0)));
        d.model.tensors.push_back(
            f32_tensor(p + "in_proj.weight_v", {1024, 1, 8}, normal_values(iv, 8192, 0.0, 1.0)));
        d.model.tensors.push_back(
            f32_tensor(p + "in_proj.weight_g", {1, 1, 8}, uniform_values(ig, 8, 0.8, 1.2)));
        d.model.tensors.push_back(
            f32_tensor(p + "in_proj.bias", {8}, normal_values(ib, 8, 0.0, 0.01)));
        d.model.tensors.push_back(
            f32_tensor(p + "out_proj.weight_v", {8, 1, 1024}, normal_values(ov, 8192, 0.0, 1.0)));
        d.model.tensors.push_back(f32_tensor(p + "out_proj.weight_g", {1, 1, 1024},
                                             uniform_values(og, 1024, 0.2, 0.4)));
        d.model.tensors.push_back(
            f32_tensor(p + "out_proj.bias", {1024}, normal_values(ob, 1024, 0.0, 0.01)));
    }
    return std::move(d.model);
}

SourceModel seeded_transformer(unsigned channels, std::uint64_t seed)
{
    require(channels == 1 || channels == 2, "seeded Transformer channels");
    SourceModel model;
    const unsigned books = channels == 1 ? 9 : 12;
    const auto linear = [&](const std::string& name, std::size_t in, std::size_t out, double damp,
                            bool has_bias)
    {
        Rng rng(seed, name);
        // Effective weight variance ~ damp^2 / in keeps unit-variance activations.
        const double s = damp * std::sqrt(3.0 / double(in)) / 127.0;
        model.tensors.push_back(
            quantized_tensor(name, Storage::bf8l, {in, out}, rng, 0.5 * s, 1.5 * s));
        if (has_bias)
        {
            const auto bias = name.substr(0, name.size() - 1) + "b";
            Rng b(seed, bias);
            model.tensors.push_back(f32_tensor(bias, {out}, normal_values(b, out, 0.0, 0.02)));
        }
    };
    const auto norm = [&](const std::string& stem)
    {
        Rng g(seed, stem + "g"), b(seed, stem + "b");
        model.tensors.push_back(f32_tensor(stem + "g", {512}, normal_values(g, 512, 1.0, 0.05)));
        model.tensors.push_back(f32_tensor(stem + "b", {512}, normal_values(b, 512, 0.0, 0.02)));
    };
    for (const auto& [prefix, layers] :
         std::array<std::pair<std::string, unsigned>, 2>{{{"", 12u}, {"codebook_decoder.", 3u}}})
    {
        for (unsigned layer = 0; layer < layers; ++layer)
        {
            const auto stem = prefix + "h" + std::to_string(layer) + "/";
            norm(stem + "ln_1/");
            linear(stem + "attn/c_attn/w", 512, 1536, 1.0, true);
            linear(stem + "attn/c_proj/w", 512, 512, 0.5, true);
            norm(stem + "ln_2/");
            linear(stem + "mlp/c_fc/w", 512, 2048, 1.0, true);
            linear(stem + "mlp/c_proj/w", 2048, 512, 0.5, true);
        }
        norm(prefix + "ln_f/");
    }
    linear("cb_proj", 1024, 512, 1.0, false);
    linear("codebook_decoder.cb_proj", 1024, 512, 1.0, false);
    {
        Rng rng(seed, "codebook_decoder.wpe");
        model.tensors.push_back(f32_tensor("codebook_decoder.wpe", {512, books},
                                           normal_values(rng, 512 * books, 0.0, 0.1)));
    }
    linear("proj_f/w", 512, 1024, 1.0, true);
    {
        // Standard rotary coefficients: pair i of position p is
        // (cos(p*theta_i), sin(p*theta_i)), theta_i = 10000^(-2i/128).
        std::vector<float> rotary(128 * 1024);
        for (std::size_t p = 0; p < 1024; ++p)
        {
            for (std::size_t i = 0; i < 64; ++i)
            {
                const double theta = std::pow(10000.0, -2.0 * double(i) / 128.0);
                rotary[p * 128 + 2 * i] = static_cast<float>(std::cos(double(p) * theta));
                rotary[p * 128 + 2 * i + 1] = static_cast<float>(std::sin(double(p) * theta));
            }
        }
        model.tensors.push_back(f32_tensor("rotary_embed", {128, 1024}, rotary));
    }
    return model;
}

// ---------------------------------------------------------------- .bin IO --
const SourceTensor& SourceModel::tensor(const std::string& name) const
{
    for (const auto& t : tensors)
    {
        if (t.name == name)
        {
            return t;
        }
    }
    throw Error("tensor not found: " + name);
}

std::vector<float> SourceModel::dequantize(const std::string& name) const
{
    const auto& t = tensor(name);
    std::vector<float> values(t.elements);
    if (t.storage == Storage::f32)
    {
        std::memcpy(values.data(), t.payload.data(), t.elements * 4);
    }
    else if (t.storage == Storage::bf16)
    {
        for (std::size_t i = 0; i < t.elements; ++i)
        {
            values[i] = bf16_at(t.payload, i * 2);
        }
    }
    else
    {
        const std::size_t block = t.storage == Storage::bf8 ? 32 : 256;
        const auto rows = t.dims[0], columns = t.dims[1];
        const auto outer = t.elements / rows / columns, padded = align_up(columns, 8);
        const auto scale_rows = rows / block;
        for (std::size_t o = 0; o < outer; ++o)
        {
            for (std::size_t c = 0; c < columns; ++c)
            {
                for (std::size_t b = 0; b < scale_rows; ++b)
                {
                    const auto index = (o * columns + c) * rows + b * block;
                    const float scale =
                        bf16_at(t.payload, t.data_plane_bytes + ((o * scale_rows + b) * padded + c) * 2);
                    for (std::size_t r = 0; r < block; ++r)
                    {
                        values[index + r] =
                            static_cast<float>(static_cast<std::int8_t>(t.payload[index + r])) *
                            scale;
                    }
                }
            }
        }
    }
    return values;
}

Bytes SourceModel::serialize() const
{
    Bytes out;
    const auto u32 = [&](std::uint32_t v)
    {
        for (unsigned j = 0; j < 4; ++j)
        {
            out.push_back(static_cast<std::uint8_t>(v >> (j * 8)));
        }
    };
    u32(0x23f4aefb);
    u32(static_cast<std::uint32_t>(metadata.size()));
    out.insert(out.end(), metadata.begin(), metadata.end());
    for (const auto& t : tensors)
    {
        u32(0x23f4aefa);
        u32(static_cast<std::uint32_t>(t.storage));
        u32(static_cast<std::uint32_t>(t.dims.size()));
        u32(static_cast<std::uint32_t>(t.name.size()));
        for (auto d : t.dims)
        {
            u32(static_cast<std::uint32_t>(d));
        }
        out.insert(out.end(), t.name.begin(), t.name.end());
        out.insert(out.end(), t.payload.begin(), t.payload.end());
    }
    return out;
}

SourceModel SourceModel::parse(ByteView data, const Limits& limits)
{
    require(data.size() <= limits.file_bytes, "model exceeds file size limit");
    require(le32(data, 0) == 0x23f4aefb, "invalid model magic");
    const auto metadata_size = le32(data, 4);
    require(metadata_size > 0 && metadata_size <= limits.metadata_bytes,
            "invalid metadata length");
    require(data.size() - 8 >= metadata_size, "truncated input");
    SourceModel model;
    model.metadata.assign(data.begin() + 8, data.begin() + 8 + metadata_size);
    std::size_t offset = 8 + metadata_size;
    while (offset < data.size())
    {
        require(model.tensors.size() < limits.tensors, "tensor count exceeds limit");
        require(le32(data, offset) == 0x23f4aefa, "invalid tensor magic");
        SourceTensor t;
        const auto storage = le32(data, offset + 4);
        require(storage == 0 || storage == 1 || storage == 0x8000b || storage == 0x8000e,
                "unsupported tensor storage");
        t.storage = static_cast<Storage>(storage);
        const auto rank = le32(data, offset + 8), name_size = le32(data, offset + 12);
        require(rank > 0 && rank <= 8, "invalid tensor rank");
        require(name_size > 0 && name_size <= limits.name_bytes, "invalid tensor name length");
        offset += 16;
        t.elements = 1;
        for (std::size_t a = 0; a < rank; ++a)
        {
            const auto d = le32(data, offset);
            require(d > 0, "zero tensor dimension");
            t.elements = checked_mul(t.elements, d);
            require(t.elements <= limits.tensor_elements, "tensor element count exceeds limit");
            t.dims.push_back(d);
            offset += 4;
        }
        require(data.size() - offset >= name_size, "truncated input");
        t.name.assign(data.begin() + offset, data.begin() + offset + name_size);
        offset += name_size;
        std::size_t bytes;
        if (t.storage == Storage::f32 || t.storage == Storage::bf16)
        {
            bytes = checked_mul(t.elements, t.storage == Storage::f32 ? 4 : 2);
            t.data_plane_bytes = bytes;
        }
        else
        {
            const std::size_t block = t.storage == Storage::bf8 ? 32 : 256;
            require(t.dims.size() >= 2 && t.dims[0] % block == 0,
                    "unsupported quantized tensor shape");
            const auto scales = checked_mul(checked_mul(t.dims[0] / block, align_up(t.dims[1], 8)),
                                            t.elements / t.dims[0] / t.dims[1]);
            t.data_plane_bytes = align_up(t.elements, 256);
            bytes = checked_add(t.data_plane_bytes, align_up(checked_mul(scales, 2), 256));
        }
        require(data.size() - offset >= bytes, "truncated input");
        t.payload.assign(data.begin() + offset, data.begin() + offset + bytes);
        offset += bytes;
        model.tensors.push_back(std::move(t));
    }
    require(!model.tensors.empty(), "model has no tensors");
    return model;
}

namespace
{
void write_bytes(const std::filesystem::path& path, ByteView bytes)
{
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    require(bool(f), "cannot create output file");
    f.write(reinterpret_cast<const char*>(bytes.data()), static_cast<std::streamsize>(bytes.size()));
    require(bool(f), "cannot write output file");
}

Bytes read_bytes(const std::filesystem::path& path)
{
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f)
    {
        throw Error("cannot open input: " + path.string());
    }
    const auto size = static_cast<std::size_t>(f.tellg());
    Bytes bytes(size);
    f.seekg(0);
    f.read(reinterpret_cast<char*>(bytes.data()), static_cast<std::streamsize>(size));
    require(bool(f), "cannot read complete input");
    return bytes;
}
} // namespace

void write_seeded_sources(const std::filesystem::path& directory, std::uint64_t seed)
{
    std::filesystem::create_directories(directory);
    for (unsigned c : {1u, 2u})
    {
        const std::string v = c == 1 ? "mono" : "stereo";
        write_bytes(directory / ("dac_" + v + "_q8.bin"), seeded_dac(c, seed).serialize());
        write_bytes(directory / ("tsac_" + v + "_q8.bin"), seeded_transformer(c, seed).serialize());
    }
}

// ------------------------------------------------------------ preparation --
std::vector<float> expand_bf8(ByteView payload, std::array<std::size_t, 3> axes)
{
    const auto rows = axes[0], columns = axes[1];
    const auto count = rows * columns * axes[2];
    const std::size_t block = 32;
    const auto padded = (columns + 7) / 8 * 8;
    const auto plane = align_up(count, 256);
    require(rows && columns && rows % block == 0, "invalid quantized source shape");
    std::vector<float> values(count);
    for (std::size_t column = 0; column < count / rows; ++column)
    {
        for (std::size_t b = 0; b < rows / block; ++b)
        {
            const float scale = bf16_at(
                payload, plane + ((column / columns * (rows / block) + b) * padded + column % columns) * 2);
            const auto begin = column * rows + b * block;
            for (std::size_t i = 0; i < block; ++i)
            {
                values[begin + i] =
                    static_cast<float>(static_cast<std::int8_t>(payload[begin + i])) * scale;
            }
        }
    }
    require_finite(values, "nonfinite source weights");
    return values;
}

void fold_dac_weight_norm(std::span<float> values, std::span<const float> gain, std::size_t fan_in)
{
    require(fan_in > 0 && !gain.empty() && values.size() == fan_in * gain.size(),
            "weight normalization shape mismatch");
    require_finite(values, "nonfinite weight normalization value");
    require_finite(gain, "nonfinite weight normalization value");
    const float inverse_width = 1.0f / std::sqrt(static_cast<float>(fan_in));
    const float reciprocal_width = 1.0f / static_cast<float>(fan_in);
    std::vector<float> squares(fan_in);
    for (std::size_t c = 0; c < gain.size(); ++c)
    {
        auto column = values.subspan(c * fan_in, fan_in);
        for (std::size_t i = 0; i < fan_in; ++i)
        {
            squares[i] = column[i] * column[i];
        }
        // Balanced adjacent-pair tree; an odd tail is carried up unchanged.
        for (std::size_t width = fan_in; width > 1; width = (width + 1) / 2)
        {
            for (std::size_t i = 0; i < width / 2; ++i)
            {
                squares[i] = squares[2 * i] + squares[2 * i + 1];
            }
            if (width % 2)
            {
                squares[width / 2] = squares[width - 1];
            }
        }
        const float mean = squares[0] * reciprocal_width;
        require(mean > 0 && std::isfinite(mean), "invalid weight normalization norm");
        const float inverse_rms = 1.0f / std::sqrt(mean);
        for (std::size_t i = 0; i < fan_in; ++i)
        {
            const float normalized = column[i] * inverse_rms;
            const float unit = normalized * inverse_width;
            column[i] = unit * gain[c];
        }
    }
    require_finite(values, "nonfinite weight normalization value");
}

void normalize_search(const float* input, float* output)
{
    const float epsilon = std::bit_cast<float>(std::uint32_t{0x2b8cbccc});
    float squares[8];
    for (int i = 0; i < 8; ++i)
    {
        squares[i] = input[i] * input[i];
    }
    for (int width = 8; width > 1; width /= 2)
    {
        for (int i = 0; i < width / 2; ++i)
        {
            squares[i] = squares[i * 2] + squares[i * 2 + 1];
        }
    }
    require(std::isfinite(squares[0]), "invalid RVQ normalization norm");
    const float mean = squares[0] * (1.0f / 8.0f);
    const float inverse_rms = 1.0f / std::sqrt(mean + epsilon);
    const float inverse_width = 1.0f / std::sqrt(8.0f);
    for (int i = 0; i < 8; ++i)
    {
        const float normalized = input[i] * inverse_rms;
        output[i] = normalized * inverse_width;
    }
}

void project_codebook(unsigned index, std::span<const float> codebook,
                      std::span<const float> weights, std::span<const float> bias, float* output)
{
    require(index < 1024 && codebook.size() == 8192 && weights.size() == 8192 &&
                bias.size() == 1024,
            "invalid codebook projection");
    for (std::size_t j = 0; j < 1024; ++j)
    {
        float sum = 0;
        for (std::size_t i = 0; i < 8; ++i)
        {
            sum = std::fma(weights[j * 8 + i], codebook[std::size_t(index) * 8 + i], sum);
        }
        output[j] = sum + bias[j];
    }
    require_finite(std::span<const float>(output, 1024), "nonfinite RVQ value");
}

// ------------------------------------------------------------------ packer --
namespace
{
constexpr std::array<const char*, 10> role_names{
    "dac-analysis-source",  "dac-analysis-shared", "dac-synthesis-source",
    "dac-synthesis-shared", "rvq-shared",          "rvq-encode-shared",
    "rvq-encode-apple",     "rvq-encode-metal",    "transformer-source",
    "transformer-shared"};

// Contract geometry (src/models/contract.cpp:51-143).
std::array<std::size_t, 3> dac_shape(bool synthesis, unsigned c, unsigned conv)
{
    if (!conv)
    {
        return synthesis ? std::array<std::size_t, 3>{1024, 7, 1536}
                         : std::array<std::size_t, 3>{c, 7, 64};
    }
    if (conv == 29)
    {
        return synthesis ? std::array<std::size_t, 3>{96, 7, c}
                         : std::array<std::size_t, 3>{1024, 3, 1024};
    }
    const auto stage = (conv - 1) / 7, within = (conv - 1) % 7;
    const std::size_t width = synthesis ? (1536u >> stage) : (64u << stage);
    const std::size_t stride = synthesis ? std::array<unsigned, 4>{8, 8, 4, 2}[stage]
                                         : std::array<unsigned, 4>{2, 4, 8, 8}[stage];
    if (synthesis && within == 0)
    {
        return {width / 2, 2 * stride, width};
    }
    if (!synthesis && within == 6)
    {
        return {width, 2 * stride, width * 2};
    }
    const auto residual = synthesis ? within - 1 : within;
    const auto w = synthesis ? width / 2 : width;
    return {w, residual % 2 == 0 ? 7u : 1u, w};
}

bool dac_f32(bool synthesis, unsigned conv)
{
    return (!synthesis && conv == 0) || (synthesis && conv >= 22);
}

std::size_t dac_alpha_width(bool synthesis, unsigned index)
{
    return index == 28 ? (synthesis ? 96u : 1024u)
           : synthesis ? (1536u >> (index / 7)) / (index % 7 == 0 ? 1u : 2u)
                       : (64u << (index / 7));
}

std::array<std::size_t, 2> projection_shape(unsigned p) // {input, output}
{
    if (p == 60 || p == 61)
    {
        return {1024, 512};
    }
    if (p == 62)
    {
        return {512, 1024};
    }
    switch (p % 4)
    {
    case 0:
        return {512, 1536};
    case 1:
        return {512, 512};
    case 2:
        return {512, 2048};
    default:
        return {2048, 512};
    }
}

std::size_t bf8_bytes(std::array<std::size_t, 3> a)
{
    const auto scales = (a[0] / 32) * align_up(a[1], 8) * a[2];
    return align_up(a[0] * a[1] * a[2], 256) + align_up(scales * 2, 256);
}

struct Ref
{
    std::int64_t region = -1;
    std::size_t offset = 0, bytes = 0;
};

class Writer
{
public:
    std::filesystem::path output;
    std::string id;
    struct File
    {
        std::string name;
        std::size_t bytes = 0;
    };
    std::vector<File> files;
    struct Region
    {
        std::size_t file, offset, bytes;
    };
    std::vector<Region> regions;
    std::ofstream stream;
    std::size_t file = 0, region = 0;
    // Bound source tensors and named prepared entries, keyed by (channels, transformer, name).
    std::map<std::tuple<unsigned, bool, std::string>, Ref> sources, prepared;

    void begin_file(unsigned channels, const std::string& role)
    {
        file = files.size();
        files.push_back({"tsac-" + std::string(channels == 1 ? "mono-" : "stereo-") + role + "-" +
                             id + ".weights",
                         0});
        stream.open(output / files.back().name, std::ios::binary | std::ios::trunc);
        require(bool(stream), "cannot create weight file");
    }
    void pad(std::size_t alignment)
    {
        const auto target = align_up(files[file].bytes, alignment);
        static const std::vector<char> zero(region_alignment, 0);
        stream.write(zero.data(), static_cast<std::streamsize>(target - files[file].bytes));
        files[file].bytes = target;
    }
    void begin_region()
    {
        pad(region_alignment);
        region = regions.size();
        regions.push_back({file, files[file].bytes, 0});
    }
    void end_region()
    {
        pad(region_alignment);
        regions[region].bytes = files[file].bytes - regions[region].offset;
    }
    void end_file()
    {
        stream.flush();
        require(bool(stream), "cannot write complete weight file");
        stream.close();
    }
    Ref put(ByteView bytes)
    {
        pad(tensor_alignment);
        const Ref r{static_cast<std::int64_t>(region), files[file].bytes - regions[region].offset,
                    bytes.size()};
        stream.write(reinterpret_cast<const char*>(bytes.data()),
                     static_cast<std::streamsize>(bytes.size()));
        files[file].bytes += bytes.size();
        return r;
    }
    Ref floats(std::span<const float> values)
    {
        require_finite(values, "nonfinite prepared weights");
        Bytes b;
        b.reserve(values.size() * 4);
        for (float v : values)
        {
            put_f32(b, v);
        }
        return put(b);
    }
    Ref halves(std::span<const std::uint16_t> values)
    {
        Bytes b(values.size() * 2);
        for (std::size_t i = 0; i < values.size(); ++i)
        {
            require((values[i] & 0x7f80u) != 0x7f80u, "nonfinite BF16 weight");
            b[i * 2] = static_cast<std::uint8_t>(values[i]);
            b[i * 2 + 1] = static_cast<std::uint8_t>(values[i] >> 8);
        }
        return put(b);
    }
    Range absolute(const Ref& r) const
    {
        require(r.region >= 0, "missing application entrypoint");
        return {regions.at(static_cast<std::size_t>(r.region)).offset + r.offset, r.bytes};
    }
};

void pack_dac(Writer& w, unsigned channels, const SourceModel& model)
{
    for (const std::string stage : {"analysis", "synthesis"})
    {
        const std::string prefix = stage == "analysis" ? "encoder." : "decoder.";
        w.begin_file(channels, "dac-" + stage + "-source");
        w.begin_region();
        for (const auto& t : model.tensors)
        {
            if (!t.name.starts_with(prefix) || !t.name.ends_with(".weight_v"))
            {
                continue;
            }
            const auto stem = t.name.substr(0, t.name.size() - 9);
            auto values = model.dequantize(t.name);
            const auto gains = model.dequantize(stem + ".weight_g");
            fold_dac_weight_norm(values, gains, t.dims[0] * t.dims[1]); // validation only
            w.sources[{channels, false, t.name}] = w.put(t.payload);
            w.sources[{channels, false, stem + ".weight_g"}] = w.floats(gains);
        }
        w.end_region();
        w.end_file();
        w.begin_file(channels, "dac-" + stage + "-shared");
        w.begin_region();
        for (const auto& t : model.tensors)
        {
            if (t.name.starts_with(prefix) &&
                (t.name.ends_with(".bias") || t.name.ends_with(".alpha")))
            {
                const auto values = model.dequantize(t.name);
                if (t.name.ends_with(".alpha"))
                {
                    const float eps = std::bit_cast<float>(std::uint32_t{0x3089705f});
                    for (float a : values)
                    {
                        require(std::isfinite(a + eps) && a + eps != 0,
                                "invalid Snake denominator");
                    }
                }
                w.sources[{channels, false, t.name}] = w.floats(values);
            }
        }
        w.end_region();
        w.end_file();
    }
}

void pack_rvq(Writer& w, unsigned channels, unsigned books, const SourceModel& dac)
{
    for (const std::string role : {"shared", "encode-shared", "encode-apple", "encode-metal"})
    {
        w.begin_file(channels, "rvq-" + role);
        for (unsigned book = 0; book < books; ++book)
        {
            w.begin_region();
            const auto prefix = "quantizer.quantizers." + std::to_string(book);
            const auto key = prefix + ".";
            if (role == "shared")
            {
                const auto codebook = dac.dequantize(prefix + ".codebook.weight");
                w.prepared[{channels, false, key + "codebook"}] = w.floats(codebook);
                auto out = dac.dequantize(prefix + ".out_proj.weight_v");
                fold_dac_weight_norm(out, dac.dequantize(prefix + ".out_proj.weight_g"), 8);
                w.prepared[{channels, false, key + "output_weights"}] = w.floats(out);
                w.prepared[{channels, false, key + "output_bias"}] =
                    w.floats(dac.dequantize(prefix + ".out_proj.bias"));
            }
            else if (role == "encode-shared")
            {
                const auto codebook = dac.dequantize(prefix + ".codebook.weight");
                std::vector<float> normalized(codebook.size());
                for (std::size_t s = 0; s < 1024; ++s)
                {
                    normalize_search(codebook.data() + s * 8, normalized.data() + s * 8);
                }
                w.prepared[{channels, false, key + "normalized_search"}] = w.floats(normalized);
                w.prepared[{channels, false, key + "input_bias"}] =
                    w.floats(dac.dequantize(prefix + ".in_proj.bias"));
            }
            else
            {
                auto in = dac.dequantize(prefix + ".in_proj.weight_v");
                fold_dac_weight_norm(in, dac.dequantize(prefix + ".in_proj.weight_g"), 1024);
                if (role == "encode-metal")
                {
                    std::vector<float> packed(in.size());
                    for (std::size_t out = 0; out < 8; ++out)
                    {
                        for (std::size_t i = 0; i < 1024; ++i)
                        {
                            packed[out + 8 * i] = in[i + 1024 * out];
                        }
                    }
                    in = std::move(packed);
                }
                w.prepared[{channels, false,
                            key + "input_" + (role == "encode-apple" ? "apple" : "metal")}] =
                    w.floats(in);
            }
            w.end_region();
        }
        w.end_file();
    }
}

void pack_transformer(Writer& w, unsigned channels, unsigned books, const SourceModel& dac,
                      const SourceModel& model)
{
    w.begin_file(channels, "transformer-source");
    w.begin_region();
    for (const auto& t : model.tensors)
    {
        if (t.name.ends_with("/w") || t.name == "cb_proj" || t.name == "codebook_decoder.cb_proj")
        {
            require(t.storage == Storage::bf8l,
                    "Transformer projections require BF8L source weights");
        }
        if (t.storage == Storage::bf8l)
        {
            require(t.dims.size() == 2 && t.dims[0] % 256 == 0 && t.dims[1] % 8 == 0,
                    "unsupported Transformer packing shape");
            w.sources[{channels, true, t.name}] =
                w.put(ByteView(t.payload).first(t.elements));
        }
    }
    w.end_region();
    w.end_file();
    w.begin_file(channels, "transformer-shared");
    w.begin_region();
    for (const auto& t : model.tensors)
    {
        if (t.storage == Storage::bf8l)
        {
            const auto d = t.dims[0], o = t.dims[1], padded = align_up(o, 8);
            std::vector<float> scales(d / 256 * o);
            for (std::size_t b = 0; b < d / 256; ++b)
            {
                for (std::size_t out = 0; out < o; ++out)
                {
                    scales[b * o + out] =
                        bf16_at(t.payload, t.data_plane_bytes + 2 * (b * padded + out));
                }
            }
            w.prepared[{channels, true, t.name + ".scales"}] = w.floats(scales);
            std::vector<float> bias(o, 0);
            if (t.name.ends_with("/w"))
            {
                bias = model.dequantize(t.name.substr(0, t.name.size() - 1) + "b");
            }
            w.prepared[{channels, true, t.name + ".bias"}] = w.floats(bias);
        }
        else if (!t.name.ends_with("/b") || t.name.find("ln_") != std::string::npos)
        {
            const auto values = model.dequantize(t.name);
            std::vector<std::uint16_t> halves(values.size());
            std::transform(values.begin(), values.end(), halves.begin(), to_bf16);
            w.sources[{channels, true, t.name}] = w.halves(halves);
        }
    }
    w.end_region();
    for (unsigned book = 0; book < books; ++book)
    {
        w.begin_region();
        const auto prefix = "quantizer.quantizers." + std::to_string(book);
        const auto codebook = dac.dequantize(prefix + ".codebook.weight");
        auto out = dac.dequantize(prefix + ".out_proj.weight_v");
        fold_dac_weight_norm(out, dac.dequantize(prefix + ".out_proj.weight_g"), 8);
        const auto bias = dac.dequantize(prefix + ".out_proj.bias");
        std::vector<std::uint16_t> embeddings(std::size_t{1024} * 1024);
        std::array<float, 1024> column;
        for (unsigned symbol = 0; symbol < 1024; ++symbol)
        {
            project_codebook(symbol, codebook, out, bias, column.data());
            std::transform(column.begin(), column.end(), embeddings.data() + symbol * 1024,
                           to_bf16);
        }
        w.prepared[{channels, true, "embeddings." + std::to_string(book)}] = w.halves(embeddings);
        w.end_region();
    }
    w.end_file();
}

// adapter_offsets.hpp in the reference packer's exact text form.
void write_adapter_header(Writer& w, bool include_transformer)
{
    std::ostringstream h;
    h << "// Generated application entrypoints. Shapes and encodings live in the contract.\n"
         "#pragma once\n#include \"model_layout.hpp\"\nnamespace tsac::adapter_generated {\n"
         "using model_layout::Range;\n";
    h << "inline constexpr char generation_id[]=\"" << w.id << "\";\n";
    h << "inline constexpr bool has_transformer=" << (include_transformer ? "true" : "false")
      << ";\n";
    h << "inline constexpr std::array<const char*,20> filenames{{\n";
    for (unsigned c : {1u, 2u})
    {
        for (auto role : role_names)
        {
            const auto name = "tsac-" + std::string(c == 1 ? "mono-" : "stereo-") + role + "-" +
                              w.id + ".weights";
            const bool present = std::any_of(w.files.begin(), w.files.end(),
                                             [&](const auto& f) { return f.name == name; });
            if (present)
            {
                h << '"' << name << "\",\n";
            }
            else
            {
                h << "nullptr,\n";
            }
        }
    }
    h << "}};\n";
    const auto print = [&](Range r) { h << '{' << r.offset << ',' << r.bytes << '}'; };
    const auto source = [&](unsigned c, bool tf, const std::string& name, std::size_t bytes)
    {
        const auto found = w.sources.find({c, tf, name});
        require(found != w.sources.end() && found->second.bytes == bytes,
                ("source disagrees with application contract: " + name).c_str());
        return w.absolute(found->second);
    };
    const auto prep = [&](unsigned c, bool tf, const std::string& name, std::size_t bytes)
    {
        const auto found = w.prepared.find({c, tf, name});
        require(found != w.prepared.end() && found->second.bytes == bytes,
                ("prepared entry disagrees with contract: " + name).c_str());
        return w.absolute(found->second);
    };
    const auto ranges = [&](const std::string& name, const std::vector<Range>& entries)
    {
        h << "inline constexpr std::array<Range," << entries.size() << "> " << name << "{{\n";
        for (auto r : entries)
        {
            print(r);
            h << ",\n";
        }
        h << "}};\n";
    };
    const auto rows = [&]<std::size_t N>(const std::string& name,
                                         const std::vector<std::array<Range, N>>& entries)
    {
        h << "inline constexpr std::array<std::array<Range," << N << ">," << entries.size() << "> "
          << name << "{{\n";
        for (const auto& row : entries)
        {
            h << "{{";
            for (auto r : row)
            {
                print(r);
                h << ',';
            }
            h << "}},\n";
        }
        h << "}};\n";
    };
    for (unsigned c : {1u, 2u})
    {
        const std::string v = c == 1 ? "mono_" : "stereo_";
        for (bool synthesis : {false, true})
        {
            const std::string prefix = synthesis ? "decoder.model." : "encoder.block.";
            const auto name = v + (synthesis ? "synthesis" : "analysis");
            std::vector<std::string> stems{prefix + "0"}, alphas;
            for (unsigned stage = 0; stage < 4; ++stage)
            {
                const auto block = prefix + std::to_string(stage + 1) + ".block.";
                if (synthesis)
                {
                    stems.push_back(block + "1");
                    alphas.push_back(block + "0.alpha");
                }
                for (unsigned unit = 0; unit < 3; ++unit)
                {
                    const auto residual =
                        block + std::to_string(unit + (synthesis ? 2 : 0)) + ".block.";
                    stems.push_back(residual + "1");
                    stems.push_back(residual + "3");
                    alphas.push_back(residual + "0.alpha");
                    alphas.push_back(residual + "2.alpha");
                }
                if (!synthesis)
                {
                    stems.push_back(block + "4");
                    alphas.push_back(block + "3.alpha");
                }
            }
            stems.push_back(prefix + "6");
            alphas.push_back(prefix + "5.alpha");
            std::vector<Range> values, gains, biases, alpha_ranges;
            for (unsigned i = 0; i < stems.size(); ++i)
            {
                const auto shape = dac_shape(synthesis, c, i);
                const bool transposed = synthesis && i > 0 && i < 29 && (i - 1) % 7 == 0;
                const auto elements = shape[0] * shape[1] * shape[2];
                values.push_back(source(c, false, stems[i] + ".weight_v",
                                        dac_f32(synthesis, i) ? elements * 4 : bf8_bytes(shape)));
                gains.push_back(source(c, false, stems[i] + ".weight_g", shape[2] * 4));
                biases.push_back(
                    source(c, false, stems[i] + ".bias", shape[transposed ? 0 : 2] * 4));
            }
            for (unsigned i = 0; i < alphas.size(); ++i)
            {
                alpha_ranges.push_back(source(c, false, alphas[i], dac_alpha_width(synthesis, i) * 4));
            }
            ranges(name + "_values", values);
            ranges(name + "_gains", gains);
            ranges(name + "_biases", biases);
            ranges(name + "_alphas", alpha_ranges);
            h << "inline constexpr model_layout::Dac " << name << '{' << name << "_values," << name
              << "_gains," << name << "_biases," << name << "_alphas};\n";
        }
        std::vector<std::array<Range, 7>> books;
        for (unsigned b = 0; b < (c == 1 ? 9u : 12u); ++b)
        {
            const auto stem = "quantizer.quantizers." + std::to_string(b) + ".";
            books.push_back({prep(c, false, stem + "codebook", 8192 * 4),
                             prep(c, false, stem + "output_weights", 8192 * 4),
                             prep(c, false, stem + "output_bias", 1024 * 4),
                             prep(c, false, stem + "normalized_search", 8192 * 4),
                             prep(c, false, stem + "input_bias", 8 * 4),
                             prep(c, false, stem + "input_apple", 8192 * 4),
                             prep(c, false, stem + "input_metal", 8192 * 4)});
        }
        rows(v + "books", books);
        std::vector<std::array<Range, 3>> projections;
        std::vector<std::array<Range, 2>> norms;
        std::array<Range, 2> constants{};
        Range embeddings{};
        if (include_transformer)
        {
            const auto linear = [&](const std::string& stem)
            {
                const auto shape = projection_shape(static_cast<unsigned>(projections.size()));
                projections.push_back({source(c, true, stem, shape[0] * shape[1]),
                                       prep(c, true, stem + ".scales", shape[1] * shape[0] / 256 * 4),
                                       prep(c, true, stem + ".bias", shape[1] * 4)});
            };
            const auto norm = [&](const std::string& stem)
            {
                norms.push_back({source(c, true, stem + "g", 1024), source(c, true, stem + "b", 1024)});
            };
            for (bool cb : {false, true})
            {
                const std::string prefix = cb ? "codebook_decoder." : "";
                for (unsigned layer = 0; layer < (cb ? 3u : 12u); ++layer)
                {
                    const auto stem = prefix + "h" + std::to_string(layer) + "/";
                    for (auto suffix : {"attn/c_attn/w", "attn/c_proj/w", "mlp/c_fc/w", "mlp/c_proj/w"})
                    {
                        linear(stem + suffix);
                    }
                    norm(stem + "ln_1/");
                    norm(stem + "ln_2/");
                }
                norm(prefix + "ln_f/");
            }
            linear("cb_proj");
            linear("codebook_decoder.cb_proj");
            linear("proj_f/w");
            constants = {source(c, true, "codebook_decoder.wpe", 512 * (c == 1 ? 9u : 12u) * 2),
                         source(c, true, "rotary_embed", 128 * 1024 * 2)};
            embeddings = prep(c, true, "embeddings.0", 1024 * 1024 * 2);
        }
        rows(v + "projections", projections);
        rows(v + "norms", norms);
        h << "inline constexpr model_layout::Transformer " << v << "transformer{" << v
          << "projections," << v << "norms,{{";
        for (auto r : constants)
        {
            print(r);
            h << ',';
        }
        h << "}},";
        print(embeddings);
        h << "};\n";
    }
    h << "}\n";
    const auto text = h.str();
    write_bytes(w.output / "adapter_offsets.hpp",
                ByteView(reinterpret_cast<const std::uint8_t*>(text.data()), text.size()));
}
} // namespace

void pack_models(const std::filesystem::path& input, const std::filesystem::path& output,
                 const std::string& pack_id, bool include_transformer)
{
    require(pack_id.size() == 16 && pack_id.find_first_not_of("0123456789abcdef") == std::string::npos,
            "invalid pack ID");
    std::filesystem::create_directories(output);
    Writer w;
    w.output = output;
    w.id = pack_id;
    for (unsigned channels : {1u, 2u})
    {
        const std::string v = channels == 1 ? "mono" : "stereo";
        const auto dac = SourceModel::parse(read_bytes(input / ("dac_" + v + "_q8.bin")));
        const auto tf = SourceModel::parse(read_bytes(input / ("tsac_" + v + "_q8.bin")));
        const auto& out = dac.tensor("decoder.model.6.weight_v").dims;
        require(out.size() == 3 && out[2] == channels, "incompatible model roles");
        const unsigned books = channels == 1 ? 9 : 12;
        require(tf.tensor("codebook_decoder.wpe").dims ==
                    std::vector<std::size_t>{512, books},
                "incompatible model roles");
        pack_dac(w, channels, dac);
        pack_rvq(w, channels, books, dac);
        if (include_transformer)
        {
            pack_transformer(w, channels, books, dac, tf);
        }
    }
    write_adapter_header(w, include_transformer);
    // Build-only staging manifest (src/weights/pack_main.cpp:706-731).
    std::ostringstream m;
    m << "set(TSAC_WEIGHT_FILES\n";
    std::size_t total = 0;
    for (const auto& f : w.files)
    {
        m << '"' << f.name << "\"\n";
        total += f.bytes;
    }
    m << ")\nset(TSAC_WEIGHT_BYTES " << total << ")\n";
    for (const auto& f : w.files)
    {
        m << "set(\"TSAC_WEIGHT_SIZE_" << f.name << "\" " << f.bytes << ")\n";
    }
    const auto manifest = m.str();
    write_bytes(output / "weights-manifest.cmake",
                ByteView(reinterpret_cast<const std::uint8_t*>(manifest.data()), manifest.size()));
    require(total < 400000000, "weight package exceeds 400 MB budget");
}

// ------------------------------------------------------------ package load --
namespace
{
std::vector<std::size_t> numbers_after(const std::string& text, std::size_t start,
                                       const std::string& stop)
{
    const auto end = text.find(stop, start);
    require(end != std::string::npos, "malformed adapter_offsets.hpp");
    std::vector<std::size_t> values;
    std::size_t i = start;
    while (i < end)
    {
        if (std::isdigit(static_cast<unsigned char>(text[i])))
        {
            std::size_t v = 0;
            while (i < end && std::isdigit(static_cast<unsigned char>(text[i])))
            {
                v = v * 10 + static_cast<std::size_t>(text[i] - '0');
                ++i;
            }
            values.push_back(v);
        }
        else
        {
            ++i;
        }
    }
    return values;
}

std::vector<Range> named_ranges(const std::string& text, const std::string& name)
{
    const auto at = text.find("> " + name + "{{");
    require(at != std::string::npos, ("adapter_offsets.hpp lacks " + name).c_str());
    const auto values = numbers_after(text, at + name.size() + 4, "}};");
    require(values.size() % 2 == 0, "malformed adapter_offsets.hpp ranges");
    std::vector<Range> result;
    for (std::size_t i = 0; i < values.size(); i += 2)
    {
        result.push_back({values[i], values[i + 1]});
    }
    return result;
}

template <std::size_t N>
std::vector<std::array<Range, N>> named_rows(const std::string& text, const std::string& name)
{
    const auto flat = named_ranges(text, name);
    require(flat.size() % N == 0, "malformed adapter_offsets.hpp rows");
    std::vector<std::array<Range, N>> rows(flat.size() / N);
    for (std::size_t i = 0; i < flat.size(); ++i)
    {
        rows[i / N][i % N] = flat[i];
    }
    return rows;
}
} // namespace

PackageLayout PackageLayout::parse(const std::string& text)
{
    PackageLayout layout;
    const auto id = text.find("generation_id[]=\"");
    require(id != std::string::npos, "adapter_offsets.hpp lacks generation_id");
    const auto id_end = text.find('"', id + 17);
    layout.generation_id = text.substr(id + 17, id_end - id - 17);
    layout.has_transformer = text.find("has_transformer=true") != std::string::npos;
    auto at = text.find("filenames{{");
    require(at != std::string::npos, "adapter_offsets.hpp lacks filenames");
    at += 11;
    for (auto& name : layout.filenames)
    {
        while (at < text.size() && (text[at] == '\n' || text[at] == ' ' || text[at] == ','))
        {
            ++at;
        }
        if (text.compare(at, 7, "nullptr") == 0)
        {
            at += 7;
        }
        else
        {
            require(text[at] == '"', "malformed adapter_offsets.hpp filenames");
            const auto close = text.find('"', at + 1);
            name = text.substr(at + 1, close - at - 1);
            at = close + 1;
        }
    }
    for (unsigned c : {1u, 2u})
    {
        auto& v = layout.variants[c - 1];
        const std::string p = c == 1 ? "mono_" : "stereo_";
        for (bool synthesis : {false, true})
        {
            auto& d = synthesis ? v.synthesis : v.analysis;
            const auto n = p + (synthesis ? "synthesis" : "analysis");
            d.values = named_ranges(text, n + "_values");
            d.gains = named_ranges(text, n + "_gains");
            d.biases = named_ranges(text, n + "_biases");
            d.alphas = named_ranges(text, n + "_alphas");
        }
        v.books = named_rows<7>(text, p + "books");
        if (layout.has_transformer)
        {
            v.projections = named_rows<3>(text, p + "projections");
            v.norms = named_rows<2>(text, p + "norms");
            const auto t = text.find("model_layout::Transformer " + p + "transformer{");
            require(t != std::string::npos, "adapter_offsets.hpp lacks transformer");
            const auto open = text.find("{{", t);
            const auto values = numbers_after(text, open, "};");
            require(values.size() == 6, "malformed adapter_offsets.hpp transformer");
            v.constants = {Range{values[0], values[1]}, Range{values[2], values[3]}};
            v.embeddings = {values[4], values[5]};
        }
    }
    return layout;
}

Package::Package(std::filesystem::path directory, const Limits& limits)
    : directory_(std::move(directory)), limits_(limits)
{
    const auto bytes = read_bytes(directory_ / "adapter_offsets.hpp");
    layout_ = PackageLayout::parse(std::string(bytes.begin(), bytes.end()));
}

Bytes Package::read(unsigned channels, Role role, Range range) const
{
    require(channels == 1 || channels == 2, "invalid model variant");
    const auto& name = layout_.filenames[(channels - 1) * 10 + role];
    require(!name.empty(), "model file is not included in this package");
    require(checked_add(range.offset, range.bytes) <= limits_.file_bytes,
            "weight mapping exceeds limit");
    const auto path = directory_ / name;
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0)
    {
        throw Error("cannot open weights: " + path.string());
    }
    Bytes bytes(range.bytes);
    std::size_t done = 0;
    while (done < range.bytes)
    {
        const auto n = ::pread(fd, bytes.data() + done, range.bytes - done,
                               static_cast<off_t>(range.offset + done));
        if (n <= 0)
        {
            ::close(fd);
            throw Error("weight file cannot cover requested range: " + path.string());
        }
        done += static_cast<std::size_t>(n);
    }
    ::close(fd);
    return bytes;
}

namespace
{
std::vector<float> as_floats(const Bytes& bytes)
{
    std::vector<float> v(bytes.size() / 4);
    std::memcpy(v.data(), bytes.data(), v.size() * 4);
    return v;
}

std::vector<std::uint16_t> as_halves(const Bytes& bytes)
{
    std::vector<std::uint16_t> v(bytes.size() / 2);
    std::memcpy(v.data(), bytes.data(), v.size() * 2);
    return v;
}
} // namespace

PreparedDac prepare_dac(const Package& package, unsigned channels, bool synthesis,
                        const Limits& limits)
{
    (void)limits;
    const auto& loc = synthesis ? package.layout().variants[channels - 1].synthesis
                                : package.layout().variants[channels - 1].analysis;
    require(loc.values.size() == 30 && loc.alphas.size() == 29, "invalid DAC layout");
    const auto source = synthesis ? dac_synthesis_source : dac_analysis_source;
    const auto shared = synthesis ? dac_synthesis_shared : dac_analysis_shared;
    PreparedDac dac;
    dac.channels = channels;
    dac.synthesis = synthesis;
    for (unsigned i = 0; i < 30; ++i)
    {
        const auto shape = dac_shape(synthesis, channels, i);
        const bool transposed = synthesis && i > 0 && i < 29 && (i - 1) % 7 == 0;
        const auto payload = package.read(channels, source, loc.values[i]);
        std::vector<float> values;
        if (dac_f32(synthesis, i))
        {
            require(payload.size() == shape[0] * shape[1] * shape[2] * 4,
                    "encoded tensor disagrees with contract");
            values = as_floats(payload);
        }
        else
        {
            require(payload.size() == bf8_bytes(shape), "encoded tensor disagrees with contract");
            values = expand_bf8(payload, shape);
        }
        const auto gains = as_floats(package.read(channels, source, loc.gains[i]));
        require(gains.size() == shape[2], "invalid DAC gain shape");
        fold_dac_weight_norm(values, gains, shape[0] * shape[1]);
        PreparedConv conv;
        // Stage/unit geometry (src/common/analysis.tpp:114-155, synthesis.tpp:113-157).
        unsigned stride = 1, dilation = 1;
        if (i > 0 && i < 29)
        {
            const auto stage = (i - 1) / 7, within = (i - 1) % 7;
            if (synthesis)
            {
                if (within == 0)
                {
                    stride = std::array<unsigned, 4>{8, 8, 4, 2}[stage];
                }
                else if ((within - 1) % 2 == 0)
                {
                    dilation = std::array<unsigned, 3>{1, 3, 9}[(within - 1) / 2];
                }
            }
            else
            {
                if (within == 6)
                {
                    stride = std::array<unsigned, 4>{2, 4, 8, 8}[stage];
                }
                else if (within % 2 == 0)
                {
                    dilation = std::array<unsigned, 3>{1, 3, 9}[within / 2];
                }
            }
        }
        const auto kernel = static_cast<unsigned>(shape[1]);
        conv.spec.input_channels = static_cast<unsigned>(transposed ? shape[2] : shape[0]);
        conv.spec.output_channels = static_cast<unsigned>(transposed ? shape[0] : shape[2]);
        conv.spec.kernel = kernel;
        conv.spec.stride = stride;
        conv.spec.dilation = dilation;
        conv.spec.padding = stride == 1 ? (kernel - 1) * dilation / 2 : (stride + 1) / 2;
        conv.spec.transposed = transposed;
        conv.weights = std::move(values);
        conv.bias = as_floats(package.read(channels, shared, loc.biases[i]));
        require(conv.bias.size() == conv.spec.output_channels,
                "normalized convolution shape mismatch");
        require_finite(conv.bias, "nonfinite DSP value");
        dac.convs.push_back(std::move(conv));
    }
    for (unsigned i = 0; i < 29; ++i)
    {
        auto alpha = as_floats(package.read(channels, shared, loc.alphas[i]));
        require(alpha.size() == dac_alpha_width(synthesis, i), "invalid DAC activation shape");
        require_finite(alpha, "nonfinite DSP value");
        dac.alphas.push_back(std::move(alpha));
    }
    return dac;
}

std::vector<PreparedRvqBook> prepare_rvq(const Package& package, unsigned channels,
                                         unsigned books)
{
    const auto& rows = package.layout().variants[channels - 1].books;
    require(books > 0 && books <= rows.size(), "invalid enabled codebook count");
    std::vector<PreparedRvqBook> result(books);
    for (unsigned b = 0; b < books; ++b)
    {
        const auto& row = rows[b];
        auto& r = result[b];
        r.codebook = as_floats(package.read(channels, rvq_shared, row[0]));
        r.output_weights = as_floats(package.read(channels, rvq_shared, row[1]));
        r.output_bias = as_floats(package.read(channels, rvq_shared, row[2]));
        r.search = as_floats(package.read(channels, rvq_encode_shared, row[3]));
        r.input_bias = as_floats(package.read(channels, rvq_encode_shared, row[4]));
        r.input_weights = as_floats(package.read(channels, rvq_encode_apple, row[5]));
        require(r.codebook.size() == 8192 && r.output_weights.size() == 8192 &&
                    r.output_bias.size() == 1024 && r.search.size() == 8192 &&
                    r.input_bias.size() == 8 && r.input_weights.size() == 8192,
                "invalid prepared codebook shape");
    }
    return result;
}

PreparedTransformer prepare_transformer(const Package& package, unsigned channels,
                                        unsigned books)
{
    const auto& layout = package.layout();
    require(layout.has_transformer, "Transformer assets were disabled");
    const auto& v = layout.variants[channels - 1];
    require(books > 0 && books <= (channels == 1 ? 9u : 12u), "invalid enabled codebook count");
    require(v.projections.size() == 63 && v.norms.size() == 32, "invalid Transformer layout");
    PreparedTransformer t;
    t.channels = channels;
    t.books = books;
    for (unsigned p = 0; p < 63; ++p)
    {
        const auto shape = projection_shape(p);
        PreparedLinear l;
        l.input = static_cast<unsigned>(shape[0]);
        l.output = static_cast<unsigned>(shape[1]);
        const auto w = package.read(channels, transformer_source, v.projections[p][0]);
        require(w.size() == shape[0] * shape[1], "stored tensor length disagrees with model contract");
        l.weights.resize(w.size());
        std::memcpy(l.weights.data(), w.data(), w.size());
        l.scales = as_floats(package.read(channels, transformer_shared, v.projections[p][1]));
        l.bias = as_floats(package.read(channels, transformer_shared, v.projections[p][2]));
        require(l.scales.size() == shape[0] / 256 * shape[1] && l.bias.size() == shape[1],
                "invalid generated linear constants");
        t.projections.push_back(std::move(l));
    }
    for (unsigned n = 0; n < 32; ++n)
    {
        t.norms.push_back({as_halves(package.read(channels, transformer_shared, v.norms[n][0])),
                           as_halves(package.read(channels, transformer_shared, v.norms[n][1]))});
        require(t.norms.back().gain.size() == 512 && t.norms.back().bias.size() == 512,
                "invalid normalization shape");
    }
    Range positions = v.constants[0];
    positions.bytes = std::size_t{512} * books * 2;
    t.positions = as_halves(package.read(channels, transformer_shared, positions));
    t.rotations = as_halves(package.read(channels, transformer_shared, v.constants[1]));
    require(t.rotations.size() == 128 * 1024, "invalid rotary shape");
    Range embeddings{v.embeddings.offset, std::size_t{books} * 1024 * 1024 * 2};
    t.embeddings = as_halves(package.read(channels, transformer_shared, embeddings));
    return t;
}
} // namespace tsacb
