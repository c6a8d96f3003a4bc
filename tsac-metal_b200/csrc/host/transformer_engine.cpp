#include "transformer_engine.hpp"

#include "kernel_timer.hpp"

#include "kernels/decode_loop.cuh"
#include "kernels/error_bits.hpp"
#include "kernels/range_decode.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/qlinear.cuh"
#include "kernels/transformer_ops.cuh"

#include <algorithm>
#include <cstdlib>
#include <deque>

namespace tsacb
{
namespace
{
using dev::RowMeta;

constexpr int context = 1024, replay_frames = 256;

int norm_index(bool temporal, int layer, bool mlp) // src/models/contract.cpp:191-196
{
    return (temporal ? 0 : 25) + layer * 2 + (mlp ? 1 : 0);
}

int final_norm(bool temporal)
{
    return temporal ? 24 : 31;
}

int projection_index(bool temporal, int layer, int op) // src/models/contract.cpp:185-189
{
    return (temporal ? 0 : 48) + layer * 4 + op;
}
} // namespace

DeviceTransformer::DeviceTransformer(const PreparedTransformer& t, cudaStream_t stream)
    : channels(t.channels), books(t.books)
{
    for (const auto& p : t.projections)
    {
        DeviceLinear l;
        l.input = static_cast<int>(p.input);
        l.output = static_cast<int>(p.output);
        l.weights = upload(p.weights, stream);
        l.scales = upload(p.scales, stream);
        l.bias = upload(p.bias, stream);
        projections.push_back(std::move(l));
    }
    for (const auto& n : t.norms)
    {
        norm_gain.push_back(upload(n.gain, stream));
        norm_bias.push_back(upload(n.bias, stream));
    }
    positions = upload(t.positions, stream);
    rotations = upload(t.rotations, stream);
    embeddings = upload(t.embeddings, stream);
    gelu.resize(65536 * 2);
    dev::build_gelu_table(gelu.as<std::uint16_t>(), stream);
    cuda_ok(cudaGetLastError(), "transformer weight upload");
    cuda_ok(cudaStreamSynchronize(stream), "transformer weight upload");
}

TransformerEngine::TransformerEngine(std::shared_ptr<const DeviceTransformer> model,
                                     cudaStream_t stream)
    : model_(std::move(model)), stream_(stream), error_(sizeof(unsigned))
{
    cuda_ok(cudaMemsetAsync(error_.as<void>(), 0, sizeof(unsigned), stream_), "memset");
}

void TransformerEngine::check_errors()
{
    unsigned word = 0;
    cuda_ok(cudaMemcpyAsync(&word, error_.as<void>(), sizeof(word), cudaMemcpyDeviceToHost, stream_),
            "error word");
    cuda_ok(cudaStreamSynchronize(stream_), "transformer");
    if (word)
    {
        cuda_ok(cudaMemsetAsync(error_.as<void>(), 0, sizeof(unsigned), stream_), "memset");
        throw NumericError("Transformer activations must be finite");
    }
}

void TransformerEngine::quantize(const std::uint16_t* x, int rows, int k, std::int8_t* xq, float* xs)
{
    KernelTimer::Scope timing("quantize", stream_, 0.0);
    dev::qlinear_quantize(x, rows, k, xq, xs, error_word(), stream_);
}

namespace
{
double linear_work(int rows, double n, double k)
{
    const double m = rows;
    // GEMV-shaped launches are weight-streaming (bytes); GEMM launches count int8 ops.
    return dev::qlinear_uses_gemm(rows, static_cast<int>(n), static_cast<int>(k))
               ? 2.0 * m * n * k
               : n * k + 4 * n * k / 256 + 4 * n + m * k + 4 * m * k / 256 + 2 * m * n;
}
} // namespace

void TransformerEngine::run_linear(int projection, const std::int8_t* xq, const float* xs,
                                   int rows, std::uint16_t* y, const std::uint16_t* residual,
                                   bool gelu, int residual_stride)
{
    const auto& l = model_->projections.at(static_cast<std::size_t>(projection));
    dev::QLinearArgs a;
    a.weights = l.weights.as<std::int8_t>();
    a.weight_scales = l.scales.as<float>();
    a.bias = l.bias.as<float>();
    a.xq = xq;
    a.xscale = xs;
    a.residual = residual;
    a.lut = gelu ? model_->gelu.as<std::uint16_t>() : nullptr;
    a.y = y;
    a.m = rows;
    a.n = l.output;
    a.k = l.input;
    a.residual_stride = residual_stride;
    a.error_word = error_word();
    KernelTimer::Scope timing(dev::qlinear_uses_gemm(rows, l.output, l.input) ? "qlinear_gemm" : "qlinear_small",
                              stream_,
                              linear_work(rows, l.output, l.input));
    dev::qlinear_matmul(a, stream_);
}

void TransformerEngine::run_linear_bf16(int projection, const std::uint16_t* x, int rows,
                                        std::uint16_t* y, const std::uint16_t* residual,
                                        bool gelu, std::int8_t* xq, float* xs)
{
    // A separate BF8L pass: quantizing inside the linear kernel was measured
    // slower on B200 (each CTA re-quantizes its rows on its critical path).
    const auto& l = model_->projections.at(static_cast<std::size_t>(projection));
    quantize(x, rows, static_cast<int>(l.input), xq, xs);
    run_linear(projection, xq, xs, rows, y, residual, gelu);
}

void TransformerEngine::run_qkv(int projection, const std::int8_t* xq, const float* xs, int rows,
                                const dev::RowMeta* meta, std::uint16_t* query,
                                std::uint16_t* cache_k, std::uint16_t* cache_v, std::uint16_t* qkv)
{
    const auto& l = model_->projections.at(static_cast<std::size_t>(projection));
    const auto* rotations = model_->rotations.as<std::uint16_t>();
    if (!dev::qlinear_qkv_fusable(rows, static_cast<int>(l.output)))
    {
        run_linear(projection, xq, xs, rows, qkv, nullptr, false);
        KernelTimer::Scope timing("rotary_scatter", stream_, 0.0);
        dev::rotary_scatter(qkv, meta, rotations, rows, query, cache_k, cache_v, stream_);
        return;
    }
    require(l.output == 1536, "QKV projection must have 1536 outputs");
    dev::QLinearArgs a;
    a.weights = l.weights.as<std::int8_t>();
    a.weight_scales = l.scales.as<float>();
    a.bias = l.bias.as<float>();
    a.xq = xq;
    a.xscale = xs;
    a.m = rows;
    a.n = l.output;
    a.k = l.input;
    a.qkv = dev::QkvScatter{meta, rotations, query, cache_k, cache_v};
    KernelTimer::Scope timing("qlinear_small", stream_, linear_work(rows, l.output, l.input));
    dev::qlinear_matmul(a, stream_);
}

// evaluate_stack (src/common/cpu_transformer.tpp:99-141) over a set of rows.
void TransformerEngine::run_stack(Workspace& ws_, bool temporal, int rows, std::uint16_t* h,
                                  const void* meta_device,
                                  int max_time, std::uint16_t* cache_k, std::uint16_t* cache_v,
                                  std::size_t cache_layer_stride, std::uint16_t* final_out,
                                  std::int8_t* final_q, float* final_s, bool sequence_rows)
{
    const auto* meta = static_cast<const RowMeta*>(meta_device);
    const int layers = temporal ? 12 : 3;
    auto* xq = ws_.get<std::int8_t>("xq", static_cast<std::size_t>(rows) * 2048);
    auto* xs = ws_.get<float>("xs", static_cast<std::size_t>(rows) * 8);
    auto* qkv = ws_.get<std::uint16_t>("qkv", static_cast<std::size_t>(rows) * 1536);
    auto* query = ws_.get<std::uint16_t>("query", static_cast<std::size_t>(rows) * 512);
    auto* att = ws_.get<std::uint16_t>("att", static_cast<std::size_t>(rows) * 512);
    auto* mlp = ws_.get<std::uint16_t>("mlp", static_cast<std::size_t>(rows) * 2048);
    auto* partials = ws_.get<float>("partials", dev::attention_partials_bytes(rows, max_time) / 4);
    for (int l = 0; l < layers; ++l)
    {
        const int n1 = norm_index(temporal, l, false), n2 = norm_index(temporal, l, true);
        auto* ck = cache_k + cache_layer_stride * static_cast<std::size_t>(l);
        auto* cv = cache_v + cache_layer_stride * static_cast<std::size_t>(l);
        {
            KernelTimer::Scope timing("layer_norm", stream_, 0.0);
            dev::layer_norm(h, model_->norm_gain[n1].as<std::uint16_t>(),
                            model_->norm_bias[n1].as<std::uint16_t>(), rows, nullptr, xq, xs,
                            error_word(), stream_);
        }
        run_qkv(projection_index(temporal, l, 0), xq, xs, rows, meta, query, ck, cv, qkv);
        bool quantized = false; // one-block histories: attention emits the BF8L input itself
        {
            KernelTimer::Scope timing("attention", stream_, 0.0);
            quantized = dev::attention(query, meta, ck, cv, rows, max_time, partials, att, stream_, xq, xs,
                                       error_word(), sequence_rows);
        }
        if (quantized)
            run_linear(projection_index(temporal, l, 1), xq, xs, rows, h, h, false);
        else
            run_linear_bf16(projection_index(temporal, l, 1), att, rows, h, h, false, xq, xs);
        {
            KernelTimer::Scope timing("layer_norm", stream_, 0.0);
            dev::layer_norm(h, model_->norm_gain[n2].as<std::uint16_t>(),
                            model_->norm_bias[n2].as<std::uint16_t>(), rows, nullptr, xq, xs,
                            error_word(), stream_);
        }
        run_linear(projection_index(temporal, l, 2), xq, xs, rows, mlp, nullptr, true);
        run_linear_bf16(projection_index(temporal, l, 3), mlp, rows, h, h, false, xq, xs);
    }
    const int f = final_norm(temporal);
    dev::layer_norm(h, model_->norm_gain[f].as<std::uint16_t>(),
                    model_->norm_bias[f].as<std::uint16_t>(), rows, final_out, final_q, final_s,
                    error_word(), stream_);
}

void TransformerEngine::predict_known(const Header& header, std::span<const std::uint16_t> tokens,
                                      std::uint16_t* q15, float* probabilities)
{
    check_header(header);
    require(header.method == 1, "Transformer predictor requires normal framing");
    require(header.model_channels == model_->channels && header.codebooks <= model_->books,
            "Transformer stream/model mismatch");
    require(tokens.size() == header.symbol_count(), "normal token count does not match header");
    for (auto t : tokens)
    {
        require(t < 1024, "Transformer feedback token exceeds alphabet");
    }
    const int F = static_cast<int>(header.frames), G = header.groups, Q = header.codebooks;
    const int B = header.batch;
    const int lanes_b = std::min(B, F);
    const int base = F / B, extra = F % B;

    // ---- temporal rows: the per-step schedule of TransformerPredictor::prepare
    // (src/common/transformer.cpp:106-142) flattened into sequences.
    std::vector<RowMeta> tmeta;
    std::vector<int> toffsets, tcounts;
    std::vector<int> cond_row(static_cast<std::size_t>(F) * G, -1);
    // Token pool: the recording's tokens followed by one all-zero frame.
    std::vector<std::uint16_t> pool(tokens.begin(), tokens.end());
    const int zero_frame = static_cast<int>(pool.size());
    pool.resize(pool.size() + static_cast<std::size_t>(Q), 0);
    int next_slot = 0, max_time = 1;
    for (int lane = 0; lane < lanes_b; ++lane)
    {
        const int length = base + (lane < extra);
        const int start = lane * base + std::min(lane, extra);
        for (int g = 0; g < G; ++g)
        {
            int used = 0, segment = next_slot;
            std::deque<int> history;
            const auto add = [&](int feedback_offset, bool replay)
            {
                const int position = used++;
                const int slot = segment + position;
                tmeta.push_back({slot, segment, position + 1, position,
                                 (position + 1 > 64 || replay) ? 1 : 0});
                toffsets.push_back(feedback_offset);
                tcounts.push_back(Q);
                next_slot = std::max(next_slot, slot + 1);
                max_time = std::max(max_time, position + 1);
            };
            for (int s = 0; s < length; ++s)
            {
                const int f = start + s;
                if (used == context)
                {
                    segment = next_slot;
                    used = 0;
                    for (int h : history)
                    {
                        add((h * G + g) * Q, true);
                    }
                }
                else
                {
                    add(s == 0 ? zero_frame : ((f - 1) * G + g) * Q, false);
                }
                cond_row[static_cast<std::size_t>(f) * G + g] = static_cast<int>(tmeta.size()) - 1;
                history.push_back(f);
                if (static_cast<int>(history.size()) > replay_frames)
                {
                    history.pop_front();
                }
            }
        }
    }
    const int trows = static_cast<int>(tmeta.size());
    auto s = stream_;
    auto* d_pool = ws_.get<std::uint16_t>("pool", pool.size());
    cuda_ok(cudaMemcpyAsync(d_pool, pool.data(), pool.size() * 2, cudaMemcpyHostToDevice, s), "H2D");
    auto* d_tmeta = ws_.get<RowMeta>("tmeta", tmeta.size());
    cuda_ok(cudaMemcpyAsync(d_tmeta, tmeta.data(), tmeta.size() * sizeof(RowMeta), cudaMemcpyHostToDevice, s), "H2D");
    auto* d_toff = ws_.get<int>("toff", toffsets.size());
    cuda_ok(cudaMemcpyAsync(d_toff, toffsets.data(), toffsets.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
    auto* d_tcnt = ws_.get<int>("tcnt", tcounts.size());
    cuda_ok(cudaMemcpyAsync(d_tcnt, tcounts.data(), tcounts.size() * 4, cudaMemcpyHostToDevice, s), "H2D");

    // Temporal stack: feedback embedding -> cb_proj -> 12 layers -> ln_f.
    auto* emb = ws_.get<std::uint16_t>("emb", static_cast<std::size_t>(trows) * 1024);
    dev::embed_sum(model_->embeddings.as<std::uint16_t>(), d_pool, d_toff, d_tcnt, trows, emb, s);
    auto* eq = ws_.get<std::int8_t>("eq", static_cast<std::size_t>(trows) * 1024);
    auto* es = ws_.get<float>("es", static_cast<std::size_t>(trows) * 4);
    auto* th = ws_.get<std::uint16_t>("th", static_cast<std::size_t>(trows) * 512);
    run_linear_bf16(60, emb, trows, th, nullptr, false, eq, es);
    const std::size_t tstride = static_cast<std::size_t>(next_slot) * 512;
    auto* tck = ws_.get<std::uint16_t>("tck", tstride * 12);
    auto* tcv = ws_.get<std::uint16_t>("tcv", tstride * 12);
    auto* cond = ws_.get<std::uint16_t>("cond", static_cast<std::size_t>(trows) * 512);
    run_stack(ws_, true, trows, th, d_tmeta, max_time, tck, tcv, tstride, cond, nullptr, nullptr, true);

    // ---- codebook stack, chunked by (frame, group) sequences of Q rows
    // (2048 sequences per launch group bound the per-chunk scratch).
    const int sequences = F * G;
    constexpr int chunk = 2048;
    for (int first = 0; first < sequences; first += chunk)
    {
        const int count = std::min(chunk, sequences - first);
        const int rows = count * Q;
        std::vector<RowMeta> cmeta(static_cast<std::size_t>(rows));
        std::vector<int> src0(static_cast<std::size_t>(count)), zero_books(static_cast<std::size_t>(count), 0);
        std::vector<int> poff, pcnt, pbook, pid;
        std::vector<int> token_index(static_cast<std::size_t>(rows));
        // Row order: all book-0 rows, then books >= 1 sequence by sequence.
        for (int i = 0; i < count; ++i)
        {
            const int fg = first + i;
            src0[static_cast<std::size_t>(i)] = cond_row[static_cast<std::size_t>(fg)];
            cmeta[static_cast<std::size_t>(i)] = {i * Q, i * Q, 1, -1, 0};
            token_index[static_cast<std::size_t>(i)] = fg * Q;
        }
        int r = count;
        for (int i = 0; i < count; ++i)
        {
            const int fg = first + i;
            for (int b = 1; b < Q; ++b, ++r)
            {
                cmeta[static_cast<std::size_t>(r)] = {i * Q + b, i * Q, b + 1, -1, 0};
                poff.push_back(fg * Q);
                pcnt.push_back(b);
                pbook.push_back(b);
                pid.push_back(static_cast<int>(pid.size()));
                token_index[static_cast<std::size_t>(r)] = fg * Q + b;
            }
        }
        const int prows = rows - count;
        auto* d_cmeta = ws_.get<RowMeta>("cmeta", cmeta.size());
        cuda_ok(cudaMemcpyAsync(d_cmeta, cmeta.data(), cmeta.size() * sizeof(RowMeta), cudaMemcpyHostToDevice, s), "H2D");
        auto* d_src0 = ws_.get<int>("src0", src0.size());
        cuda_ok(cudaMemcpyAsync(d_src0, src0.data(), src0.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
        auto* d_zero = ws_.get<int>("zbook", zero_books.size());
        cuda_ok(cudaMemcpyAsync(d_zero, zero_books.data(), zero_books.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
        auto* d_tidx = ws_.get<int>("tidx", token_index.size());
        cuda_ok(cudaMemcpyAsync(d_tidx, token_index.data(), token_index.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
        auto* ch = ws_.get<std::uint16_t>("ch", static_cast<std::size_t>(rows) * 512);
        dev::add_positions(cond, d_src0, d_zero, model_->positions.as<std::uint16_t>(), count, ch, s);
        if (prows > 0)
        {
            auto* d_poff = ws_.get<int>("poff", poff.size());
            cuda_ok(cudaMemcpyAsync(d_poff, poff.data(), poff.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
            auto* d_pcnt = ws_.get<int>("pcnt", pcnt.size());
            cuda_ok(cudaMemcpyAsync(d_pcnt, pcnt.data(), pcnt.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
            auto* d_pbook = ws_.get<int>("pbook", pbook.size());
            cuda_ok(cudaMemcpyAsync(d_pbook, pbook.data(), pbook.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
            auto* d_pid = ws_.get<int>("pid", pid.size());
            cuda_ok(cudaMemcpyAsync(d_pid, pid.data(), pid.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
            auto* pemb = ws_.get<std::uint16_t>("pemb", static_cast<std::size_t>(prows) * 1024);
            dev::embed_sum(model_->embeddings.as<std::uint16_t>(), d_pool, d_poff, d_pcnt, prows, pemb, s);
            auto* pq = ws_.get<std::int8_t>("pq", static_cast<std::size_t>(prows) * 1024);
            auto* ps = ws_.get<float>("ps", static_cast<std::size_t>(prows) * 4);
            auto* pproj = ws_.get<std::uint16_t>("pproj", static_cast<std::size_t>(prows) * 512);
            run_linear_bf16(61, pemb, prows, pproj, nullptr, false, pq, ps);
            dev::add_positions(pproj, d_pid, d_pbook, model_->positions.as<std::uint16_t>(), prows,
                               ch + static_cast<std::size_t>(count) * 512, s);
        }
        const std::size_t cstride = static_cast<std::size_t>(rows) * 512;
        auto* cck = ws_.get<std::uint16_t>("cck", cstride * 3);
        auto* ccv = ws_.get<std::uint16_t>("ccv", cstride * 3);
        auto* fq = ws_.get<std::int8_t>("fq", static_cast<std::size_t>(rows) * 512);
        auto* fs = ws_.get<float>("fs", static_cast<std::size_t>(rows) * 2);
        run_stack(ws_, false, rows, ch, d_cmeta, Q, cck, ccv, cstride, nullptr, fq, fs);
        auto* logits = ws_.get<std::uint16_t>("logits", static_cast<std::size_t>(rows) * 1024);
        run_linear(62, fq, fs, rows, logits, nullptr, false);
        auto* tree = ws_.get<float>("tree", static_cast<std::size_t>(rows) * 1023);
        float* probs = probabilities ? ws_.get<float>("probs", static_cast<std::size_t>(rows) * 1024) : nullptr;
        dev::softmax_tree(logits, rows, nullptr, probs, tree, error_word(), s);
        auto* dq = ws_.get<std::uint16_t>("q15", static_cast<std::size_t>(rows) * 10);
        dev::categorical_path_q15(tree, d_pool, d_tidx, rows, dq, s);
        cuda_ok(cudaGetLastError(), "transformer launch");
        std::vector<std::uint16_t> hq(static_cast<std::size_t>(rows) * 10);
        cuda_ok(cudaMemcpyAsync(hq.data(), dq, hq.size() * 2, cudaMemcpyDeviceToHost, s), "D2H");
        std::vector<float> hp;
        if (probabilities)
        {
            hp.resize(static_cast<std::size_t>(rows) * 1024);
            cuda_ok(cudaMemcpyAsync(hp.data(), probs, hp.size() * 4, cudaMemcpyDeviceToHost, s), "D2H");
        }
        check_errors();
        for (int i = 0; i < rows; ++i)
        {
            const auto t = static_cast<std::size_t>(token_index[static_cast<std::size_t>(i)]);
            std::copy_n(hq.data() + static_cast<std::size_t>(i) * 10, 10, q15 + t * 10);
            if (probabilities)
            {
                std::copy_n(hp.data() + static_cast<std::size_t>(i) * 1024, 1024, probabilities + t * 1024);
            }
        }
    }
}

// ------------------------------------------------------------------ decode --
namespace
{
// Device row buffers of one decode step (decode_setup writes them), laid out
// in one allocation for `rows` codebook rows and `temporal` temporal rows.
struct StepRowsLayout
{
    std::size_t tmeta, toffsets, tcounts, csource, clane, cmeta, clanes, cbooks, coffsets, ccounts, dest, bytes;
    StepRowsLayout(std::size_t rows, std::size_t temporal)
    {
        std::size_t at = 0;
        const auto take = [&](std::size_t n)
        {
            const auto here = at;
            at = align_up(at + n, 256);
            return here;
        };
        tmeta = take(temporal * sizeof(RowMeta));
        toffsets = take(temporal * 4);
        tcounts = take(temporal * 4);
        csource = take(rows * 4);
        clane = take(rows * 4);
        cmeta = take(rows * sizeof(RowMeta));
        clanes = take(rows * 4);
        cbooks = take(rows * 4);
        coffsets = take(rows * 4);
        ccounts = take(rows * 4);
        dest = take(rows * 4);
        bytes = at;
    }
    dev::DecodeStepRows at(char* base) const
    {
        return {reinterpret_cast<RowMeta*>(base + tmeta), reinterpret_cast<int*>(base + toffsets),
                reinterpret_cast<int*>(base + tcounts),   reinterpret_cast<int*>(base + csource),
                reinterpret_cast<int*>(base + clane),     reinterpret_cast<RowMeta*>(base + cmeta),
                reinterpret_cast<int*>(base + clanes),    reinterpret_cast<int*>(base + cbooks),
                reinterpret_cast<int*>(base + coffsets),  reinterpret_cast<int*>(base + ccounts),
                reinterpret_cast<int*>(base + dest)};
    }
};
} // namespace

struct TransformerEngine::DecodeState
{
    std::vector<Header> headers;
    std::vector<dev::DecodeLane> lanes;
    std::vector<int> lengths;        // frames per lane
    std::vector<int> step_position;  // per step: temporal position, -1 = context replay
    std::vector<std::size_t> token_base;
    std::size_t tstride = 0, cstride = 0, total_tokens = 0;
    int max_books = 0;
    Workspace ws; // sized once per call: graph-captured pointers stay valid
    std::uint16_t *tck = nullptr, *tcv = nullptr, *cck = nullptr, *ccv = nullptr, *cond = nullptr;
    std::uint16_t* tokens = nullptr; // batch token array + 12 zero tokens
    int zero_row = 0;
    std::uint8_t* payload = nullptr;
    std::uint64_t *offsets = nullptr, *sizes = nullptr;
    dev::RangeCursor* cursors = nullptr;
    dev::DecodeLane* d_lanes = nullptr;
    dev::DecodeClock* clock = nullptr;
    int* d_step_position = nullptr;
    dev::DecodeStepRows rows{};
    struct Shape
    {
        DeviceBuffer row_lane, row_begin;
        int rows = 0;
    };
    // (book, active lanes, temporal rows per lane): the lanes active at a
    // step are those longer than it, so the count names the set.
    std::map<std::tuple<int, int, int>, Shape> shapes;
    // One graph per step shape (active lanes, temporal rows per lane) holding
    // every book of the step, so consecutive books' kernels overlap through
    // programmatic dependent launch instead of meeting at graph boundaries.
    struct StepGraph
    {
        cudaGraphExec_t exec = nullptr;
        unsigned long long kernels = 0; // kernel nodes, for the launch tally
    };
    std::map<std::pair<int, int>, StepGraph> step_graphs;

    ~DecodeState()
    {
        for (auto& [key, graph] : step_graphs)
            if (graph.exec)
                cudaGraphExecDestroy(graph.exec);
    }
};

TransformerEngine::~TransformerEngine() = default;

void TransformerEngine::decode_streams(const std::vector<Header>& headers, const std::vector<ByteView>& payloads,
                                       std::vector<std::vector<std::uint16_t>>& tokens)
{
    require(headers.size() == payloads.size(), "decode: one payload per header");
    tokens.assign(headers.size(), {});
    if (headers.empty())
        return;
    decode_ = std::make_unique<DecodeState>();
    auto& st = *decode_;
    auto s = stream_;
    st.headers = headers;
    int tslots = 0, cslots = 0;
    std::size_t payload_bytes = 0;
    for (std::size_t r = 0; r < headers.size(); ++r)
    {
        const auto& h = headers[r];
        check_header(h);
        require(h.method == 1 && h.model_channels == model_->channels && h.codebooks <= model_->books,
                "Transformer stream/model mismatch");
        require(payloads[r].size() == h.payload_bytes, "decode: payload size does not match header");
        st.token_base.push_back(st.total_tokens);
        st.total_tokens = checked_add(st.total_tokens, h.symbol_count());
        payload_bytes = checked_add(payload_bytes, align_up(h.payload_bytes, 16));
        st.max_books = std::max<int>(st.max_books, h.codebooks);
        const LaneSchedule schedule(h);
        for (std::size_t lane = 0; lane < schedule.lanes; ++lane)
            for (int g = 0; g < h.groups; ++g)
            {
                require(st.token_base[r] <= 0x7fffffffu, "decode batch exceeds 2^31 tokens");
                st.lanes.push_back({static_cast<int>(r), g, h.groups, h.codebooks,
                                    static_cast<int>(schedule.first_frame(lane)), tslots, cslots,
                                    static_cast<int>(st.token_base[r])});
                st.lengths.push_back(static_cast<int>(schedule.length(lane)));
                tslots += context;
                cslots += h.codebooks;
            }
    }
    require(st.total_tokens + 16 <= 0x7fffffffu, "decode batch exceeds 2^31 tokens");
    const int steps = *std::max_element(st.lengths.begin(), st.lengths.end());
    // Temporal positions: TransformerPredictor's context use, the same for
    // every lane (all lanes start at step 0): positions 0..1023, then a
    // replay of the last 256 frames at positions 0..255, and so on.
    bool replay = false;
    for (int step = 0, used = 0; step < steps; ++step)
    {
        if (used == context)
        {
            st.step_position.push_back(-1);
            used = replay_frames;
            replay = true;
        }
        else
        {
            st.step_position.push_back(used++);
        }
    }
    const int lane_count = static_cast<int>(st.lanes.size());
    const int temporal_cap = lane_count * (replay ? replay_frames : 1);
    const auto cap = static_cast<std::size_t>(temporal_cap);
    st.tstride = static_cast<std::size_t>(tslots) * 512;
    st.cstride = static_cast<std::size_t>(cslots) * 512;
    auto& ws = st.ws;
    st.tck = ws.get<std::uint16_t>("tck", st.tstride * 12);
    st.tcv = ws.get<std::uint16_t>("tcv", st.tstride * 12);
    st.cck = ws.get<std::uint16_t>("cck", st.cstride * 3);
    st.ccv = ws.get<std::uint16_t>("ccv", st.cstride * 3);
    st.cond = ws.get<std::uint16_t>("cond", static_cast<std::size_t>(lane_count) * 512);
    // Every scratch name at its call maximum, so no pointer moves later.
    ws.get<std::int8_t>("xq", cap * 2048);
    ws.get<float>("xs", cap * 8);
    ws.get<std::uint16_t>("qkv", cap * 1536);
    ws.get<std::uint16_t>("query", cap * 512);
    ws.get<std::uint16_t>("att", cap * 512);
    ws.get<std::uint16_t>("mlp", cap * 2048);
    ws.get<float>("partials", dev::attention_partials_bytes(static_cast<int>(cap), context) / 4);
    for (const char* name : {"emb", "pemb"})
        ws.get<std::uint16_t>(name, cap * 1024);
    for (const char* name : {"eq", "pq"})
        ws.get<std::int8_t>(name, cap * 1024);
    for (const char* name : {"es", "ps"})
        ws.get<float>(name, cap * 4);
    for (const char* name : {"th", "tout", "ch"})
        ws.get<std::uint16_t>(name, cap * 512);
    ws.get<std::int8_t>("fq", cap * 512);
    ws.get<float>("fs", cap * 2);
    ws.get<std::uint16_t>("logits", cap * 1024);
    ws.get<float>("tree", cap * 1023);
    const StepRowsLayout layout(static_cast<std::size_t>(lane_count), cap);
    st.rows = layout.at(ws.get<char>("step_rows", layout.bytes));
    // Batch token array (+ 16 zero tokens: the feedback before frame 0).
    st.zero_row = static_cast<int>(st.total_tokens);
    st.tokens = ws.get<std::uint16_t>("tokens", st.total_tokens + 16);
    cuda_ok(cudaMemsetAsync(st.tokens, 0, (st.total_tokens + 16) * 2, s), "memset");
    // Range decoders: payloads, cursors.
    std::vector<std::uint8_t> packed(payload_bytes);
    std::vector<std::uint64_t> offs, sizes;
    for (std::size_t r = 0, at = 0; r < headers.size(); ++r)
    {
        std::copy(payloads[r].begin(), payloads[r].end(), packed.begin() + static_cast<std::ptrdiff_t>(at));
        offs.push_back(at);
        sizes.push_back(payloads[r].size());
        at += align_up(payloads[r].size(), 16);
    }
    st.payload = ws.get<std::uint8_t>("payload", packed.size() + 16);
    st.offsets = ws.get<std::uint64_t>("payload_offsets", offs.size());
    st.sizes = ws.get<std::uint64_t>("payload_sizes", sizes.size());
    st.cursors = ws.get<dev::RangeCursor>("cursors", headers.size());
    st.d_lanes = ws.get<dev::DecodeLane>("lanes", st.lanes.size());
    st.clock = ws.get<dev::DecodeClock>("clock", 1);
    st.d_step_position = ws.get<int>("step_position", st.step_position.size());
    cuda_ok(cudaMemcpyAsync(st.payload, packed.data(), packed.size(), cudaMemcpyHostToDevice, s), "H2D");
    cuda_ok(cudaMemcpyAsync(st.offsets, offs.data(), offs.size() * 8, cudaMemcpyHostToDevice, s), "H2D");
    cuda_ok(cudaMemcpyAsync(st.sizes, sizes.data(), sizes.size() * 8, cudaMemcpyHostToDevice, s), "H2D");
    cuda_ok(cudaMemcpyAsync(st.d_lanes, st.lanes.data(), st.lanes.size() * sizeof(dev::DecodeLane),
                            cudaMemcpyHostToDevice, s),
            "H2D");
    cuda_ok(cudaMemcpyAsync(st.d_step_position, st.step_position.data(), st.step_position.size() * 4,
                            cudaMemcpyHostToDevice, s),
            "H2D");
    cuda_ok(cudaMemsetAsync(st.clock, 0, sizeof(dev::DecodeClock), s), "memset");
    dev::range_start(st.payload, st.offsets, st.sizes, st.cursors, static_cast<int>(headers.size()),
                     error_word(), s);
    cuda_ok(cudaStreamSynchronize(s), "decode setup"); // host staging vectors go out of scope

    // TSAC_CUDA_DECODE_GRAPHS=0 runs every step's kernels directly (each
    // kernel family then shows in the kernel timing).
    static const bool graphs_enabled = []
    {
        const char* e = std::getenv("TSAC_CUDA_DECODE_GRAPHS");
        return !(e && e[0] == '0');
    }();
    // Algorithmic bytes of one step: the int8 weights it streams.
    const auto weights = [&](int p)
    {
        const auto& l = model_->projections[static_cast<std::size_t>(p)];
        return static_cast<double>(l.input) * l.output;
    };
    double codebook_bytes = weights(61) + weights(62), temporal_bytes = weights(60);
    for (int p = 48; p < 60; ++p)
        codebook_bytes += weights(p);
    for (int p = 0; p < 48; ++p)
        temporal_bytes += weights(p);

    // Row data of (book, active lanes, temporal rows per lane): lanes longer
    // than the step whose recording has the book, in stream order; each
    // recording's rows are consecutive.
    const auto shape_of = [&](int step, int book, int active, int per_lane) -> DecodeState::Shape&
    {
        const auto key = std::make_tuple(book, active, book == 0 ? per_lane : 1);
        auto found = st.shapes.find(key);
        if (found != st.shapes.end())
            return found->second;
        DecodeState::Shape shape;
        std::vector<int> row_lane;
        std::vector<int> row_begin(headers.size() + 1, 0);
        for (int i = 0; i < lane_count; ++i)
        {
            const auto& lane = st.lanes[static_cast<std::size_t>(i)];
            if (st.lengths[static_cast<std::size_t>(i)] > step && book < lane.books)
            {
                row_lane.push_back(i);
                ++row_begin[static_cast<std::size_t>(lane.recording) + 1];
            }
        }
        for (std::size_t r = 0; r < headers.size(); ++r)
            row_begin[r + 1] += row_begin[r];
        shape.rows = static_cast<int>(row_lane.size());
        shape.row_lane.resize(std::max<std::size_t>(row_lane.size(), 1) * 4);
        shape.row_begin.resize(row_begin.size() * 4);
        cuda_ok(cudaMemcpy(shape.row_lane.as<void>(), row_lane.data(), row_lane.size() * 4, cudaMemcpyHostToDevice),
                "H2D");
        cuda_ok(cudaMemcpy(shape.row_begin.as<void>(), row_begin.data(), row_begin.size() * 4,
                           cudaMemcpyHostToDevice),
                "H2D");
        return st.shapes.emplace(key, std::move(shape)).first->second;
    };

    for (int step = 0; step < steps; ++step)
    {
        int active = 0;
        for (const int length : st.lengths)
            active += length > step;
        const int per_lane = st.step_position[static_cast<std::size_t>(step)] < 0 ? replay_frames : 1;
        std::vector<DecodeState::Shape*> books;
        double step_bytes = 0.0;
        for (int book = 0; book < st.max_books; ++book)
        {
            auto& sh = shape_of(step, book, active, per_lane);
            books.push_back(&sh);
            if (sh.rows > 0)
                step_bytes += codebook_bytes + (book == 0 ? temporal_bytes : 0.0);
        }
        const auto enqueue_books = [&]
        {
            for (int book = 0; book < st.max_books; ++book)
            {
                const auto& sh = *books[static_cast<std::size_t>(book)];
                if (sh.rows > 0)
                    enqueue_decode_step(sh.row_lane.as<int>(), sh.row_begin.as<int>(), sh.rows, book,
                                        book == 0 ? per_lane : 1);
            }
        };
        if (!graphs_enabled)
        {
            KernelTimer::Scope timing("decode_step", s, step_bytes);
            enqueue_books();
            continue;
        }
        auto& graph = st.step_graphs[std::make_pair(active, per_lane)];
        if (!graph.exec)
        {
            cudaGraph_t captured = nullptr;
            {
                dev::CaptureTally tally;
                cuda_ok(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "capture");
                enqueue_books();
                cuda_ok(cudaStreamEndCapture(s, &captured), "capture");
                graph.kernels = tally.kernels();
            }
            const auto status = cudaGraphInstantiate(&graph.exec, captured, 0);
            cudaGraphDestroy(captured);
            cuda_ok(status, "cudaGraphInstantiate");
        }
        if (graph.kernels == 0)
            continue;
        KernelTimer::Scope timing("decode_step", s, step_bytes);
        cuda_ok(cudaGraphLaunch(graph.exec, s), "cudaGraphLaunch");
        dev::note_launch(graph.kernels);
    }
    unsigned word = 0;
    cuda_ok(cudaMemcpyAsync(&word, error_word(), 4, cudaMemcpyDeviceToHost, s), "D2H");
    for (std::size_t r = 0; r < headers.size(); ++r)
    {
        tokens[r].resize(headers[r].symbol_count());
        cuda_ok(cudaMemcpyAsync(tokens[r].data(), st.tokens + st.token_base[r], tokens[r].size() * 2,
                                cudaMemcpyDeviceToHost, s),
                "D2H");
    }
    cuda_ok(cudaStreamSynchronize(s), "decode loop");
    if (word)
    {
        cuda_ok(cudaMemset(error_word(), 0, 4), "memset");
        if (word & dev::error_nonfinite)
            throw NumericError("Transformer activations must be finite");
        throw Error("range code outside interval");
    }
}

void TransformerEngine::enqueue_decode_step(const int* row_lane, const int* row_begin, int n, int book,
                                            int per_lane)
{
    auto& st = *decode_;
    auto& ws = st.ws;
    auto s = stream_;
    const auto& r = st.rows;
    dev::decode_setup(st.d_lanes, row_lane, n, book, per_lane, st.d_step_position, st.clock, st.zero_row, r, s);
    if (book == 0)
    {
        const int trows = n * per_lane;
        auto* emb = ws.get<std::uint16_t>("emb", static_cast<std::size_t>(trows) * 1024);
        dev::embed_sum(model_->embeddings.as<std::uint16_t>(), st.tokens, r.temporal_offsets, r.temporal_counts,
                       trows, emb, s);
        auto* eq = ws.get<std::int8_t>("eq", static_cast<std::size_t>(trows) * 1024);
        auto* es = ws.get<float>("es", static_cast<std::size_t>(trows) * 4);
        auto* th = ws.get<std::uint16_t>("th", static_cast<std::size_t>(trows) * 512);
        run_linear_bf16(60, emb, trows, th, nullptr, false, eq, es);
        auto* tout = ws.get<std::uint16_t>("tout", static_cast<std::size_t>(trows) * 512);
        run_stack(ws, true, trows, th, r.temporal_meta, context, st.tck, st.tcv, st.tstride, tout, nullptr,
                  nullptr, per_lane > 1);
        // Conditioning: each active lane's last temporal row.
        dev::scatter_rows(tout, r.cond_source, r.cond_lane, n, st.cond, s);
    }
    auto* ch = ws.get<std::uint16_t>("ch", static_cast<std::size_t>(n) * 512);
    if (book == 0)
    {
        dev::add_positions(st.cond, r.codebook_lane, r.codebook_book, model_->positions.as<std::uint16_t>(), n, ch,
                           s);
    }
    else
    {
        // Prefix embedding sum (BF8L-quantized in the same kernel), cb_proj,
        // and the book's position row added as a residual broadcast to every
        // row: all rows of a step share `book`, and bf16(pos + y) is
        // add_positions' bf16(y + pos).
        auto* pemb = ws.get<std::uint16_t>("pemb", static_cast<std::size_t>(n) * 1024);
        auto* pq = ws.get<std::int8_t>("pq", static_cast<std::size_t>(n) * 1024);
        auto* ps = ws.get<float>("ps", static_cast<std::size_t>(n) * 4);
        dev::embed_sum(model_->embeddings.as<std::uint16_t>(), st.tokens, r.codebook_offsets, r.codebook_counts, n,
                       pemb, s, pq, ps, error_word());
        run_linear(61, pq, ps, n, ch, model_->positions.as<std::uint16_t>() + book * 512, false, 0);
    }
    auto* fq = ws.get<std::int8_t>("fq", static_cast<std::size_t>(n) * 512);
    auto* fs = ws.get<float>("fs", static_cast<std::size_t>(n) * 2);
    run_stack(ws, false, n, ch, r.codebook_meta, 12, st.cck, st.ccv, st.cstride, nullptr, fq, fs);
    auto* logits = ws.get<std::uint16_t>("logits", static_cast<std::size_t>(n) * 1024);
    run_linear(62, fq, fs, n, logits, nullptr, false);
    auto* tree = ws.get<float>("tree", static_cast<std::size_t>(n) * 1023);
    {
        KernelTimer::Scope timing("softmax_tree", s, 0.0);
        dev::softmax_tree(logits, n, nullptr, nullptr, tree, error_word(), s);
    }
    KernelTimer::Scope timing("range_decode", s, 0.0);
    dev::range_decode_rows(st.payload, st.offsets, st.sizes, st.cursors, static_cast<int>(st.headers.size()),
                           row_begin, tree, r.destination, st.tokens, error_word(), s);
}
} // namespace tsacb
