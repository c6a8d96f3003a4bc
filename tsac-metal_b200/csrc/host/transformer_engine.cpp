#include "transformer_engine.hpp"

#include "kernel_timer.hpp"

#include "kernels/codebook_step.cuh"
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
    return rows <= 256 ? n * k + 4 * n * k / 256 + 4 * n + m * k + 4 * m * k / 256 + 2 * m * n
                       : 2.0 * m * n * k;
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
    KernelTimer::Scope timing(rows <= 256 ? "qlinear_small" : "qlinear_gemm", stream_,
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
                                  std::int8_t* final_q, float* final_s)
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
                                       error_word());
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
    run_stack(ws_, true, trows, th, d_tmeta, max_time, tck, tcv, tstride, cond, nullptr, nullptr);

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
// Page-locked host staging (graph memcpy nodes need fixed host addresses).
class PinnedBuffer
{
public:
    explicit PinnedBuffer(std::size_t bytes) : bytes_(bytes)
    {
        cuda_ok(cudaHostAlloc(&ptr_, bytes ? bytes : 1, cudaHostAllocDefault), "cudaHostAlloc");
    }
    ~PinnedBuffer()
    {
        if (ptr_)
            cudaFreeHost(ptr_);
    }
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
    template <class T> T* as() const
    {
        return static_cast<T*>(ptr_);
    }
    std::size_t bytes() const
    {
        return bytes_;
    }

private:
    void* ptr_ = nullptr;
    std::size_t bytes_;
};

// Packed per-step inputs: struct-of-arrays for up to `rows` rows and 12 books.
struct StepBlock
{
    std::size_t meta, lane_rows, books, offsets, counts, tokens, bytes;
    explicit StepBlock(std::size_t rows)
    {
        std::size_t at = 0;
        const auto take = [&](std::size_t n)
        {
            const auto here = at;
            at = align_up(at + n, 256);
            return here;
        };
        meta = take(rows * sizeof(RowMeta));
        lane_rows = take(rows * 4);
        books = take(rows * 4);
        offsets = take(rows * 4);
        counts = take(rows * 4);
        tokens = take(rows * 12 * 2);
        bytes = at;
    }
};
} // namespace

struct TransformerEngine::DecodeState
{
    struct Lane
    {
        int recording = 0, lane_b = 0, group = 0;
        int start = 0, length = 0, used = 0;
        std::vector<std::uint16_t> current;
        std::deque<std::vector<std::uint16_t>> history;
        int tslot = 0; // first temporal cache slot (1024 per lane)
        int cslot = 0; // first codebook cache slot (books per lane)
    };
    std::vector<Header> headers;
    std::vector<Lane> lanes;
    int max_rows = 0, replay_rows = 0;
    std::size_t tstride = 0, cstride = 0;
    Workspace ws; // sized once per session: graph-captured pointers stay valid
    std::uint16_t *tck = nullptr, *tcv = nullptr, *cck = nullptr, *ccv = nullptr,
                  *cond = nullptr;
    // Temporal and codebook inputs, staged together with one copy.
    std::unique_ptr<StepBlock> temporal_block, codebook_block;
    std::unique_ptr<PinnedBuffer> host_in, host_masses, host_error;
    char* dev_in = nullptr;
    int* identity = nullptr;
    struct StepGraph
    {
        cudaGraphExec_t exec;
        unsigned long long kernels; // kernel nodes, for the launch tally
    };
    std::map<std::tuple<int, int, int>, StepGraph> graphs; // (temporal, book, rows)
    std::vector<LaneRef> last;
    std::vector<int> last_lanes;
    std::size_t last_book = 0;

    ~DecodeState()
    {
        for (auto& [key, graph] : graphs)
            cudaGraphExecDestroy(graph.exec);
    }
};

TransformerEngine::~TransformerEngine() = default;

void TransformerEngine::decode_begin(const std::vector<Header>& headers)
{
    decode_.reset();
    auto state = std::make_unique<DecodeState>();
    state->headers = headers;
    int tslots = 0, cslots = 0;
    bool replay = false;
    for (std::size_t r = 0; r < headers.size(); ++r)
    {
        const auto& h = headers[r];
        check_header(h);
        require(h.method == 1 && h.model_channels == model_->channels &&
                    h.codebooks <= model_->books,
                "Transformer stream/model mismatch");
        const int F = static_cast<int>(h.frames), B = h.batch, G = h.groups;
        const int lanes_b = std::min(B, F), base = F / B, extra = F % B;
        for (int lane = 0; lane < lanes_b; ++lane)
        {
            for (int g = 0; g < G; ++g)
            {
                DecodeState::Lane l;
                l.recording = static_cast<int>(r);
                l.lane_b = lane;
                l.group = g;
                l.length = base + (lane < extra);
                l.start = lane * base + std::min(lane, extra);
                l.current.assign(h.codebooks, 0);
                l.tslot = tslots;
                l.cslot = cslots;
                tslots += context;
                cslots += h.codebooks;
                replay = replay || l.length > context;
                state->lanes.push_back(std::move(l));
            }
        }
    }
    auto& st = *state;
    st.max_rows = static_cast<int>(st.lanes.size());
    st.replay_rows = st.max_rows * (replay ? replay_frames : 1);
    const auto cap = static_cast<std::size_t>(std::max(st.replay_rows, 1));
    st.tstride = static_cast<std::size_t>(tslots) * 512;
    st.cstride = static_cast<std::size_t>(cslots) * 512;
    st.tck = st.ws.get<std::uint16_t>("tck", st.tstride * 12);
    st.tcv = st.ws.get<std::uint16_t>("tcv", st.tstride * 12);
    st.cck = st.ws.get<std::uint16_t>("cck", st.cstride * 3);
    st.ccv = st.ws.get<std::uint16_t>("ccv", st.cstride * 3);
    st.cond = st.ws.get<std::uint16_t>("cond", cap * 512);
    // Every scratch name at its session maximum, so no pointer moves later.
    st.ws.get<std::int8_t>("xq", cap * 2048);
    st.ws.get<float>("xs", cap * 8);
    st.ws.get<std::uint16_t>("qkv", cap * 1536);
    st.ws.get<std::uint16_t>("query", cap * 512);
    st.ws.get<std::uint16_t>("att", cap * 512);
    st.ws.get<std::uint16_t>("mlp", cap * 2048);
    st.ws.get<float>("partials", dev::attention_partials_bytes(static_cast<int>(cap), context) / 4);
    for (const char* name : {"emb", "pemb"})
        st.ws.get<std::uint16_t>(name, cap * 1024);
    for (const char* name : {"eq", "pq"})
        st.ws.get<std::int8_t>(name, cap * 1024);
    for (const char* name : {"es", "ps"})
        st.ws.get<float>(name, cap * 4);
    for (const char* name : {"th", "tout", "ch"})
        st.ws.get<std::uint16_t>(name, cap * 512);
    st.ws.get<std::int8_t>("fq", cap * 512);
    st.ws.get<float>("fs", cap * 2);
    st.ws.get<std::uint16_t>("logits", cap * 1024);
    st.ws.get<float>("tree", cap * 1023);
    st.temporal_block = std::make_unique<StepBlock>(cap);
    st.codebook_block = std::make_unique<StepBlock>(cap);
    const auto in_bytes = st.temporal_block->bytes + st.codebook_block->bytes;
    st.dev_in = st.ws.get<char>("in", in_bytes);
    st.host_in = std::make_unique<PinnedBuffer>(in_bytes);
    st.host_masses = std::make_unique<PinnedBuffer>(cap * 1023 * 4);
    st.host_error = std::make_unique<PinnedBuffer>(4);
    std::vector<int> ident(cap);
    for (std::size_t i = 0; i < cap; ++i)
        ident[i] = static_cast<int>(i);
    st.identity = st.ws.get<int>("identity", cap);
    cuda_ok(cudaMemcpyAsync(st.identity, ident.data(), cap * 4, cudaMemcpyHostToDevice, stream_),
            "H2D");
    cuda_ok(cudaStreamSynchronize(stream_), "decode session");
    decode_ = std::move(state);
}

std::vector<TransformerEngine::LaneRef>
TransformerEngine::decode_predict(std::size_t step, std::size_t book, const float** masses)
{
    require(decode_ != nullptr, "decode session not started");
    auto& st = *decode_;
    auto s = stream_;
    std::vector<int> active;
    for (int i = 0; i < static_cast<int>(st.lanes.size()); ++i)
    {
        const auto& l = st.lanes[static_cast<std::size_t>(i)];
        if (static_cast<int>(step) < l.length && book < l.current.size())
            active.push_back(i);
    }
    st.last.clear();
    st.last_lanes = active;
    st.last_book = book;
    if (active.empty())
        return {};
    const int n = static_cast<int>(active.size());
    char* host = st.host_in->as<char>();
    const auto& tb = *st.temporal_block;
    const auto& cb = *st.codebook_block;
    char* host_c = host + tb.bytes;
    char* dev_t = st.dev_in;
    char* dev_c = st.dev_in + tb.bytes;

    // ---- temporal inputs (book 0): one row per lane, or a 256-row replay.
    int temporal_rows = 0;
    bool replay = false;
    if (book == 0)
    {
        auto* meta = reinterpret_cast<RowMeta*>(host + tb.meta);
        auto* lane_rows = reinterpret_cast<int*>(host + tb.lane_rows);
        auto* offsets = reinterpret_cast<int*>(host + tb.offsets);
        auto* counts = reinterpret_cast<int*>(host + tb.counts);
        auto* tokens = reinterpret_cast<std::uint16_t*>(host + tb.tokens);
        int tok = 0;
        for (std::size_t j = 0; j < active.size(); ++j)
        {
            const int i = active[j];
            auto& l = st.lanes[static_cast<std::size_t>(i)];
            const int Q = static_cast<int>(l.current.size());
            const auto add = [&](const std::vector<std::uint16_t>& fb, bool is_replay)
            {
                const int position = l.used++;
                meta[temporal_rows] = {l.tslot + position, l.tslot, position + 1, position,
                                       (position + 1 > 64 || is_replay) ? 1 : 0};
                offsets[temporal_rows] = tok;
                counts[temporal_rows] = Q;
                std::copy(fb.begin(), fb.end(), tokens + tok);
                tok += 12;
                ++temporal_rows;
            };
            std::fill(l.current.begin(), l.current.end(), 0);
            if (l.used == context)
            {
                require(static_cast<int>(l.history.size()) == replay_frames,
                        "incomplete Transformer replay history");
                l.used = 0;
                replay = true;
                for (const auto& fb : l.history)
                    add(fb, true);
            }
            else
            {
                add(l.history.empty() ? l.current : l.history.back(), false);
            }
            // The lane's conditioning is its last temporal row: entry j of the
            // scatter maps row (temporal_rows - 1) to lane i.
            lane_rows[j] = i;
            reinterpret_cast<int*>(host + tb.books)[j] = temporal_rows - 1;
        }
    }
    // ---- codebook inputs: one row per active lane.
    {
        auto* meta = reinterpret_cast<RowMeta*>(host_c + cb.meta);
        auto* lane_rows = reinterpret_cast<int*>(host_c + cb.lane_rows);
        auto* books = reinterpret_cast<int*>(host_c + cb.books);
        auto* offsets = reinterpret_cast<int*>(host_c + cb.offsets);
        auto* counts = reinterpret_cast<int*>(host_c + cb.counts);
        auto* tokens = reinterpret_cast<std::uint16_t*>(host_c + cb.tokens);
        for (int j = 0; j < n; ++j)
        {
            const auto& l = st.lanes[static_cast<std::size_t>(active[static_cast<std::size_t>(j)])];
            meta[j] = {l.cslot + static_cast<int>(book), l.cslot, static_cast<int>(book) + 1, -1, 0};
            lane_rows[j] = active[static_cast<std::size_t>(j)];
            books[j] = static_cast<int>(book);
            offsets[j] = j * 12;
            counts[j] = static_cast<int>(book);
            std::copy_n(l.current.begin(), book, tokens + j * 12);
            st.last.push_back({l.recording,
                               l.lane_b * st.headers[static_cast<std::size_t>(l.recording)].groups + l.group});
        }
    }

    // TSAC_CUDA_FUSED_CODEBOOK=1 runs each codebook step as one cluster
    // launch (codebook_step.cu).  Bit-identical, but measured slower on B200
    // (about 178 us against 150 us per step at 48 lanes: each cluster's
    // phases are serial dependent chains on a few SMs, while the separate
    // kernels spread every phase over 100+ CTAs), so it is off by default.
    static const bool fused_codebook_step = []
    {
        const char* e = std::getenv("TSAC_CUDA_FUSED_CODEBOOK");
        return e && e[0] == '1';
    }();
    const auto enqueue = [&](int trows)
    {
        cuda_ok(cudaMemcpyAsync(st.dev_in, host, tb.bytes + cb.bytes, cudaMemcpyHostToDevice, s), "H2D");
        auto& ws = st.ws;
        if (trows > 0)
        {
            const auto* d_meta = reinterpret_cast<const RowMeta*>(dev_t + tb.meta);
            auto* emb = ws.get<std::uint16_t>("emb", static_cast<std::size_t>(trows) * 1024);
            dev::embed_sum(model_->embeddings.as<std::uint16_t>(),
                           reinterpret_cast<const std::uint16_t*>(dev_t + tb.tokens),
                           reinterpret_cast<const int*>(dev_t + tb.offsets),
                           reinterpret_cast<const int*>(dev_t + tb.counts), trows, emb, s);
            auto* eq = ws.get<std::int8_t>("eq", static_cast<std::size_t>(trows) * 1024);
            auto* es = ws.get<float>("es", static_cast<std::size_t>(trows) * 4);
            auto* th = ws.get<std::uint16_t>("th", static_cast<std::size_t>(trows) * 512);
            run_linear_bf16(60, emb, trows, th, nullptr, false, eq, es);
            auto* tout = ws.get<std::uint16_t>("tout", static_cast<std::size_t>(trows) * 512);
            run_stack(ws, true, trows, th, d_meta, context, st.tck, st.tcv, st.tstride, tout,
                      nullptr, nullptr);
            // Conditioning: each active lane's last temporal row.
            dev::scatter_rows(tout, reinterpret_cast<const int*>(dev_t + tb.books),
                              reinterpret_cast<const int*>(dev_t + tb.lane_rows), n, st.cond, s);
        }
        const auto* d_meta = reinterpret_cast<const RowMeta*>(dev_c + cb.meta);
        const auto* d_books = reinterpret_cast<const int*>(dev_c + cb.books);
        auto* tree = ws.get<float>("tree", static_cast<std::size_t>(n) * 1023);
        if (fused_codebook_step)
        {
            // The whole codebook step in one cluster launch (codebook_step.cu).
            dev::CodebookStepArgs a{};
            a.rows = n;
            a.book = static_cast<int>(book);
            a.cond = st.cond;
            a.lane_rows = reinterpret_cast<const int*>(dev_c + cb.lane_rows);
            a.embeddings = model_->embeddings.as<std::uint16_t>();
            a.tokens = reinterpret_cast<const std::uint16_t*>(dev_c + cb.tokens);
            a.offsets = reinterpret_cast<const int*>(dev_c + cb.offsets);
            a.counts = reinterpret_cast<const int*>(dev_c + cb.counts);
            const auto linear = [&](int p)
            {
                const auto& l = model_->projections[static_cast<std::size_t>(p)];
                return dev::CodebookLinear{l.weights.as<std::int8_t>(), l.scales.as<float>(),
                                           l.bias.as<float>()};
            };
            a.proj61 = linear(61);
            a.positions = model_->positions.as<std::uint16_t>();
            a.books = d_books;
            for (int l = 0; l < 3; ++l)
            {
                for (int op = 0; op < 4; ++op)
                    a.layer[l][op] = linear(projection_index(false, l, op));
                for (int second = 0; second < 2; ++second)
                {
                    const int nrm = norm_index(false, l, second != 0);
                    a.norm_gain[2 * l + second] = model_->norm_gain[static_cast<std::size_t>(nrm)].as<std::uint16_t>();
                    a.norm_bias[2 * l + second] = model_->norm_bias[static_cast<std::size_t>(nrm)].as<std::uint16_t>();
                }
            }
            a.norm_gain[6] = model_->norm_gain[static_cast<std::size_t>(final_norm(false))].as<std::uint16_t>();
            a.norm_bias[6] = model_->norm_bias[static_cast<std::size_t>(final_norm(false))].as<std::uint16_t>();
            a.proj62 = linear(62);
            a.gelu = model_->gelu.as<std::uint16_t>();
            a.meta = d_meta;
            a.cache_k = st.cck;
            a.cache_v = st.ccv;
            a.cache_stride = st.cstride;
            a.tree = tree;
            a.error_word = error_word();
            KernelTimer::Scope timing("codebook_step", s, 0.0);
            dev::codebook_step(a, s);
        }
        else
        {
            auto* ch = ws.get<std::uint16_t>("ch", static_cast<std::size_t>(n) * 512);
            if (book == 0)
            {
                dev::add_positions(st.cond, reinterpret_cast<const int*>(dev_c + cb.lane_rows), d_books,
                                   model_->positions.as<std::uint16_t>(), n, ch, s);
            }
            else
            {
                // Prefix embedding sum (BF8L-quantized in the same kernel),
                // cb_proj, and the book's position row added as a residual
                // broadcast to every row: all rows of a step share `book`, and
                // bf16(pos + y) is add_positions' bf16(y + pos).
                auto* pemb = ws.get<std::uint16_t>("pemb", static_cast<std::size_t>(n) * 1024);
                auto* pq = ws.get<std::int8_t>("pq", static_cast<std::size_t>(n) * 1024);
                auto* ps = ws.get<float>("ps", static_cast<std::size_t>(n) * 4);
                dev::embed_sum(model_->embeddings.as<std::uint16_t>(),
                               reinterpret_cast<const std::uint16_t*>(dev_c + cb.tokens),
                               reinterpret_cast<const int*>(dev_c + cb.offsets),
                               reinterpret_cast<const int*>(dev_c + cb.counts), n, pemb, s, pq, ps,
                               error_word());
                run_linear(61, pq, ps, n, ch, model_->positions.as<std::uint16_t>() + book * 512, false, 0);
            }
            auto* fq = ws.get<std::int8_t>("fq", static_cast<std::size_t>(n) * 512);
            auto* fs = ws.get<float>("fs", static_cast<std::size_t>(n) * 2);
            run_stack(ws, false, n, ch, d_meta, 12, st.cck, st.ccv, st.cstride, nullptr, fq, fs);
            auto* logits = ws.get<std::uint16_t>("logits", static_cast<std::size_t>(n) * 1024);
            run_linear(62, fq, fs, n, logits, nullptr, false);
            KernelTimer::Scope timing("softmax_tree", s, 0.0);
            dev::softmax_tree(logits, n, nullptr, nullptr, tree, error_word(), s);
        }
        cuda_ok(cudaMemcpyAsync(st.host_masses->as<void>(), tree, static_cast<std::size_t>(n) * 1023 * 4,
                                cudaMemcpyDeviceToHost, s),
                "D2H");
        cuda_ok(cudaMemcpyAsync(st.host_error->as<void>(), error_word(), 4, cudaMemcpyDeviceToHost, s),
                "D2H");
    };

    // Algorithmic bytes of one step: the int8 weights it streams.
    const auto weights = [&](int p)
    {
        const auto& l = model_->projections[static_cast<std::size_t>(p)];
        return static_cast<double>(l.input) * l.output;
    };
    double weight_bytes = weights(61) + weights(62);
    for (int p = 48; p < 60; ++p)
        weight_bytes += weights(p);
    if (book == 0)
    {
        weight_bytes += weights(60);
        for (int p = 0; p < 48; ++p)
            weight_bytes += weights(p);
    }
    // TSAC_CUDA_DECODE_GRAPHS=0 runs every step's kernels directly (each
    // kernel family then shows in the kernel timing); replay steps (once per
    // 768 frames of a lane) always run directly.
    static const bool graphs_enabled = []
    {
        const char* e = std::getenv("TSAC_CUDA_DECODE_GRAPHS");
        return !(e && e[0] == '0');
    }();
    if (replay || !graphs_enabled)
    {
        enqueue(temporal_rows);
    }
    else
    {
        const auto key = std::make_tuple(book == 0 ? 1 : 0, static_cast<int>(book), n);
        auto found = st.graphs.find(key);
        if (found == st.graphs.end())
        {
            cudaGraph_t graph = nullptr;
            unsigned long long kernels = 0;
            {
                dev::CaptureTally tally;
                cuda_ok(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "capture");
                enqueue(temporal_rows);
                cuda_ok(cudaStreamEndCapture(s, &graph), "capture");
                kernels = tally.kernels();
            }
            cudaGraphExec_t exec = nullptr;
            const auto status = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            cuda_ok(status, "cudaGraphInstantiate");
            found = st.graphs.emplace(key, DecodeState::StepGraph{exec, kernels}).first;
        }
        KernelTimer::Scope timing("decode_step", s, weight_bytes);
        cuda_ok(cudaGraphLaunch(found->second.exec, s), "cudaGraphLaunch");
        dev::note_launch(found->second.kernels);
    }
    cuda_ok(cudaStreamSynchronize(s), "decode step");
    if (*st.host_error->as<unsigned>())
    {
        cuda_ok(cudaMemset(error_word(), 0, 4), "memset");
        throw NumericError("Transformer activations must be finite");
    }
    *masses = st.host_masses->as<float>();
    return st.last;
}

void TransformerEngine::decode_commit(std::span<const std::uint16_t> tokens)
{
    require(decode_ != nullptr, "decode session not started");
    auto& st = *decode_;
    require(tokens.size() == st.last_lanes.size(), "decode commit does not match prediction");
    for (std::size_t j = 0; j < tokens.size(); ++j)
    {
        require(tokens[j] < 1024, "Transformer feedback token exceeds alphabet");
        auto& l = st.lanes[static_cast<std::size_t>(st.last_lanes[j])];
        l.current[st.last_book] = tokens[j];
        if (st.last_book + 1 == l.current.size())
        {
            l.history.push_back(l.current);
            if (static_cast<int>(l.history.size()) > replay_frames)
                l.history.pop_front();
        }
    }
}
} // namespace tsacb
