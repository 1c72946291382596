// bnn-infer-b200: the command line of the device-resident engine.
//
//   bnn-infer-b200 llm MODEL.gguf [--prompt TEXT | --ids FILE]
//                                 [--steps N] [--ctx N] [--chat] [--stats]
//   bnn-infer-b200 classify MODEL.gguf --input FILE [--labels FILE]
//                                      [--batch N] [--verbose] [--stats]
//
// The same commands, arguments, defaults, files and standard output as the
// reference CLI (bnn-infer-v2.c: `llm` :163-293, `classify` :376-522), so
// scripts can switch binaries: llm streams the generated text (stopping
// before an end-of-generation token, after --steps tokens or at a full
// context) then a newline; classify prints the per-sample lines (--verbose),
// the accuracy or sample count, and the class histogram. The work runs on
// BNND_*: the text loop is BNND_GenerateStream, which keeps device steps
// queued ahead of the pieces being printed. --stats (not in the reference)
// reports timings on standard error.
#include <chrono>
#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "bnn_b200_engine.h"

namespace {

constexpr uint32_t kDefaultSteps = 40;
constexpr uint32_t kDefaultCtx = 1024;
const char* const kDefaultPrompt = "\xe6\x98\xa5\xe5\xa4\xa9";  // the reference CLI's default prompt

void usage(const char* program) {
    const int w = (int)std::strlen(program);
    std::fprintf(stderr,
                 "usage: %s llm MODEL.gguf [--prompt TEXT | --ids FILE]\n"
                 "       %*s [--steps N] [--ctx N] [--chat] [--stats]\n"
                 "       %s classify MODEL.gguf --input FILE [--labels FILE]\n"
                 "       %*s [--batch N] [--verbose] [--stats]\n",
                 program, w, "", program, w, "");
}

const char* status_name(BNND_Status st) {
    switch (st) {
    case BNND_OK: return "ok";
    case BNND_EINVAL: return "invalid argument";
    case BNND_ENOMEM: return "out of memory";
    case BNND_ENOTSUP: return "not supported";
    case BNND_ERANGE: return "out of range";
    case BNND_EIO: return "device error";
    case BNND_EFORMAT: return "bad model file";
    case BNND_ECOMPUTE: return "computation failed";
    default: return "unknown status";
    }
}

bool report(BNND_Status st, const char* what) {
    const char* detail = BNND_LastError();
    std::fprintf(stderr, "error: %s: %s%s%s\n", what, status_name(st), detail && *detail ? ": " : "",
                 detail ? detail : "");
    return false;
}

// Decimal digits only, no sign or spaces, within uint32_t.
bool parse_u32(const char* text, uint32_t* out) {
    if (!text || !*text)
        return false;
    uint64_t v = 0;
    for (const char* p = text; *p; ++p) {
        if (*p < '0' || *p > '9')
            return false;
        v = v * 10 + (uint64_t)(*p - '0');
        if (v > UINT32_MAX)
            return false;
    }
    *out = (uint32_t)v;
    return true;
}

bool read_file(const char* path, std::vector<unsigned char>* out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) {
        std::fprintf(stderr, "error: %s: cannot open file\n", path);
        return false;
    }
    std::vector<unsigned char> data;
    unsigned char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0)
        data.insert(data.end(), buf, buf + n);
    const bool err = std::ferror(f) != 0;
    std::fclose(f);
    if (err || data.empty()) {
        std::fprintf(stderr, "error: %s: %s\n", path, err ? "read failed" : "invalid file size");
        return false;
    }
    *out = std::move(data);
    return true;
}

// Whitespace-separated decimal ids, each below `vocab`, at most `capacity`,
// nothing else in the file, at least one.
bool load_ids(const char* path, uint32_t capacity, uint32_t vocab, std::vector<int32_t>* ids) {
    FILE* f = std::fopen(path, "r");
    if (!f) {
        std::fprintf(stderr, "error: %s: cannot open token file\n", path);
        return false;
    }
    long v = 0;
    while (std::fscanf(f, "%ld", &v) == 1) {
        if (v < 0 || v >= (long)vocab || ids->size() == capacity) {
            std::fprintf(stderr, "error: %s: invalid or too many token IDs\n", path);
            std::fclose(f);
            return false;
        }
        ids->push_back((int32_t)v);
    }
    bool trailing = false;
    for (int ch; (ch = std::fgetc(f)) != EOF;)
        if (ch != ' ' && ch != '\t' && ch != '\n' && ch != '\r' && ch != '\v' && ch != '\f') {
            trailing = true;
            break;
        }
    const bool bad = std::ferror(f) || trailing || ids->empty();
    std::fclose(f);
    if (bad)
        std::fprintf(stderr, "error: %s: invalid token file\n", path);
    return !bad;
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

struct Handles {
    BNN_Device dev = nullptr;
    BNND_Model model = nullptr;
    BNND_Context ctx = nullptr;
    ~Handles() {
        if (ctx)
            BNND_ContextFree(ctx);
        if (model)
            BNND_ModelFree(model);
        if (dev && BNN_DeviceClose(dev) != BNN_OK)
            std::fprintf(stderr, "warning: device is still busy\n");
    }
};

bool open_model(Handles& h, const char* path, BNND_ModelInfo* info) {
    const BNN_Status ds = BNN_DeviceOpen(0, &h.dev);
    if (ds != BNN_OK) {
        std::fprintf(stderr, "error: BNN_DeviceOpen: %s\n", BNN_StatusString(ds));
        return false;
    }
    BNND_Status st = BNND_ModelLoad(h.dev, path, &h.model);
    if (st != BNND_OK)
        return report(st, "BNND_ModelLoad");
    st = BNND_ModelGetInfo(h.model, info);
    return st == BNND_OK || report(st, "BNND_ModelGetInfo");
}

int piece_out(void*, int32_t, const char* bytes, size_t len) {
    std::fwrite(bytes, 1, len, stdout);
    std::fflush(stdout);
    return 0;
}

int llm(const char* program, int argc, char** argv) {
    const char *model = nullptr, *prompt = nullptr, *ids_path = nullptr;
    uint32_t steps = kDefaultSteps, ctx_len = kDefaultCtx;
    bool chat = false, stats = false, steps_set = false, ctx_set = false;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--chat" || arg == "--stats") {
            bool& flag = arg == "--chat" ? chat : stats;
            if (flag)
                return usage(program), 1;
            flag = true;
        } else if (arg == "--prompt" || arg == "--ids" || arg == "--steps" || arg == "--ctx") {
            if (++i == argc)
                return usage(program), 1;
            if (arg == "--prompt") {
                if (prompt)
                    return usage(program), 1;
                prompt = argv[i];
            } else if (arg == "--ids") {
                if (ids_path)
                    return usage(program), 1;
                ids_path = argv[i];
            } else if (arg == "--steps") {
                if (steps_set || !parse_u32(argv[i], &steps))
                    return usage(program), 1;
                steps_set = true;
            } else {
                if (ctx_set || !parse_u32(argv[i], &ctx_len) || ctx_len == 0)
                    return usage(program), 1;
                ctx_set = true;
            }
        } else if (arg[0] == '-' || model) {
            return usage(program), 1;
        } else {
            model = argv[i];
        }
    }
    if (!model || (prompt && ids_path))
        return usage(program), 1;

    Handles h;
    BNND_ModelInfo info;
    if (!open_model(h, model, &info))
        return 1;
    if (info.task != BNND_TASK_LLM) {
        std::fprintf(stderr, "error: '%s' is not a language model\n", model);
        return 1;
    }
    BNND_ContextParams params;
    BNND_ContextParamsInit(&params);
    params.n_ctx = ctx_len;
    BNND_Status st = BNND_ContextCreate(h.model, &params, &h.ctx);
    if (st != BNND_OK)
        return report(st, "BNND_ContextCreate"), 1;

    std::vector<int32_t> ids;
    if (ids_path) {
        if (!load_ids(ids_path, ctx_len, info.n_vocab, &ids))
            return 1;
    } else {
        std::string text = prompt ? prompt : kDefaultPrompt;
        if (chat)
            text = "<|im_start|>user\n" + text + "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n";
        ids.resize(ctx_len);
        uint32_t n = 0;
        st = BNND_Tokenize(h.model, text.c_str(), 1, ids.data(), ctx_len, &n);
        if (st != BNND_OK)
            return report(st, "BNND_Tokenize"), 1;
        if (n == 0) {
            std::fprintf(stderr, "error: prompt encoded to zero tokens\n");
            return 1;
        }
        ids.resize(n);
    }
    const uint32_t count = (uint32_t)ids.size();
    if (count >= ctx_len && steps > 0) {
        std::fprintf(stderr, "error: prompt leaves no room for generation\n");
        return 1;
    }
    const double t0 = now_s();
    int32_t next = 0;
    st = BNND_DecodeArgmax(h.ctx, ids.data(), count, &next);
    if (st != BNND_OK)
        return report(st, "BNND_DecodeArgmax(prefill)"), 1;
    const double t1 = now_s();
    uint32_t emitted = 0;
    if (steps > 0) {
        st = BNND_GenerateStream(h.ctx, steps, piece_out, nullptr, nullptr, &emitted);
        if (st != BNND_OK)
            return report(st, "BNND_GenerateStream"), 1;
    }
    const double t2 = now_s();
    std::putchar('\n');
    if (stats)
        std::fprintf(stderr, "prompt %u tokens in %.3f ms (%.1f tok/s); generated %u tokens in %.3f ms (%.1f tok/s)\n",
                     count, (t1 - t0) * 1e3, count / (t1 - t0), emitted, (t2 - t1) * 1e3,
                     emitted ? emitted / (t2 - t1) : 0.0);
    return 0;
}

int classify(const char* program, int argc, char** argv) {
    const char *model = nullptr, *input = nullptr, *labels_path = nullptr;
    uint32_t batch = 64;
    bool verbose = false, stats = false, batch_set = false;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--verbose" || arg == "--stats") {
            bool& flag = arg == "--verbose" ? verbose : stats;
            if (flag)
                return usage(program), 1;
            flag = true;
        } else if (arg == "--input" || arg == "--labels" || arg == "--batch") {
            if (++i == argc)
                return usage(program), 1;
            if (arg == "--input") {
                if (input)
                    return usage(program), 1;
                input = argv[i];
            } else if (arg == "--labels") {
                if (labels_path)
                    return usage(program), 1;
                labels_path = argv[i];
            } else {
                if (batch_set || !parse_u32(argv[i], &batch) || batch == 0)
                    return usage(program), 1;
                batch_set = true;
            }
        } else if (arg[0] == '-' || model) {
            return usage(program), 1;
        } else {
            model = argv[i];
        }
    }
    if (!model || !input)
        return usage(program), 1;

    Handles h;
    BNND_ModelInfo info;
    if (!open_model(h, model, &info))
        return 1;
    if (info.task != BNND_TASK_CLASSIFY) {
        std::fprintf(stderr, "error: '%s' is not a classification model\n", model);
        return 1;
    }
    if (!info.input_size || !info.n_classes) {
        std::fprintf(stderr, "error: model has an invalid input/class shape\n");
        return 1;
    }
    std::vector<unsigned char> data, labels;
    if (!read_file(input, &data))
        return 1;
    const uint64_t sample_bytes = (uint64_t)info.input_size * sizeof(float);
    if (data.size() % sample_bytes != 0) {
        std::fprintf(stderr, "error: input file size is not a multiple of %" PRIu64 " bytes\n", sample_bytes);
        return 1;
    }
    const uint64_t n64 = data.size() / sample_bytes;
    if (n64 == 0 || n64 > UINT32_MAX) {
        std::fprintf(stderr, "error: invalid sample count\n");
        return 1;
    }
    const uint32_t n = (uint32_t)n64;
    if (labels_path) {
        if (!read_file(labels_path, &labels))
            return 1;
        if (labels.size() != n) {
            std::fprintf(stderr, "error: labels file must contain %" PRIu32 " bytes\n", n);
            return 1;
        }
        for (unsigned char l : labels)
            if (l >= info.n_classes) {
                std::fprintf(stderr, "error: label %u outside class range\n", (unsigned)l);
                return 1;
            }
    }
    BNND_ContextParams params;
    BNND_ContextParamsInit(&params);
    params.n_batch = batch < n ? batch : n;
    BNND_Status st = BNND_ContextCreate(h.model, &params, &h.ctx);
    if (st != BNND_OK)
        return report(st, "BNND_ContextCreate"), 1;
    const uint32_t rows = params.n_batch;
    std::vector<float> logits((size_t)rows * info.n_classes);
    std::vector<uint64_t> counts(info.n_classes, 0);
    const float* x = reinterpret_cast<const float*>(data.data());
    uint64_t correct = 0;
    const double t0 = now_s();
    for (uint32_t off = 0; off < n; off += rows) {
        const uint32_t cnt = n - off < rows ? n - off : rows;
        st = BNND_Classify(h.ctx, x + (size_t)off * info.input_size, cnt, logits.data());
        if (st != BNND_OK)
            return report(st, "BNND_Classify"), 1;
        for (uint32_t i = 0; i < cnt; ++i) {
            const float* row = logits.data() + (size_t)i * info.n_classes;
            uint32_t best = 0;  // first maximum
            for (uint32_t c = 1; c < info.n_classes; ++c)
                if (row[c] > row[best])
                    best = c;
            counts[best]++;
            if (!labels.empty() && best == labels[off + i])
                correct++;
            if (verbose) {
                if (!labels.empty())
                    std::printf("sample %" PRIu32 ": class %" PRIu32 " label %u\n", off + i, best,
                                (unsigned)labels[off + i]);
                else
                    std::printf("sample %" PRIu32 ": class %" PRIu32 "\n", off + i, best);
            }
        }
    }
    const double t1 = now_s();
    if (!labels.empty())
        std::printf("accuracy: %" PRIu64 "/%" PRIu32 " (%.4f)\n", correct, n, (double)correct / (double)n);
    else
        std::printf("samples: %" PRIu32 "\n", n);
    std::printf("class counts:");
    for (uint64_t c : counts)
        std::printf(" %" PRIu64, c);
    std::putchar('\n');
    if (stats)
        std::fprintf(stderr, "%u samples in %.3f ms (%.1f samples/s)\n", n, (t1 - t0) * 1e3, n / (t1 - t0));
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2)
        return usage(argv[0]), 1;
    if (std::strcmp(argv[1], "llm") == 0)
        return llm(argv[0], argc - 1, argv + 1);
    if (std::strcmp(argv[1], "classify") == 0)
        return classify(argv[0], argc - 1, argv + 1);
    usage(argv[0]);
    return 1;
}
