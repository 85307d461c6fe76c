// llama_generate -- the generation program of llama_generate.f90 on libq35: prompt ->
// token ids -> prefill + KV-cached decode on the GPU -> sampled tokens -> text.
//
// Behaviour kept from the reference program:
//  * the prompt is read from stdin when not given (:39-44; empty -> the default prompt);
//  * token ids come from an external tokenizer command run as
//    `<cmd> encode prompt.txt tokens.bin` (:162-214) and go back through
//    `<cmd> decode output_tokens.bin output.txt` (:219-253); tokens.bin /
//    output_tokens.bin hold an int32 count then the int32 ids (Fortran stream files).
//    Without a tokenizer, or when it fails, the prompt becomes the placeholder ids 1..10
//    (:181-186) and the text output is the ids;
//  * MAX_NEW_TOKENS 100, TEMPERATURE 0.8 > 0 -> sample_top_p with TOP_P 0.95 (the
//    reference's top-p does not scale by the temperature), else greedy (:93-98); EOS id 2
//    stops (:101-105); at most MAX_SEQ_LEN 2048 positions (:108-113);
//  * the statistics block (:125-140): prompt / generated / total tokens, time,
//    tokens per second, ms per token (wall clock around the loop, prefill included).
// Added for the serving API (api/inference_api.py:464-477 runs
// `llama_generate --prompt P --max-tokens N --temperature T --json` and reads
// {"text", "tokens"} from stdout): those flags and a one-line JSON result.
// Weights: a 3.5-bit safetensors checkpoint (--weights, repeatable for shards), the
// INT4 stream-binary layer files DIR/weights_layer{l}.bin (--layer-dir, over random
// embeddings), or random weights (the reference's fallback when no weight file exists).
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <string>
#include <sys/stat.h>
#include <sys/wait.h>
#include <unistd.h>
#include <vector>

#include "q35.h"

namespace {

struct Options {
    std::string prompt;
    bool have_prompt = false;
    int max_tokens = 100;            // MAX_NEW_TOKENS
    float temperature = 0.8f;        // TEMPERATURE
    float top_p = 0.95f;             // TOP_P
    int top_k = 40;                  // TOP_K (declared at :16, used by --sampler top_k)
    std::string sampler = "auto";    // auto: top_p when temperature > 0, else greedy
    bool json = false;
    bool stop_at_eos = true;
    std::string model = "70b";
    int n_layers = -1, hidden = -1, heads = -1, kv_heads = -1, head_dim = -1, ffn = -1, vocab = -1, max_seq = -1;
    int format = -1;                 // Q35_FMT_*; default from the weights
    int rope_mode = 0;
    std::vector<std::string> weights;
    std::string layer_dir;
    uint64_t init_seed = 0;
    uint64_t seed = 0;
    std::string tokenizer;
    std::string tokens_in, tokens_out;
    int device = 0;
};

void usage(FILE *f) {
    std::fprintf(f,
                 "usage: llama_generate [options]\n"
                 "  --prompt TEXT          prompt (default: read one line from stdin)\n"
                 "  --max-tokens N         new tokens (default 100)\n"
                 "  --temperature T        > 0: nucleus sampling, <= 0: greedy (default 0.8)\n"
                 "  --top-p P              nucleus mass (default 0.95)\n"
                 "  --top-k K              top-k size for --sampler top_k (default 40)\n"
                 "  --sampler S            auto | greedy | temperature | top_k | top_p (default auto)\n"
                 "  --seed S               seed of the sampling draws (default 0)\n"
                 "  --json                 print one JSON object {text, tokens, ...} on stdout\n"
                 "  --no-eos               do not stop at the end-of-sequence token 2\n"
                 "  --model NAME           70b | 13b | tiny (shape presets; default 70b)\n"
                 "  --layers/--hidden/--heads/--kv-heads/--head-dim/--ffn/--vocab/--max-seq N\n"
                 "                         override the preset's shape\n"
                 "  --format 3p5|int4      weight format (default: 3p5, int4 with --layer-dir)\n"
                 "  --rope-mode 0|1        0: the reference's position-in-call angles, 1: absolute\n"
                 "  --weights FILE         3.5-bit safetensors checkpoint (repeat for shards)\n"
                 "  --layer-dir DIR        INT4 stream-binary files DIR/weights_layer{l}.bin\n"
                 "  --init-seed S          seed of random weights (used without --weights)\n"
                 "  --tokenizer CMD        tokenizer command: CMD encode IN OUT / CMD decode IN OUT\n"
                 "  --tokens-in FILE       prompt ids (int32 count + int32 ids), skips the tokenizer\n"
                 "  --tokens-out FILE      write prompt + generated ids in the same format\n"
                 "  --device D             CUDA device (default 0)\n"
                 "environment: LLAMA_GENERATE_MODEL, LLAMA_GENERATE_WEIGHTS (':'-separated),\n"
                 "  LLAMA_GENERATE_LAYER_DIR, LLAMA_GENERATE_TOKENIZER give the defaults of\n"
                 "  --model, --weights, --layer-dir and --tokenizer\n");
}

// defaults from the environment, so a caller that passes only the serving flags (the API)
// still picks the model: LLAMA_GENERATE_MODEL, LLAMA_GENERATE_WEIGHTS (':'-separated
// shards), LLAMA_GENERATE_LAYER_DIR, LLAMA_GENERATE_TOKENIZER
void env_defaults(Options &o) {
    if (const char *v = std::getenv("LLAMA_GENERATE_MODEL")) o.model = v;
    if (const char *v = std::getenv("LLAMA_GENERATE_WEIGHTS")) {
        std::string s = v;
        size_t a = 0;
        while (a <= s.size()) {
            const size_t b = s.find(':', a);
            const std::string part = s.substr(a, b == std::string::npos ? std::string::npos : b - a);
            if (!part.empty()) o.weights.push_back(part);
            if (b == std::string::npos) break;
            a = b + 1;
        }
    }
    if (const char *v = std::getenv("LLAMA_GENERATE_LAYER_DIR")) o.layer_dir = v;
    if (const char *v = std::getenv("LLAMA_GENERATE_TOKENIZER")) o.tokenizer = v;
}

bool parse(int argc, char **argv, Options &o) {
    bool weights_flag = false;
    auto need = [&](int &i) -> const char * {
        if (i + 1 >= argc) {
            std::fprintf(stderr, "llama_generate: %s needs a value\n", argv[i]);
            return nullptr;
        }
        return argv[++i];
    };
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        const char *v = nullptr;
        if (a == "-h" || a == "--help") { usage(stdout); std::exit(0); }
        else if (a == "--json") o.json = true;
        else if (a == "--no-eos") o.stop_at_eos = false;
        else if (a == "--prompt") { if (!(v = need(i))) return false; o.prompt = v; o.have_prompt = true; }
        else if (a == "--max-tokens") { if (!(v = need(i))) return false; o.max_tokens = std::atoi(v); }
        else if (a == "--temperature") { if (!(v = need(i))) return false; o.temperature = (float)std::atof(v); }
        else if (a == "--top-p") { if (!(v = need(i))) return false; o.top_p = (float)std::atof(v); }
        else if (a == "--top-k") { if (!(v = need(i))) return false; o.top_k = std::atoi(v); }
        else if (a == "--sampler") { if (!(v = need(i))) return false; o.sampler = v; }
        else if (a == "--seed") { if (!(v = need(i))) return false; o.seed = std::strtoull(v, nullptr, 10); }
        else if (a == "--model") { if (!(v = need(i))) return false; o.model = v; }
        else if (a == "--layers") { if (!(v = need(i))) return false; o.n_layers = std::atoi(v); }
        else if (a == "--hidden") { if (!(v = need(i))) return false; o.hidden = std::atoi(v); }
        else if (a == "--heads") { if (!(v = need(i))) return false; o.heads = std::atoi(v); }
        else if (a == "--kv-heads") { if (!(v = need(i))) return false; o.kv_heads = std::atoi(v); }
        else if (a == "--head-dim") { if (!(v = need(i))) return false; o.head_dim = std::atoi(v); }
        else if (a == "--ffn") { if (!(v = need(i))) return false; o.ffn = std::atoi(v); }
        else if (a == "--vocab") { if (!(v = need(i))) return false; o.vocab = std::atoi(v); }
        else if (a == "--max-seq") { if (!(v = need(i))) return false; o.max_seq = std::atoi(v); }
        else if (a == "--rope-mode") { if (!(v = need(i))) return false; o.rope_mode = std::atoi(v); }
        else if (a == "--format") {
            if (!(v = need(i))) return false;
            const std::string f = v;
            if (f == "3p5" || f == "3.5") o.format = Q35_FMT_3P5BIT;
            else if (f == "int4") o.format = Q35_FMT_INT4;
            else { std::fprintf(stderr, "llama_generate: unknown format %s\n", v); return false; }
        }
        else if (a == "--weights") {
            if (!(v = need(i))) return false;
            if (!weights_flag) o.weights.clear();        // flags replace the environment's list
            weights_flag = true;
            o.weights.push_back(v);
        }
        else if (a == "--layer-dir") { if (!(v = need(i))) return false; o.layer_dir = v; }
        else if (a == "--init-seed") { if (!(v = need(i))) return false; o.init_seed = std::strtoull(v, nullptr, 10); }
        else if (a == "--tokenizer") { if (!(v = need(i))) return false; o.tokenizer = v; }
        else if (a == "--tokens-in") { if (!(v = need(i))) return false; o.tokens_in = v; }
        else if (a == "--tokens-out") { if (!(v = need(i))) return false; o.tokens_out = v; }
        else if (a == "--device") { if (!(v = need(i))) return false; o.device = std::atoi(v); }
        else { std::fprintf(stderr, "llama_generate: unknown option %s\n", a.c_str()); usage(stderr); return false; }
    }
    return true;
}

bool read_ids(const std::string &path, std::vector<int32_t> &ids) {
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    int32_t n = 0;
    bool ok = std::fread(&n, 4, 1, f) == 1 && n > 0 && n <= 10000;   // :199
    if (ok) {
        ids.resize((size_t)n);
        ok = std::fread(ids.data(), 4, (size_t)n, f) == (size_t)n;
    }
    std::fclose(f);
    return ok;
}

bool write_ids(const std::string &path, const std::vector<int32_t> &ids) {
    FILE *f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    const int32_t n = (int32_t)ids.size();
    bool ok = std::fwrite(&n, 4, 1, f) == 1 && std::fwrite(ids.data(), 4, ids.size(), f) == ids.size();
    return std::fclose(f) == 0 && ok;
}

std::string quote(const std::string &s) {   // for /bin/sh
    std::string q = "'";
    for (char c : s) q += c == '\'' ? std::string("'\\''") : std::string(1, c);
    return q + "'";
}

int run(const std::string &cmd) {
    const int rc = std::system(cmd.c_str());
    return rc == -1 ? -1 : WIFEXITED(rc) ? WEXITSTATUS(rc) : -1;
}

std::string json_escape(const std::string &s) {
    std::string o;
    for (unsigned char c : s) {
        if (c == '"') o += "\\\"";
        else if (c == '\\') o += "\\\\";
        else if (c == '\n') o += "\\n";
        else if (c == '\r') o += "\\r";
        else if (c == '\t') o += "\\t";
        else if (c < 0x20) { char b[8]; std::snprintf(b, sizeof b, "\\u%04x", c); o += b; }
        else o += (char)c;
    }
    return o;
}

// the scratch directory of the tokenizer files, removed on every way out of main
struct ScratchDir {
    std::string path;
    ~ScratchDir() {
        if (path.empty()) return;
        for (const char *f : {"prompt.txt", "tokens.bin", "output_tokens.bin", "output.txt"})
            std::remove((path + "/" + f).c_str());
        rmdir(path.c_str());
    }
};

int fail(const char *what, int st) {
    std::fprintf(stderr, "llama_generate: %s: %s (%s)\n", what, q35_status_string(st), q35_last_error());
    return 1;
}

}  // namespace

int main(int argc, char **argv) {
    Options o;
    env_defaults(o);
    if (!parse(argc, argv, o)) return 2;
    FILE *log = o.json ? stderr : stdout;   // with --json stdout carries the result only

    // ---- model shape ----
    q35_model_config c{};
    if (o.model == "70b") c = {80, 8192, 64, 8, 128, 28672, 32000, 2048, 1e-5f, 10000.0f, 0, Q35_FMT_3P5BIT, 1};
    else if (o.model == "13b") c = {40, 5120, 40, 40, 128, 13824, 32000, 2048, 1e-5f, 10000.0f, 0, Q35_FMT_3P5BIT, 1};
    else if (o.model == "tiny") c = {2, 512, 4, 2, 128, 1024, 1000, 96, 1e-5f, 10000.0f, 0, Q35_FMT_3P5BIT, 1};
    else { std::fprintf(stderr, "llama_generate: unknown model %s\n", o.model.c_str()); return 2; }
    if (o.n_layers > 0) c.n_layers = o.n_layers;
    if (o.hidden > 0) c.hidden = o.hidden;
    if (o.heads > 0) c.n_heads = o.heads;
    if (o.kv_heads > 0) c.n_kv_heads = o.kv_heads;
    if (o.head_dim > 0) c.head_dim = o.head_dim;
    if (o.ffn > 0) c.ffn = o.ffn;
    if (o.vocab > 0) c.vocab = o.vocab;
    if (o.max_seq > 0) c.max_seq = o.max_seq;
    c.rope_mode = o.rope_mode;
    c.wformat = o.format >= 0 ? o.format : (!o.layer_dir.empty() ? Q35_FMT_INT4 : Q35_FMT_3P5BIT);
    c.max_batch = 1;

    // ---- Step 1: prompt (:38-45) ----
    if (!o.have_prompt && o.tokens_in.empty()) {
        std::fprintf(log, " Enter prompt (or press Enter for default):\n");
        std::getline(std::cin, o.prompt);
    }
    if (o.prompt.find_first_not_of(" \t\r\n") == std::string::npos && o.tokens_in.empty()) {
        o.prompt = "Explain quantum computing in simple terms:";
        std::fprintf(log, " Using default prompt: %s\n", o.prompt.c_str());
    }

    // ---- Step 2: tokens (:47-53, :162-214) ----
    std::vector<int32_t> ids;
    char tmpdir[] = "/tmp/llama_generate_XXXXXX";
    const bool have_tmp = mkdtemp(tmpdir) != nullptr;
    const std::string td = have_tmp ? tmpdir : ".";
    ScratchDir scratch;
    if (have_tmp) scratch.path = td;
    bool tokenized = false;
    if (!o.tokens_in.empty()) {
        if (!read_ids(o.tokens_in, ids)) {
            std::fprintf(stderr, "llama_generate: cannot read token ids from %s\n", o.tokens_in.c_str());
            return 2;
        }
        tokenized = true;
    } else if (!o.tokenizer.empty()) {
        const std::string pf = td + "/prompt.txt", tf = td + "/tokens.bin";
        FILE *f = std::fopen(pf.c_str(), "w");
        if (f) { std::fprintf(f, "%s\n", o.prompt.c_str()); std::fclose(f); }
        if (f && run(o.tokenizer + " encode " + quote(pf) + " " + quote(tf)) == 0 && read_ids(tf, ids)) tokenized = true;
        else std::fprintf(stderr, " Warning: Tokenizer failed, using placeholder tokens\n");
    }
    if (!tokenized) {
        ids.clear();
        for (int i = 1; i <= 10; ++i) ids.push_back(i);      // :184-185
    }
    std::fprintf(log, " Prompt tokens: %zu\n", ids.size());

    // ---- Steps 3-4: model and weights (:55-64) ----
    q35_ctx ctx = nullptr;
    int st = q35_ctx_create(o.device, nullptr, &ctx);
    if (st) return fail("context", st);
    q35_model m = nullptr;
    st = q35_model_create(ctx, &c, &m);
    if (st) return fail("init_llama_model", st);
    if (!o.weights.empty()) {
        std::vector<const char *> ps;
        for (const std::string &w : o.weights) ps.push_back(w.c_str());
        st = q35_model_load_safetensors(m, ps.data(), (int32_t)ps.size());
        if (st) return fail("loading the checkpoint", st);
    } else {
        st = q35_model_init_random(m, o.init_seed, 0.02);
        if (st) return fail("random weights", st);
        if (!o.layer_dir.empty()) {
            for (int l = 0; l < c.n_layers; ++l) {
                const std::string p = o.layer_dir + "/weights_layer" + std::to_string(l) + ".bin";
                struct stat sb;
                if (stat(p.c_str(), &sb) != 0) continue;          // layers without a file stay random
                st = q35_model_load_layer_file(m, l, p.c_str());
                if (st) return fail(("load_layer_weights " + p).c_str(), st);
            }
        } else {
            std::fprintf(log, " No weight files given - using random initialization\n");
        }
    }

    // ---- Step 5: generation loop (:66-123) ----
    q35_sampling smp{};
    const std::string sm = o.sampler == "auto" ? (o.temperature > 0.0f ? "top_p" : "greedy") : o.sampler;
    if (sm == "greedy") smp.mode = Q35_SAMPLE_GREEDY;
    else if (sm == "temperature") smp.mode = Q35_SAMPLE_TEMPERATURE;
    else if (sm == "top_k") smp.mode = Q35_SAMPLE_TOP_K;
    else if (sm == "top_p") smp.mode = Q35_SAMPLE_TOP_P;
    else { std::fprintf(stderr, "llama_generate: unknown sampler %s\n", o.sampler.c_str()); return 2; }
    smp.temperature = o.temperature;
    smp.top_k = o.top_k;
    smp.top_p = o.top_p;
    smp.seed = o.seed;
    st = q35_model_set_sampling(m, &smp);
    if (st) return fail("sampling", st);
    const int plen = (int)ids.size();
    const int steps = std::max(0, std::min(o.max_tokens, c.max_seq - plen));
    std::vector<int32_t> out((size_t)std::max(1, steps));
    int32_t n_out = 0;
    const auto t0 = std::chrono::steady_clock::now();
    if (steps > 0) {
        st = q35_model_generate(m, ids.data(), plen, steps, o.stop_at_eos ? 1 : 0, out.data(), &n_out);
        if (st) return fail("generate", st);
    }
    const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::vector<int32_t> all(ids);
    all.insert(all.end(), out.begin(), out.begin() + n_out);
    const bool eos = o.stop_at_eos && n_out < steps;
    if (eos) std::fprintf(log, "\n [EOS]\n");
    else if (plen + n_out >= c.max_seq) std::fprintf(log, "\n [MAX LENGTH REACHED]\n");
    const double tps = secs > 0 ? n_out / secs : 0.0;

    std::fprintf(log, " Generation Statistics:\n");
    std::fprintf(log, "   Prompt tokens: %d\n", plen);
    std::fprintf(log, "   Generated tokens: %d\n", n_out);
    std::fprintf(log, "   Total tokens: %d\n", plen + n_out);
    std::fprintf(log, "   Time elapsed: %8.2f seconds\n", secs);
    std::fprintf(log, "   Throughput: %8.2f tokens/sec\n", tps);
    std::fprintf(log, "   Latency: %8.2f ms/token\n", tps > 0 ? 1000.0 / tps : 0.0);

    // ---- Step 6: detokenize (:141-148, :219-253) ----
    if (!o.tokens_out.empty() && !write_ids(o.tokens_out, all))
        std::fprintf(stderr, "llama_generate: cannot write %s\n", o.tokens_out.c_str());
    std::string text;
    bool detok = false;
    if (!o.tokenizer.empty()) {
        const std::string of = td + "/output_tokens.bin", xf = td + "/output.txt";
        if (write_ids(of, all) && run(o.tokenizer + " decode " + quote(of) + " " + quote(xf)) == 0) {
            FILE *f = std::fopen(xf.c_str(), "r");
            if (f) {
                char buf[4096];
                size_t n;
                while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
                std::fclose(f);
                while (!text.empty() && (text.back() == '\n' || text.back() == '\r')) text.pop_back();
                detok = true;
            }
        }
        if (!detok) text = "[Detokenization failed]";
    } else {
        for (int i = 0; i < n_out; ++i) text += (i ? " " : "") + std::to_string(out[i]);
    }
    if (o.json) {
        std::string idl;
        for (int i = 0; i < n_out; ++i) idl += (i ? "," : "") + std::to_string(out[i]);
        std::printf("{\"text\": \"%s\", \"tokens\": %d, \"prompt_tokens\": %d, \"token_ids\": [%s], "
                    "\"eos\": %s, \"time_s\": %.6f, \"tokens_per_sec\": %.3f}\n",
                    json_escape(text).c_str(), n_out, plen, idl.c_str(), eos ? "true" : "false", secs, tps);
    } else {
        std::printf(" Final output:\n ===========================================\n %s\n"
                    " ===========================================\n", text.c_str());
    }
    q35_model_destroy(m);
    q35_ctx_destroy(ctx);
    return 0;
}
