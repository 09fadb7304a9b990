// mocha-gguf-cli: the GGUF text-generation host for B200, driven with the llama-cli
// command line the reference launcher builds (mocha-llm:42-47):
//
//   mocha-gguf-cli -m MODEL.gguf -p TEXT -n N -c 1024 -b 32 -ub 32 -t THREADS -ngl 0
//                  -no-cnv --no-display-prompt --no-context-shift --temp T --seed S
//                  --repeat-penalty P --top-k K --top-p P
//
// with the launcher's environment: MOCHA_GGUF_CUDA=1 selects this GPU engine (the
// reference's `--backend cuda`); MOCHA_GGUF_CUDA=0 asks for llama.cpp's CPU path, which
// stays with llama-cli, so this host refuses it (exit 1).  MOCHA_GGUF_GPU_CACHE_MIB is
// accepted: the reference bridge caps its device weight cache with it, while here every
// weight is resident in HBM.
//
// The prompt text is tokenized from the file's tokenizer.ggml.* metadata (byte-level
// BPE; pre-tokenizers qwen2, llama-bpe and the GPT-2 rule; special tokens written in the
// text are recognised; BOS added when add_bos_token says so) -- the same rules as
// gguf_tokenizer.py.  The token loop runs on the device (mocha_gguf_generate):
// --temp 0 is greedy; otherwise penalty, top-k (at most 64), temperature, top-p and a
// xorshift32 draw seeded with --seed, the reference engine's sampling rule
// (src/minimind.cpp:160-179).  The generated text goes to stdout (control tokens print
// nothing, EOS ends the text); a summary line goes to stderr.
//
// -b, -ub, -t, -ngl, -no-cnv, --no-context-shift are accepted and have nothing to set:
// the prompt runs on the device in one pass, there is no CPU thread pool, no
// conversation mode, and prompt + N must fit the context (-c, at most the engine's).
// --no-display-prompt is the only behaviour: the prompt is never echoed.
// --print-token-ids prints the prompt's token ids and exits without touching a GPU.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "mocha_b200.h"
#include "unicode_tables.h"

namespace {

// ---- GGUF metadata ------------------------------------------------------------------

enum { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };

struct Meta {
    std::unordered_map<std::string, double> nums;
    std::unordered_map<std::string, std::string> strs;
    std::unordered_map<std::string, std::vector<std::string>> str_arrays;
    std::unordered_map<std::string, std::vector<int64_t>> int_arrays;
};

struct Reader {
    const uint8_t *p;
    size_t n, at = 0;
    bool ok = true;
    template <typename T>
    T get()
    {
        T v{};
        if (at + sizeof(T) > n) {
            ok = false;
            return v;
        }
        std::memcpy(&v, p + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    std::string str()
    {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > n - at) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char *>(p + at), (size_t)len);
        at += (size_t)len;
        return s;
    }
    double number(uint32_t t)
    {
        switch (t) {
        case T_U8: return get<uint8_t>();
        case T_I8: return get<int8_t>();
        case T_U16: return get<uint16_t>();
        case T_I16: return get<int16_t>();
        case T_U32: return get<uint32_t>();
        case T_I32: return get<int32_t>();
        case T_F32: return get<float>();
        case T_BOOL: return get<uint8_t>();
        case T_U64: return (double)get<uint64_t>();
        case T_I64: return (double)get<int64_t>();
        case T_F64: return get<double>();
        default: ok = false; return 0;
        }
    }
};

bool read_meta(const uint8_t *p, size_t n, Meta *m)
{
    Reader r{p, n};
    if (r.get<uint32_t>() != 0x46554747u) return false;  // "GGUF"
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) return false;
    r.get<uint64_t>();  // tensors
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || n_kv > (1u << 20)) return false;
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        if (t == T_STR) {
            m->strs[key] = r.str();
        } else if (t == T_ARR) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t count = r.get<uint64_t>();
            if (count > n) return false;
            if (et == T_STR) {
                auto &v = m->str_arrays[key];
                v.reserve((size_t)count);
                for (uint64_t j = 0; j < count && r.ok; j++) v.push_back(r.str());
            } else if (et == T_STR || et == T_ARR || et > T_F64) {
                return false;
            } else {
                auto &v = m->int_arrays[key];
                v.reserve((size_t)count);
                for (uint64_t j = 0; j < count && r.ok; j++) v.push_back((int64_t)r.number(et));
            }
        } else {
            m->nums[key] = r.number(t);
        }
    }
    return r.ok;
}

// ---- byte-level BPE tokenizer -------------------------------------------------------

bool in_table(const uint32_t (*t)[2], int count, uint32_t cp)
{
    int lo = 0, hi = count - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) / 2;
        if (cp < t[mid][0]) hi = mid - 1;
        else if (cp > t[mid][1]) lo = mid + 1;
        else return true;
    }
    return false;
}
bool is_l(uint32_t c) { return in_table(kLetter, kLetterCount, c); }
bool is_n(uint32_t c) { return in_table(kNumber, kNumberCount, c); }
bool is_s(uint32_t c) { return in_table(kSpace, kSpaceCount, c); }
bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }
bool is_other(uint32_t c) { return !is_s(c) && !is_l(c) && !is_n(c); }

std::vector<uint32_t> utf8_decode(const std::string &s)
{
    std::vector<uint32_t> out;
    for (size_t i = 0; i < s.size();) {
        const uint8_t c = (uint8_t)s[i];
        int len = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
        if (len == 0 || i + len > s.size()) {  // invalid byte: U+FFFD, as a decoder replacing errors does
            out.push_back(0xFFFD);
            i++;
            continue;
        }
        uint32_t cp = len == 1 ? c : len == 2 ? c & 0x1F : len == 3 ? c & 0x0F : c & 0x07;
        for (int k = 1; k < len; k++) cp = (cp << 6) | ((uint8_t)s[i + k] & 0x3F);
        out.push_back(cp);
        i += len;
    }
    return out;
}

void utf8_append(std::string &s, uint32_t cp)
{
    if (cp < 0x80) {
        s += (char)cp;
    } else if (cp < 0x800) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xF0 | (cp >> 18));
        s += (char)(0x80 | ((cp >> 12) & 0x3F));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

uint32_t lower_ascii(uint32_t c) { return c >= 'A' && c <= 'Z' ? c + 32 : c; }

// End of the pre-tokenizer piece starting at i.  modern: the qwen2 / llama-bpe pattern
//   (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,D}| ?[^\s\p{L}\p{N}]+[\r\n]*
//   |\s*[\r\n]+|\s+(?!\S)|\s+
// with D = digits (1 for qwen2, 3 for llama-bpe); otherwise the GPT-2 pattern
//   's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
// Alternatives are tried in order, as a regular-expression engine does.
size_t piece_end(const std::vector<uint32_t> &c, size_t i, bool modern, int digits)
{
    const size_t n = c.size();
    auto run = [&](size_t j, bool (*pred)(uint32_t)) {
        while (j < n && pred(c[j])) j++;
        return j;
    };
    if (c[i] == '\'' && i + 1 < n) {  // contractions
        const uint32_t a = modern ? lower_ascii(c[i + 1]) : c[i + 1];
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
        if (i + 2 < n) {
            const uint32_t b = modern ? lower_ascii(c[i + 2]) : c[i + 2];
            if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return i + 3;
        }
    }
    if (modern) {
        if (is_l(c[i])) return run(i + 1, is_l);
        if (!is_nl(c[i]) && !is_l(c[i]) && !is_n(c[i]) && i + 1 < n && is_l(c[i + 1])) return run(i + 2, is_l);
        if (is_n(c[i])) {
            size_t j = i + 1;
            while (j < n && (int)(j - i) < digits && is_n(c[j])) j++;
            return j;
        }
        size_t o = (c[i] == ' ' && i + 1 < n && is_other(c[i + 1])) ? i + 1 : i;
        if (is_other(c[o])) return run(run(o + 1, is_other), is_nl);
        // white space run [i, k)
        const size_t k = run(i, is_s);
        for (size_t p = k; p > i; p--)
            if (is_nl(c[p - 1])) return p;  // \s*[\r\n]+ ends after the run's last line break
        if (k == n) return k;                // \s+(?!\S) at the end of the text
        if (k - i >= 2) return k - 1;        // \s+(?!\S): leave the last space to the next piece
        return k;                            // \s+
    }
    size_t o = (c[i] == ' ' && i + 1 < n) ? i + 1 : i;
    if (is_l(c[o])) return run(o + 1, is_l);
    if (is_n(c[o])) return run(o + 1, is_n);
    if (is_other(c[o])) return run(o + 1, is_other);
    const size_t k = run(i, is_s);
    if (k == n) return k;
    if (k - i >= 2) return k - 1;
    return k;
}

struct Tokenizer {
    std::vector<std::string> tokens;
    std::vector<int> types;
    std::unordered_map<std::string, int> ids;
    std::unordered_map<std::string, int> ranks;  // "left right" -> rank
    std::vector<std::pair<std::string, int>> special;  // text, id; longest first
    std::string byte_char[256];                        // GPT-2 byte alphabet as UTF-8
    std::unordered_map<uint32_t, uint8_t> char_byte;
    bool modern = false;
    int digits = 1, bos = -1, eos = -1;
    bool add_bos = false;

    bool load(const Meta &m, std::string *why)
    {
        auto s = m.strs.find("tokenizer.ggml.model");
        if (s == m.strs.end() || s->second != "gpt2") {
            *why = "tokenizer.ggml.model is not gpt2 (byte-level BPE)";
            return false;
        }
        auto t = m.str_arrays.find("tokenizer.ggml.tokens");
        if (t == m.str_arrays.end()) {
            *why = "no tokenizer.ggml.tokens";
            return false;
        }
        tokens = t->second;
        types.assign(tokens.size(), 1);
        auto ty = m.int_arrays.find("tokenizer.ggml.token_type");
        if (ty != m.int_arrays.end())
            for (size_t i = 0; i < tokens.size() && i < ty->second.size(); i++) types[i] = (int)ty->second[i];
        for (size_t i = 0; i < tokens.size(); i++) ids.emplace(tokens[i], (int)i);
        auto mg = m.str_arrays.find("tokenizer.ggml.merges");
        if (mg != m.str_arrays.end())
            for (size_t i = 0; i < mg->second.size(); i++) ranks.emplace(mg->second[i], (int)i);
        auto pre = m.strs.find("tokenizer.ggml.pre");
        const std::string p = pre == m.strs.end() ? "" : pre->second;
        modern = p == "qwen2" || p == "llama-bpe";
        digits = p == "llama-bpe" ? 3 : 1;
        auto num = [&](const char *k, double d) {
            auto it = m.nums.find(k);
            return it == m.nums.end() ? d : it->second;
        };
        bos = (int)num("tokenizer.ggml.bos_token_id", -1);
        eos = (int)num("tokenizer.ggml.eos_token_id", -1);
        add_bos = num("tokenizer.ggml.add_bos_token", 0) != 0;
        for (size_t i = 0; i < tokens.size(); i++)
            if ((types[i] == 3 || types[i] == 4) && !tokens[i].empty()) special.emplace_back(tokens[i], (int)i);
        std::stable_sort(special.begin(), special.end(),
                         [](const auto &a, const auto &b) { return a.first.size() > b.first.size(); });
        // GPT-2's byte alphabet: printable bytes map to themselves, the rest to 256 + n
        int n = 0;
        for (int b = 0; b < 256; b++) {
            const bool printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
            const uint32_t cp = printable ? (uint32_t)b : 256u + (uint32_t)n++;
            byte_char[b].clear();
            utf8_append(byte_char[b], cp);
            char_byte[cp] = (uint8_t)b;
        }
        return true;
    }

    void bpe(const std::string &piece_bytes, std::vector<int> &out)
    {
        std::vector<std::string> w;
        for (unsigned char b : piece_bytes) w.push_back(byte_char[b]);
        while (w.size() > 1) {
            int best = -1, best_rank = 0;
            for (size_t i = 0; i + 1 < w.size(); i++) {
                auto it = ranks.find(w[i] + " " + w[i + 1]);
                if (it != ranks.end() && (best < 0 || it->second < best_rank)) {
                    best = (int)i;
                    best_rank = it->second;
                }
            }
            if (best < 0) break;
            const std::string left = w[best], right = w[best + 1];
            std::vector<std::string> merged;
            for (size_t i = 0; i < w.size();) {
                if (i + 1 < w.size() && w[i] == left && w[i + 1] == right) {
                    merged.push_back(left + right);
                    i += 2;
                } else {
                    merged.push_back(w[i]);
                    i++;
                }
            }
            w.swap(merged);
        }
        for (const std::string &p : w) {
            auto it = ids.find(p);
            if (it != ids.end()) {
                out.push_back(it->second);
            } else {  // not in the vocabulary: its single characters
                for (uint32_t cp : utf8_decode(p)) {
                    std::string ch;
                    utf8_append(ch, cp);
                    auto jt = ids.find(ch);
                    if (jt != ids.end()) out.push_back(jt->second);
                }
            }
        }
    }

    void encode_plain(const std::string &text, std::vector<int> &out)
    {
        const std::vector<uint32_t> c = utf8_decode(text);
        for (size_t i = 0; i < c.size();) {
            const size_t j = piece_end(c, i, modern, digits);
            std::string bytes;
            for (size_t k = i; k < j; k++) utf8_append(bytes, c[k]);
            bpe(bytes, out);
            i = j;
        }
    }

    std::vector<int> encode(const std::string &text)
    {
        std::vector<int> out;
        if (add_bos && bos >= 0) out.push_back(bos);
        size_t start = 0, i = 0;
        while (i < text.size()) {
            int hit = -1;
            size_t len = 0;
            for (const auto &sp : special)
                if (text.compare(i, sp.first.size(), sp.first) == 0) {
                    hit = sp.second;
                    len = sp.first.size();
                    break;
                }
            if (hit < 0) {
                i++;
                continue;
            }
            encode_plain(text.substr(start, i - start), out);
            out.push_back(hit);
            i += len;
            start = i;
        }
        encode_plain(text.substr(start), out);
        if (add_bos && out.size() > 1 && out[0] == bos && out[1] == bos)
            fprintf(stderr, "mocha-gguf-cli: the prompt starts with a BOS token and one was added: two BOS tokens\n");
        return out;
    }

    std::string piece(int id) const
    {
        if (id < 0 || id >= (int)tokens.size() || types[id] == 3) return {};
        if (types[id] == 4) return tokens[id];
        std::string out;
        for (uint32_t cp : utf8_decode(tokens[id])) {
            auto it = char_byte.find(cp);
            if (it != char_byte.end()) out += (char)it->second;
        }
        return out;
    }
};

// ---- command line -------------------------------------------------------------------

struct Args {
    std::string model, prompt;
    int n_predict = -1, ctx = 0, top_k = 40;
    float temp = 0.8f, repeat_penalty = 1.0f, top_p = 0.95f;
    long long seed = -1;
    bool print_ids = false;
};

int usage(const char *why)
{
    fprintf(stderr, "mocha-gguf-cli: %s\n", why);
    fprintf(stderr,
            "usage: mocha-gguf-cli -m MODEL.gguf -p TEXT [-n N] [-c CTX] [--temp T] [--seed S] "
            "[--repeat-penalty P] [--top-k K] [--top-p P] [-b N] [-ub N] [-t N] [-ngl N] [-no-cnv] "
            "[--no-display-prompt] [--no-context-shift] [--print-token-ids]\n");
    return 1;
}

bool parse(int argc, char **argv, Args *a, std::string *why)
{
    for (int i = 1; i < argc; i++) {
        const std::string k = argv[i];
        auto value = [&](const char *name) -> const char * {
            if (i + 1 >= argc) {
                *why = std::string("missing value for ") + name;
                return nullptr;
            }
            return argv[++i];
        };
        const char *v = nullptr;
        if (k == "-m" || k == "--model") {
            if (!(v = value("-m"))) return false;
            a->model = v;
        } else if (k == "-p" || k == "--prompt") {
            if (!(v = value("-p"))) return false;
            a->prompt = v;
        } else if (k == "-n" || k == "--n-predict") {
            if (!(v = value("-n"))) return false;
            a->n_predict = atoi(v);
        } else if (k == "-c" || k == "--ctx-size") {
            if (!(v = value("-c"))) return false;
            a->ctx = atoi(v);
        } else if (k == "--temp") {
            if (!(v = value("--temp"))) return false;
            a->temp = (float)atof(v);
        } else if (k == "--seed" || k == "-s") {
            if (!(v = value("--seed"))) return false;
            a->seed = atoll(v);
        } else if (k == "--repeat-penalty") {
            if (!(v = value("--repeat-penalty"))) return false;
            a->repeat_penalty = (float)atof(v);
        } else if (k == "--top-k") {
            if (!(v = value("--top-k"))) return false;
            a->top_k = atoi(v);
        } else if (k == "--top-p") {
            if (!(v = value("--top-p"))) return false;
            a->top_p = (float)atof(v);
        } else if (k == "-b" || k == "--batch-size" || k == "-ub" || k == "--ubatch-size" || k == "-t" ||
                   k == "--threads" || k == "-ngl" || k == "--n-gpu-layers" || k == "--gpu-layers") {
            if (!value(k.c_str())) return false;  // nothing to set on this engine
        } else if (k == "-no-cnv" || k == "--no-conversation" || k == "--no-display-prompt" ||
                   k == "--no-context-shift") {
            // conversation mode, prompt echo and context shifting do not exist here
        } else if (k == "--print-token-ids") {
            a->print_ids = true;
        } else {
            *why = "unknown argument " + k;
            return false;
        }
    }
    if (a->model.empty()) {
        *why = "no model (-m)";
        return false;
    }
    return true;
}

double now() { return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count(); }

}  // namespace

int main(int argc, char **argv)
{
    Args a;
    std::string why;
    if (!parse(argc, argv, &a, &why)) return usage(why.c_str());
    const char *cuda = getenv("MOCHA_GGUF_CUDA");
    if (!a.print_ids && cuda && strcmp(cuda, "0") == 0) {
        fprintf(stderr, "mocha-gguf-cli: MOCHA_GGUF_CUDA=0 asks for the CPU backend, which is llama-cli's; "
                        "this host runs the B200 engine only\n");
        return 1;
    }
    const double t_start = now();
    const int fd = open(a.model.c_str(), O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st)) return usage("cannot open the model file");
    void *base = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (base == MAP_FAILED) return usage("cannot map the model file");
    Meta meta;
    Tokenizer tok;
    if (!read_meta(static_cast<const uint8_t *>(base), (size_t)st.st_size, &meta)) return usage("not a GGUF v2/v3 file");
    if (!tok.load(meta, &why)) return usage(why.c_str());
    const std::vector<int> prompt = tok.encode(a.prompt);
    if (a.print_ids) {
        for (size_t i = 0; i < prompt.size(); i++) printf("%d%c", prompt[i], i + 1 == prompt.size() ? '\n' : ' ');
        if (prompt.empty()) printf("\n");
        munmap(base, (size_t)st.st_size);
        return 0;
    }
    if (prompt.empty()) return usage("empty prompt");
    const char *cache = getenv("MOCHA_GGUF_GPU_CACHE_MIB");
    if (cache) fprintf(stderr, "mocha-gguf-cli: MOCHA_GGUF_GPU_CACHE_MIB=%s: every weight stays resident in HBM\n", cache);
    mocha_gguf *m = nullptr;
    if (mocha_gguf_open(0, base, (unsigned long long)st.st_size, &m)) {
        munmap(base, (size_t)st.st_size);
        return 1;
    }
    mocha_gguf_info info{};
    mocha_gguf_get_info(m, &info);
    const int ctx = a.ctx > 0 ? std::min(a.ctx, info.context) : info.context;
    int n_new = a.n_predict < 0 ? ctx - (int)prompt.size() : a.n_predict;
    if ((int)prompt.size() >= ctx || n_new < 1 || (int)prompt.size() + n_new > ctx) {
        fprintf(stderr, "mocha-gguf-cli: prompt %zu + %d tokens exceed the context %d\n", prompt.size(), n_new, ctx);
        mocha_gguf_close(m);
        munmap(base, (size_t)st.st_size);
        return 1;
    }
    mocha_sampling s{};
    s.temperature = a.temp > 0.f ? a.temp : 0.f;
    s.top_k = a.top_k < 1 ? 1 : a.top_k;
    if (s.temperature > 0.f && s.top_k > 64) {
        fprintf(stderr, "mocha-gguf-cli: --top-k %d above the device sampler's 64: using 64\n", s.top_k);
        s.top_k = 64;
    }
    s.top_p = a.top_p > 0.f && a.top_p <= 1.f ? a.top_p : 1.f;
    s.repeat_penalty = a.repeat_penalty >= 1.f ? a.repeat_penalty : 1.f;
    s.seed = a.seed < 0 ? (unsigned)std::chrono::steady_clock::now().time_since_epoch().count() : (unsigned)a.seed;
    if (s.seed == 0) s.seed = 1;  // xorshift32 needs a nonzero state
    std::vector<int> out((size_t)n_new);
    int n_out = 0;
    mocha_timing t{};
    const double t_ready = now();
    const int rc = mocha_gguf_generate(m, prompt.data(), (int)prompt.size(), n_new, &s, out.data(), &n_out, &t);
    if (rc == 0) {
        std::string text;
        for (int i = 0; i < n_out; i++) text += tok.piece(out[(size_t)i]);
        fwrite(text.data(), 1, text.size(), stdout);
        fflush(stdout);
        fprintf(stderr,
                "\nBACKEND=cuda MODEL_ARCH=%s PROMPT_TOKENS=%zu GENERATED=%d STARTUP_S=%.3f PREFILL_S=%.3f "
                "DECODE_TPS=%.3f WALL_S=%.3f\n",
                info.arch == 0 ? "llama" : "qwen2", prompt.size(), n_out, t_ready - t_start, t.prefill_s,
                t.generated > 1 && t.decode_s > 0 ? (t.generated - 1) / t.decode_s : 0.0, now() - t_start);
    }
    mocha_gguf_close(m);
    munmap(base, (size_t)st.st_size);
    return rc ? 1 : 0;
}
