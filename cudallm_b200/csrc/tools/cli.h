// Command-line options and JSON output of the command-line tools (cudallm_bench, cudallm_kernelbench,
// cudallm_bandwidth). The tools keep the flags and JSON keys of wasiqnauman/cudallm's tools
// (src/tools/*.cpp), which its bench scripts (bench/bench_decode.py, bench_bandwidth.py, sweep_matvec.py)
// pass and read.
//
// Options are declared up front (name, default, help); parse() accepts "--name value" and, for booleans,
// "--name 0|1"; anything undeclared, a missing value or a malformed number prints the usage and exits with
// status 2. JsonValue is a small ordered tree written out once at the end.
#pragma once

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

namespace cudallm::tools {

class Options {
public:
    Options(std::string tool, std::string synopsis) : tool_(std::move(tool)), synopsis_(std::move(synopsis)) {}

    Options& add(const std::string& name, const std::string& def, const std::string& help) {
        order_.push_back(name);
        spec_[name] = {def, help};
        return *this;
    }

    void parse(int argc, char** argv) {
        for (int i = 1; i < argc; ++i) {
            const std::string tok = argv[i];
            if (tok == "--help" || tok == "-h") usage(0);
            if (tok.rfind("--", 0) != 0) die("unexpected argument '" + tok + "'");
            const std::string name = tok.substr(2);
            if (!spec_.count(name)) die("unknown option '" + tok + "'");
            if (i + 1 >= argc) die("option '" + tok + "' needs a value");
            given_[name] = argv[++i];
        }
    }

    bool given(const std::string& name) const { return given_.count(name) != 0; }

    std::string str(const std::string& name) const {
        auto g = given_.find(name);
        return g != given_.end() ? g->second : spec_.at(name).def;
    }

    long long integer(const std::string& name) const {
        const std::string v = str(name);
        char* end = nullptr;
        const long long r = std::strtoll(v.c_str(), &end, 10);
        if (v.empty() || *end != '\0') die("option '--" + name + "' expects an integer, got '" + v + "'");
        return r;
    }

    bool flag(const std::string& name) const {
        const std::string v = str(name);
        if (v == "1" || v == "true") return true;
        if (v == "0" || v == "false") return false;
        die("option '--" + name + "' expects 0 or 1, got '" + v + "'");
    }

    std::string choice(const std::string& name, const std::vector<std::string>& allowed) const {
        const std::string v = str(name);
        for (const auto& a : allowed) {
            if (a == v) return v;
        }
        std::string list;
        for (const auto& a : allowed) list += (list.empty() ? "" : "|") + a;
        die("option '--" + name + "' must be " + list + ", got '" + v + "'");
    }

    [[noreturn]] void die(const std::string& msg) const {
        std::fprintf(stderr, "%s: %s\n", tool_.c_str(), msg.c_str());
        usage(2);
    }

    [[noreturn]] void usage(int status) const {
        std::FILE* f = status ? stderr : stdout;
        std::fprintf(f, "usage: %s %s\n", tool_.c_str(), synopsis_.c_str());
        for (const auto& n : order_) {
            const Spec& s = spec_.at(n);
            std::fprintf(f, "  --%-14s %s%s\n", n.c_str(), s.help.c_str(),
                         s.def.empty() ? "" : (" (default " + s.def + ")").c_str());
        }
        std::exit(status);
    }

private:
    struct Spec {
        std::string def, help;
    };
    std::string tool_, synopsis_;
    std::vector<std::string> order_;
    std::map<std::string, Spec> spec_;
    std::map<std::string, std::string> given_;
};

// Ordered JSON value: null, bool, number, string, array or object.
class JsonValue {
public:
    JsonValue() = default;
    JsonValue(bool b) : kind_(Kind::BOOL), b_(b) {}                                            // NOLINT
    JsonValue(int v) : kind_(Kind::INT), i_(v) {}                                              // NOLINT
    JsonValue(long long v) : kind_(Kind::INT), i_(v) {}                                        // NOLINT
    JsonValue(unsigned long long v) : kind_(Kind::INT), i_(static_cast<long long>(v)) {}       // NOLINT
    JsonValue(unsigned long v) : kind_(Kind::INT), i_(static_cast<long long>(v)) {}            // NOLINT
    JsonValue(double v) : kind_(Kind::NUM), d_(v) {}                                           // NOLINT
    JsonValue(const char* s) : kind_(Kind::STR), s_(s) {}                                      // NOLINT
    JsonValue(std::string s) : kind_(Kind::STR), s_(std::move(s)) {}                           // NOLINT

    static JsonValue object() {
        JsonValue v;
        v.kind_ = Kind::OBJ;
        return v;
    }
    static JsonValue array() {
        JsonValue v;
        v.kind_ = Kind::ARR;
        return v;
    }

    // Object member (added in order on first use).
    JsonValue& operator[](const std::string& key) {
        for (auto& kv : members_) {
            if (kv.first == key) return kv.second;
        }
        members_.emplace_back(key, JsonValue());
        return members_.back().second;
    }
    JsonValue& push(JsonValue v) {
        items_.push_back(std::move(v));
        return items_.back();
    }

    std::string dump(int indent = 0) const {
        std::ostringstream o;
        write(o, indent, 0);
        return o.str();
    }

    bool write_file(const std::string& path) const {
        std::FILE* f = std::fopen(path.c_str(), "w");
        if (f == nullptr) return false;
        const std::string s = dump(2) + "\n";
        const bool ok = std::fwrite(s.data(), 1, s.size(), f) == s.size();
        return std::fclose(f) == 0 && ok;
    }

private:
    enum class Kind { NUL, BOOL, INT, NUM, STR, ARR, OBJ };

    static void quote(std::ostringstream& o, const std::string& s) {
        o << '"';
        for (char c : s) {
            switch (c) {
                case '"': o << "\\\""; break;
                case '\\': o << "\\\\"; break;
                case '\n': o << "\\n"; break;
                case '\t': o << "\\t"; break;
                default:
                    if (static_cast<unsigned char>(c) < 0x20) {
                        char buf[8];
                        std::snprintf(buf, sizeof(buf), "\\u%04x", c);
                        o << buf;
                    } else {
                        o << c;
                    }
            }
        }
        o << '"';
    }

    void write(std::ostringstream& o, int indent, int depth) const {
        const std::string pad = indent ? std::string(static_cast<size_t>(indent) * (depth + 1), ' ') : "";
        const std::string close = indent ? std::string(static_cast<size_t>(indent) * depth, ' ') : "";
        const char* nl = indent ? "\n" : "";
        switch (kind_) {
            case Kind::NUL: o << "null"; break;
            case Kind::BOOL: o << (b_ ? "true" : "false"); break;
            case Kind::INT: o << i_; break;
            case Kind::NUM:
                if (std::isfinite(d_)) {
                    char buf[32];
                    std::snprintf(buf, sizeof(buf), "%.17g", d_);
                    o << buf;
                } else {
                    o << "null";
                }
                break;
            case Kind::STR: quote(o, s_); break;
            case Kind::ARR:
                o << '[' << nl;
                for (size_t i = 0; i < items_.size(); ++i) {
                    o << pad;
                    items_[i].write(o, indent, depth + 1);
                    o << (i + 1 < items_.size() ? "," : "") << nl;
                }
                o << close << ']';
                break;
            case Kind::OBJ:
                o << '{' << nl;
                for (size_t i = 0; i < members_.size(); ++i) {
                    o << pad;
                    quote(o, members_[i].first);
                    o << (indent ? ": " : ":");
                    members_[i].second.write(o, indent, depth + 1);
                    o << (i + 1 < members_.size() ? "," : "") << nl;
                }
                o << close << '}';
                break;
        }
    }

    Kind kind_ = Kind::NUL;
    bool b_ = false;
    long long i_ = 0;
    double d_ = 0;
    std::string s_;
    std::vector<JsonValue> items_;
    std::vector<std::pair<std::string, JsonValue>> members_;
};

}  // namespace cudallm::tools
