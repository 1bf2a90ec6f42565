// server.cpp -- HTTP/1.1 front end over the engine: see server.h. Request framing
// (header block, then exactly Content-Length body bytes; chunked bodies refused), the
// routes, their status codes and the response fields follow src/app/Opure_Server.cpp;
// the socket handling and the per-GPU worker pool are this build's own.
#include "server.h"

#include <arpa/inet.h>
#include <netinet/in.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <chrono>
#include <cstdlib>
#include <cstdio>
#include <cstring>

#include "json.h"
#include "platform.h"
#include "sample_decode.h"

namespace opure::server {

namespace {

const char *Reason(int status) {
    switch (status) {
        case 200: return "OK";
        case 400: return "Bad Request";
        case 404: return "Not Found";
        case 405: return "Method Not Allowed";
        case 413: return "Payload Too Large";
        case 503: return "Service Unavailable";
        default: return "Internal Server Error";
    }
}

bool SendAll(int fd, std::string_view data) {
    size_t sent = 0;
    while (sent < data.size()) {
        const ssize_t n = ::send(fd, data.data() + sent, data.size() - sent, MSG_NOSIGNAL);
        if (n <= 0) return false;
        sent += size_t(n);
    }
    return true;
}

void Send(int fd, const Response &r) {
    char head[256];
    const int n = std::snprintf(head, sizeof(head),
                                "HTTP/1.1 %d %s\r\nContent-Type: application/json\r\nContent-Length: %zu\r\n"
                                "Connection: close\r\n\r\n",
                                r.status, Reason(r.status), r.body.size());
    if (SendAll(fd, std::string_view(head, size_t(n)))) SendAll(fd, r.body);
}

std::string_view Trim(std::string_view s) {
    while (!s.empty() && (s.front() == ' ' || s.front() == '\t')) s.remove_prefix(1);
    while (!s.empty() && (s.back() == ' ' || s.back() == '\t')) s.remove_suffix(1);
    return s;
}

bool IEquals(std::string_view a, std::string_view b) {
    if (a.size() != b.size()) return false;
    for (size_t i = 0; i < a.size(); ++i)
        if (std::tolower(static_cast<unsigned char>(a[i])) != std::tolower(static_cast<unsigned char>(b[i])))
            return false;
    return true;
}

// Value of header `name` (case-insensitive, at a line start) in the header block, or "".
std::string_view Header(std::string_view head, std::string_view name) {
    size_t line = 0;
    while (line < head.size()) {
        size_t end = head.find("\r\n", line);
        if (end == std::string_view::npos) end = head.size();
        const std::string_view l = head.substr(line, end - line);
        const size_t colon = l.find(':');
        if (colon != std::string_view::npos && IEquals(Trim(l.substr(0, colon)), name))
            return Trim(l.substr(colon + 1));
        line = end + 2;
    }
    return {};
}

// Reads one request from fd within 10 s: the header block, then exactly Content-Length
// body bytes. Returns false when the peer closes, stalls or sends a header block over
// 64 KB; *too_large is set (and nothing more is read) when Content-Length exceeds
// kMaxBodyBytes.
bool ReadRequest(int fd, std::string &raw, bool *too_large) {
    *too_large = false;
    raw.clear();
    char buf[4096];
    size_t hdr_end = std::string::npos, need = 0;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        if (hdr_end != std::string::npos && raw.size() >= need) return true;
        const auto left = std::chrono::milliseconds(10000) - (std::chrono::steady_clock::now() - t0);
        if (left.count() <= 0) return false;
        pollfd p{fd, POLLIN, 0};
        if (::poll(&p, 1, int(std::chrono::duration_cast<std::chrono::milliseconds>(left).count())) <= 0) return false;
        const ssize_t n = ::recv(fd, buf, sizeof(buf), 0);
        if (n <= 0) return false;
        raw.append(buf, size_t(n));
        if (hdr_end == std::string::npos) {
            hdr_end = raw.find("\r\n\r\n");
            if (hdr_end == std::string::npos) {
                if (raw.size() > 64 * 1024) return false;  // no header block that long
                continue;
            }
            const std::string_view cl = Header(std::string_view(raw.data(), hdr_end), "Content-Length");
            const unsigned long long len = cl.empty() ? 0ull : std::strtoull(std::string(cl).c_str(), nullptr, 10);
            if (len > kMaxBodyBytes) {
                *too_large = true;
                return true;
            }
            need = hdr_end + 4 + size_t(len);
        }
    }
}

}  // namespace

std::string JsonString(std::string_view s) {
    std::string out = "\"";
    for (const char c : s) {
        switch (c) {
            case '"': out += "\\\""; break;
            case '\\': out += "\\\\"; break;
            case '\n': out += "\\n"; break;
            case '\r': out += "\\r"; break;
            case '\t': out += "\\t"; break;
            default:
                if (static_cast<unsigned char>(c) < 0x20) {
                    char b[8];
                    std::snprintf(b, sizeof(b), "\\u%04x", unsigned(static_cast<unsigned char>(c)));
                    out += b;
                } else {
                    out += c;
                }
        }
    }
    return out + "\"";
}

bool ParseGenerate(std::string_view body, uint32_t vocab, GenerateRequest &out, std::string &err) {
    out = GenerateRequest{};
    json::Value v;
    try {
        v = json::ParseObject(body, "/generate");
    } catch (const std::exception &e) {
        err = e.what();
        return false;
    }
    const json::Value *toks = v.Find("tokens");
    if (!toks) {
        err = v.Find("prompt") ? "this server loads no tokenizer: send the prompt as token ids in \"tokens\""
                               : "missing \"tokens\"";
        return false;
    }
    if (!toks->IsArray() || toks->arr.empty()) {
        err = "\"tokens\" must be a non-empty array of token ids";
        return false;
    }
    for (const json::Value &t : toks->arr) {
        if (!t.IsNumber() || !t.integral || t.inum < 0 || (vocab && t.inum >= int64_t(vocab))) {
            err = "\"tokens\" holds an entry that is not a token id of this model";
            return false;
        }
        out.tokens.push_back(uint32_t(t.inum));
    }
    if (const json::Value *m = v.Find("max_tokens")) {
        if (!m->IsNumber()) {
            err = "\"max_tokens\" must be a number";
            return false;
        }
        const double n = m->num;
        out.maxTokens = n < 1.0 ? 1u : (n > double(kMaxNewTokens) ? kMaxNewTokens : uint32_t(n));
    }
    if (const json::Value *t = v.Find("temperature")) {
        if (!t->IsNumber()) {
            err = "\"temperature\" must be a number";
            return false;
        }
        out.temperature = t->num < 0.0 ? 0.0f : float(t->num);
    }
    if (const json::Value *s = v.Find("seed")) {
        if (!s->IsNumber() || !s->integral || s->inum < 0) {
            err = "\"seed\" must be a non-negative integer";
            return false;
        }
        out.seed = uint64_t(s->inum);
    }
    return true;
}

Server::Server(std::vector<std::unique_ptr<engine::VoxelEngine>> engines, uint16_t port)
    : engines_(std::move(engines)) {
    listenFd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    OPURE_CHECK(listenFd_ >= 0, "socket() failed");
    const int one = 1;
    ::setsockopt(listenFd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_addr.s_addr = htonl(INADDR_LOOPBACK);  // loopback only, as the reference
    a.sin_port = htons(port);
    if (::bind(listenFd_, reinterpret_cast<sockaddr *>(&a), sizeof(a)) != 0 || ::listen(listenFd_, 128) != 0) {
        ::close(listenFd_);
        ThrowError("cannot listen on 127.0.0.1:" + std::to_string(port));
    }
    socklen_t len = sizeof(a);
    ::getsockname(listenFd_, reinterpret_cast<sockaddr *>(&a), &len);
    port_ = ntohs(a.sin_port);
    const int n = std::max<int>(1, int(engines_.size()));
    for (int w = 0; w < n; ++w) workers_.emplace_back(&Server::Worker, this, engines_.empty() ? -1 : w);
    acceptThread_ = std::thread(&Server::AcceptLoop, this);
}

Server::~Server() { Stop(); }

void Server::Stop() {
    if (stop_.exchange(true)) return;
    ::shutdown(listenFd_, SHUT_RDWR);
    if (acceptThread_.joinable()) acceptThread_.join();
    ::close(listenFd_);
    cv_.notify_all();
    for (auto &t : workers_)
        if (t.joinable()) t.join();
    for (int fd : queue_) ::close(fd);
    queue_.clear();
}

void Server::AcceptLoop() {
    while (!stop_) {
        pollfd p{listenFd_, POLLIN, 0};
        if (::poll(&p, 1, 100) <= 0) continue;
        const int fd = ::accept(listenFd_, nullptr, nullptr);
        if (fd < 0) continue;  // a failed accept must not end the loop
        {
            std::lock_guard<std::mutex> lk(mu_);
            queue_.push_back(fd);
        }
        cv_.notify_one();
    }
}

void Server::Worker(int slot) {
    for (;;) {
        int fd;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
            if (queue_.empty()) return;  // stopping
            fd = queue_.front();
            queue_.pop_front();
        }
        std::string raw;
        bool too_large = false;
        if (ReadRequest(fd, raw, &too_large)) {
            if (too_large)
                Send(fd, Response{413, R"({"error":"request body too large"})"});
            else
                Send(fd, Handle(raw, slot));
        }
        // Lingering close: stop sending, then discard what the client still sends (an
        // oversized body answered early) for up to 2 s, so it can read the response
        // instead of meeting a reset.
        ::shutdown(fd, SHUT_WR);
        char sink[4096];
        const auto t0 = std::chrono::steady_clock::now();
        for (size_t drained = 0; drained < (size_t(16) << 20);) {
            pollfd p{fd, POLLIN, 0};
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2) || ::poll(&p, 1, 200) <= 0) break;
            const ssize_t n = ::recv(fd, sink, sizeof(sink), 0);
            if (n <= 0) break;
            drained += size_t(n);
        }
        ::close(fd);
    }
}

Response Server::Handle(std::string_view raw, int slot) {
    const size_t hdr_end = raw.find("\r\n\r\n");
    if (hdr_end == std::string_view::npos) return {400, R"({"error":"malformed request"})"};
    const std::string_view head = raw.substr(0, hdr_end);
    if (!Header(head, "Transfer-Encoding").empty())
        return {400, R"({"error":"chunked transfer-encoding not supported; send Content-Length"})"};
    const std::string_view cl = Header(head, "Content-Length");
    const size_t len = cl.empty() ? 0 : size_t(std::strtoull(std::string(cl).c_str(), nullptr, 10));
    if (len > kMaxBodyBytes) return {413, R"({"error":"request body too large"})"};
    if (raw.size() < hdr_end + 4 + len) return {400, R"({"error":"body shorter than Content-Length"})"};
    const std::string_view body = raw.substr(hdr_end + 4, len);  // exactly Content-Length bytes

    const size_t line_end = head.find("\r\n");
    const std::string_view line = head.substr(0, line_end);
    const size_t sp1 = line.find(' ');
    if (sp1 == std::string_view::npos) return {400, R"({"error":"malformed request line"})"};
    const std::string_view method = line.substr(0, sp1);
    const size_t sp2 = line.find(' ', sp1 + 1);
    const std::string_view target = sp2 == std::string_view::npos ? line.substr(sp1 + 1) : line.substr(sp1 + 1, sp2 - sp1 - 1);
    const std::string_view route = target.substr(0, target.find('?'));

    if (route == "/health" && method == "GET") return {200, HealthJson()};
    if (route == "/metrics" && method == "GET") return {200, MetricsJson()};
    if (route == "/generate" && method == "POST") {
        if (slot < 0) return {503, R"({"error":"no engine is loaded"})"};
        GenerateRequest req;
        std::string err;
        if (!ParseGenerate(body, engines_[size_t(slot)]->Model().vocabSize, req, err))
            return {400, "{\"error\":" + JsonString(err) + "}"};
        return Generate(req, slot);
    }
    if (route == "/health" || route == "/metrics" || route == "/generate")
        return {405, R"({"error":"method not allowed"})"};
    return {404, R"({"error":"no such route"})"};
}

Response Server::Generate(const GenerateRequest &req, int slot) {
    engine::VoxelEngine &eng = *engines_[size_t(slot)];
    engine::GenerateResult r;
    const auto t0 = std::chrono::steady_clock::now();
    try {
        if (req.temperature > 0.0f) {
            // EngineOptions.temperature is declared by the reference but its Generate
            // ignores it; here it selects device-side sampling at that temperature.
            engine::SampleOptions so;
            so.temperature = req.temperature;
            so.seed = req.seed;
            so.maxNew = req.maxTokens;
            r.promptTokens = req.tokens;
            r.generated = engine::SampleGenerate(eng, {req.tokens}, so, nullptr).front();
        } else {
            engine::EngineOptions o = eng.Options();
            o.maxNewTokens = req.maxTokens;
            r = eng.Generate(req.tokens, o);
        }
    } catch (const std::exception &e) {
        // The reference answers a failed generation with 200 and an error field (:334-337).
        return {200, "{\"error\":" + JsonString(e.what()) + "}"};
    }
    const double total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    {
        std::lock_guard<std::mutex> lk(metricsMu_);
        last_ = eng.SnapshotMetrics();
        ++served_;
    }
    std::string j = "{\"tokens\":[";
    for (size_t i = 0; i < r.generated.size(); ++i) j += (i ? "," : "") + std::to_string(r.generated[i]);
    j += "],\"prompt_tokens\":" + std::to_string(r.promptTokens.size());
    j += ",\"generated_tokens\":" + std::to_string(r.generated.size());
    char perf[160];
    std::snprintf(perf, sizeof(perf), ",\"ms_per_token\":%.4f,\"total_ms\":%.4f,\"hit_stop\":%s,\"engine\":%d}",
                  r.msPerToken, total_ms, r.hitStop ? "true" : "false", slot);
    return {200, j + perf};
}

std::string Server::HealthJson() const {
    std::string j = "{\"status\":\"ok\",\"engines\":" + std::to_string(engines_.size());
    if (!engines_.empty()) {
        const graph::ModelConfig &c = engines_.front()->Model();
        j += ",\"architecture\":" + JsonString(c.architecture);
        j += ",\"layers\":" + std::to_string(c.numLayers);
        j += ",\"hidden_size\":" + std::to_string(c.hiddenSize);
        j += ",\"num_heads\":" + std::to_string(c.numHeads);
        j += ",\"num_kv_heads\":" + std::to_string(c.numKvHeads);
        j += ",\"head_dim\":" + std::to_string(c.HeadDim());
        j += ",\"vocab_size\":" + std::to_string(c.vocabSize);
        j += ",\"eos_token_id\":" + std::to_string(c.eosTokenId);
        j += ",\"weight_mib_per_engine\":" + std::to_string(engines_.front()->GraphModel().Plan().weightBytes >> 20);
    }
    return j + "}";
}

std::string Server::MetricsJson() {
    std::lock_guard<std::mutex> lk(metricsMu_);
    char buf[512];
    std::snprintf(buf, sizeof(buf),
                  "{\"kv_occupancy\":%.4f,\"tokens_per_sec\":%.3f,\"memory_pressure\":%.4f,"
                  "\"speculative_acceptance\":%.3f,\"requests_served\":%llu}",
                  double(last_.kvOccupancy), double(last_.tokensPerSec), double(last_.memoryPressure),
                  double(last_.speculativeAcceptance), static_cast<unsigned long long>(served_));
    return buf;
}

}  // namespace opure::server
