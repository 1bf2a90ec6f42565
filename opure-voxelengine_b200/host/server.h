// server.h -- the HTTP front end re-attached to this engine: GET /health, POST /generate,
// GET /metrics (the reference's src/app/Opure_Server.cpp:10-13,280-339,376-437), with one
// engine per GPU so that requests run concurrently (the reference serves one request at a
// time on one device and notes that concurrency needs several engines, :21-25).
//
// Differences from the reference, each forced by this build's scope: there is no
// tokenizer, so /generate takes token ids ("tokens": [...]) and answers with token ids
// (a text "prompt" is refused with 400); sockets are POSIX; and a request that arrives
// while every engine is busy waits in a queue instead of in the listen backlog.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

#include "voxel_engine.h"

namespace opure::server {

constexpr size_t kMaxBodyBytes = size_t(1) << 20;  // the reference's cap (Opure_Server.cpp:95)
constexpr uint32_t kMaxNewTokens = 2048;           // max_tokens is clamped to [1, 2048] (:426-429)

// A parsed POST /generate body.
struct GenerateRequest {
    std::vector<uint32_t> tokens;
    uint32_t maxTokens = 64;   // the reference's default (:394)
    float temperature = 0.0f;  // <= 0: greedy Generate; > 0: sampled at this temperature
    uint64_t seed = 0;
};

// Parses a /generate body. On failure returns false with the client-facing message in err
// (the reference's wording where it has one). Validates every token against `vocab`
// (0: unchecked) and clamps max_tokens and temperature as the reference does.
bool ParseGenerate(std::string_view body, uint32_t vocab, GenerateRequest &out, std::string &err);

// One HTTP request: status and JSON body, from the raw bytes (header block + exactly
// Content-Length body bytes). Routing and method checks follow the reference (:366-437).
struct Response {
    int status = 200;
    std::string body;
};

std::string JsonString(std::string_view s);

class Server {
public:
    // engines: one per GPU, owned; may be empty (the routes still answer, /generate with
    // 503). Binds 127.0.0.1:port (0: any free port) and starts one worker per engine (one
    // when there are none) and an accept thread.
    Server(std::vector<std::unique_ptr<engine::VoxelEngine>> engines, uint16_t port);
    ~Server();
    Server(const Server &) = delete;
    Server &operator=(const Server &) = delete;

    uint16_t Port() const { return port_; }
    // Closes the listening socket, drains the queue and joins every thread.
    void Stop();
    // Handles one request on engine `slot` (or none: slot < 0).
    Response Handle(std::string_view raw, int slot);

private:
    void AcceptLoop();
    void Worker(int slot);
    std::string HealthJson() const;
    std::string MetricsJson();
    Response Generate(const GenerateRequest &req, int slot);

    std::vector<std::unique_ptr<engine::VoxelEngine>> engines_;
    int listenFd_ = -1;
    uint16_t port_ = 0;
    std::atomic<bool> stop_{false};
    std::thread acceptThread_;
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<int> queue_;        // accepted sockets waiting for a worker
    std::mutex metricsMu_;
    engine::VoxelEngine::MetricsSnapshot last_{};  // the last /generate's snapshot
    uint64_t served_ = 0;
};

}  // namespace opure::server
