// opure_server -- the HTTP front end (GET /health, POST /generate, GET /metrics) over
// libopure_engine: `opure_server --model <dir> [--port N] [--gpus 0,1,...]`, one engine
// per listed GPU (the reference's opure_server, src/app/Opure_Server.cpp:470-540, runs one
// engine on its one D3D12 device). Runs until SIGINT/SIGTERM.
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <unistd.h>

#include "opure_engine.h"

namespace {
volatile std::sig_atomic_t g_stop = 0;
void OnSignal(int) { g_stop = 1; }
}  // namespace

int main(int argc, char **argv) {
    std::string model;
    unsigned port = 8080;
    std::vector<int> gpus{0};
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a == "--model" && i + 1 < argc) {
            model = argv[++i];
        } else if (a == "--port" && i + 1 < argc) {
            port = unsigned(std::strtoul(argv[++i], nullptr, 10));
        } else if (a == "--gpus" && i + 1 < argc) {
            gpus.clear();
            for (const char *p = argv[++i]; *p;) {
                char *end = nullptr;
                gpus.push_back(int(std::strtol(p, &end, 10)));
                p = *end == ',' ? end + 1 : end;
                if (end == p && *p) break;
            }
        } else {
            std::printf("usage: opure_server --model <dir> [--port N] [--gpus 0,1,...]\n"
                        "routes: GET /health, POST /generate {\"tokens\":[...],\"max_tokens\":64}, GET /metrics\n");
            return a == "--help" || a == "-h" ? 0 : 2;
        }
    }
    if (model.empty() || port > 65535) {
        std::fprintf(stderr, "opure_server: --model <dir> is required (and --port must be < 65536)\n");
        return 2;
    }
    opure_server *srv = nullptr;
    const opure_status st =
        opure_server_start(model.c_str(), gpus.data(), uint32_t(gpus.size()), uint16_t(port), nullptr, &srv);
    if (st != OPURE_OK) {
        std::fprintf(stderr, "opure_server: %s: %s\n", opure_strerror(st), opure_engine_last_error(nullptr));
        return 1;
    }
    std::signal(SIGINT, OnSignal);
    std::signal(SIGTERM, OnSignal);
    std::printf("opure_server listening on http://127.0.0.1:%u with %zu engine(s)\n", unsigned(opure_server_port(srv)),
                gpus.size());
    std::fflush(stdout);
    while (!g_stop) ::pause();
    opure_server_stop(srv);
    return 0;
}
