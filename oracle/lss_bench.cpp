// lss_bench.cpp -- times the reference's CPU LSS ReLU backend (TEST / BASELINE
// INFRASTRUCTURE ONLY; linked against the reference's own, unmodified
// gpu_mpc/lss/{lss_keygen,lss_online,lss_compare}.cpp by oracle/Makefile into
// oracle/_ref/lss_bench).  Used by bench.py's cpu_baseline leg and its
// --impl reference arm; the product never runs it.
//
// Follows the reference's own two-process harness (gpu_mpc/lss/lss_test.cpp:
// 392-437): the dealer writes both parties' key files with LssKeygen::gen_relu
// (lss_keygen.h: one Millionaires compare of bw-1 bits + MUX per element),
// then two forked party processes connect over loopback TCP
// (Channel::listen_and_accept / connect) and run LssParty::relu on random
// additive shares.  Each party prints its wall time; the driver prints one JSON
// line with the slower party's time.
//
//   lss_bench <n> <bw> <threads_per_party>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "lss_keygen.h"
#include "lss_online.h"

static int run_party(int party, int port, const char *dir, size_t n, int bw)
{
    lss::Channel chan = party == 0 ? lss::Channel::listen_and_accept(port) : lss::Channel::connect("127.0.0.1", port);
    lss::LssParty P(party, std::string(dir) + "/lss_keys_party" + std::to_string(party) + ".bin", chan, 7);
    std::mt19937_64 rng(1234 + party);
    const uint64_t mask = bw >= 64 ? ~0ULL : ((1ULL << bw) - 1);
    std::vector<uint64_t> x(n), y(n);
    for (auto &v : x) v = rng() & mask;
    std::vector<uint8_t> sync_in(1, 1), sync_out(1);
    P.open_bits(sync_in.data(), sync_out.data(), 1);  // both parties ready
    auto t0 = std::chrono::steady_clock::now();
    P.relu(x.data(), y.data(), n, bw);
    double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::string out = std::string(dir) + "/time" + std::to_string(party);
    FILE *f = fopen(out.c_str(), "w");
    if (!f) return 1;
    fprintf(f, "%.9f\n", sec);
    fclose(f);
    return 0;
}

int main(int argc, char **argv)
{
    if (argc >= 2 && strcmp(argv[1], "party") == 0) {
        return run_party(atoi(argv[2]), atoi(argv[3]), argv[4], strtoull(argv[5], nullptr, 10), atoi(argv[6]));
    }
    if (argc < 4) {
        fprintf(stderr, "usage: lss_bench <n> <bw> <threads_per_party>\n");
        return 2;
    }
    const size_t n = strtoull(argv[1], nullptr, 10);
    const int bw = atoi(argv[2]);
    const int threads = atoi(argv[3]);
    char dir[] = "/tmp/lss_bench_XXXXXX";
    if (!mkdtemp(dir)) return 1;
    auto tk = std::chrono::steady_clock::now();
    {
        lss::LssKeygen kg(0x5eed);
        kg.gen_relu(n, bw);
        kg.write_files(std::string(dir) + "/lss_keys_party0.bin", std::string(dir) + "/lss_keys_party1.bin");
    }
    double keygen_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - tk).count();
    setenv("DDG_LSS_THREADS", std::to_string(threads).c_str(), 1);
    const int port = 44200 + int(getpid() % 2000);
    pid_t kids[2];
    for (int p = 0; p < 2; p++) {
        kids[p] = fork();
        if (kids[p] == 0) {
            std::string ps = std::to_string(p), po = std::to_string(port), ns = std::to_string(n),
                        bs = std::to_string(bw);
            execl("/proc/self/exe", "lss_bench", "party", ps.c_str(), po.c_str(), dir, ns.c_str(), bs.c_str(),
                  (char *)nullptr);
            _exit(127);
        }
        if (p == 0) usleep(100000);
    }
    int rc = 0;
    for (int p = 0; p < 2; p++) {
        int st = 0;
        waitpid(kids[p], &st, 0);
        if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) rc = 1;
    }
    double t[2] = {0, 0};
    for (int p = 0; p < 2 && rc == 0; p++) {
        std::string path = std::string(dir) + "/time" + std::to_string(p);
        FILE *f = fopen(path.c_str(), "r");
        if (!f || fscanf(f, "%lf", &t[p]) != 1) rc = 1;
        if (f) fclose(f);
    }
    std::string cmd = std::string("rm -rf ") + dir;
    if (system(cmd.c_str()) != 0) rc = rc ? rc : 1;
    if (rc) {
        printf("{\"error\": \"party failed\"}\n");
        return rc;
    }
    double sec = t[0] > t[1] ? t[0] : t[1];
    printf("{\"n\": %zu, \"bw\": %d, \"threads_per_party\": %d, \"seconds\": %.6f, \"relu_per_s\": %.1f, "
           "\"keygen_s\": %.3f}\n",
           n, bw, threads, sec, double(n) / sec, keygen_s);
    return 0;
}
