// ddg_inference: command-line drop-in for the reference's driver binary
// (gpu_mpc/deepdtagen_inference.cu, argv parsed at :186-200), built on the C ABI
// of libddg.so only (include/ddg_fss.h).
//
//   ddg_inference <bw> <scale> <role> <party> <keydir> <sampledir> <B> [peer_ip]
//
// role 0 (dealer, offline): generates the key chunks of party <party> (2 = both
//   parties) for NC = ceil(N / B) micro-batches of B samples and writes them to
//   <keydir>/DeepDTAGen_<bw>_<scale>_party<p>_inference_key<p>.dat, chunk k at
//   k * ddg_key_chunk_bytes (the reference's file name and chunk placement,
//   deepdtagen_inference.cu:280-281, 383-398), plus <keydir>/meta.json
//   {B, NC, N, bw, scale} as run_party.sh:73-74 writes it.  The masks come from
//   the dealer seed (DDG_SEED, default 1) and the chunk index, so the dealer
//   runs of the two parties produce matching keys.
// role 1 (evaluator, online): party 0 or 1 in its own process, one GPU each
//   (DDG_DEVICE, default = party); the two processes meet over TCP (party 1
//   listens on DDG_PEER_PORT, default 29650; party 0 connects to [peer_ip],
//   default 127.0.0.1) only to hand over the NCCL unique id, after which the
//   openings run over NCCL (NVLink on one box, sockets or InfiniBand across
//   hosts).  Party 2 runs both parties in this process on one GPU.  Keys are
//   streamed chunk by chunk from the key file through the double-buffered key
//   stream (verified on the GPU); shares are read per chunk from
//   <sampledir>/{x,adj,mask}_share<p>.dat and protein_emb.dat.  Party 0 (or
//   the process of party 2) prints AFFINITY[i]=%.6f for every sample
//   (deepdtagen_inference.cu:594-606; AFFINITY= when N == 1).
//
// Environment: DDG_WEIGHTS_BIN (default <sampledir>/weights.bin), DDG_NUM_CHUNKS
// (default ceil(N / B)), DDG_SEED, DDG_DEVICE, DDG_PEER_PORT, DDG_RELU_SPLIT
// (2 or 3) and DDG_RELU_BACKEND (tt, the default, ot or dcf); both must
// match between dealer and evaluators.
// Exit status 0 on success, 1 on usage errors, 2 on library or I/O errors.
#include <arpa/inet.h>
#include <fcntl.h>
#include <netinet/in.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "ddg_fss.h"

namespace {

constexpr int NMAX = 138, FEAT = 94, POOL = 376, PROT = 128;

[[noreturn]] void die(int code, const char *fmt, const char *a = "", const char *b = "")
{
    std::fprintf(stderr, "ddg_inference: ");
    std::fprintf(stderr, fmt, a, b);
    std::fprintf(stderr, "\n");
    std::exit(code);
}

void check(int st, const char *what)
{
    if (st != DDG_OK) die(2, "%s: %s", what, ddg_last_error());
}

void check_cuda(cudaError_t e, const char *what)
{
    if (e != cudaSuccess) die(2, "%s: %s", what, cudaGetErrorString(e));
}

long env_long(const char *name, long dflt)
{
    const char *v = std::getenv(name);
    return v && *v ? std::strtol(v, nullptr, 10) : dflt;
}

// DDG_RELU_BACKEND: tt (default), ot or dcf
int relu_backend_env()
{
    const char *v = std::getenv("DDG_RELU_BACKEND");
    if (!v || !*v || std::strcmp(v, "tt") == 0) return DDG_RELU_TT;
    if (std::strcmp(v, "ot") == 0) return DDG_RELU_OT;
    if (std::strcmp(v, "dcf") == 0) return DDG_RELU_DCF;
    die(1, "DDG_RELU_BACKEND must be tt, ot or dcf");
    return DDG_RELU_TT;
}

std::string env_str(const char *name, const std::string &dflt)
{
    const char *v = std::getenv(name);
    return v && *v ? std::string(v) : dflt;
}

uint64_t file_size(const std::string &path)
{
    struct stat st;
    if (::stat(path.c_str(), &st) != 0) die(2, "cannot stat %s", path.c_str());
    return uint64_t(st.st_size);
}

std::vector<int64_t> read_weights(const std::string &path)
{
    const uint64_t bytes = file_size(path);
    if (bytes % 8) die(2, "%s: size is not a multiple of 8", path.c_str());
    std::vector<int64_t> w(bytes / 8);
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f || std::fread(w.data(), 8, w.size(), f) != w.size()) die(2, "cannot read %s", path.c_str());
    std::fclose(f);
    return w;
}

std::string key_file(const std::string &keydir, int bw, int scale, int p)
{
    return keydir + "/DeepDTAGen_" + std::to_string(bw) + "_" + std::to_string(scale) + "_party" + std::to_string(p) +
           "_inference_key" + std::to_string(p) + ".dat";
}

// Rows [first, first + count) of a share file of `row_bytes` per sample into the
// pinned buffer `dst` of `cap` samples; rows past the end of the file are zero.
void read_rows(int fd, const char *name, uint64_t row_bytes, uint64_t first, uint64_t count, uint64_t cap,
               uint8_t *dst)
{
    std::memset(dst, 0, cap * row_bytes);
    uint64_t want = count * row_bytes, off = first * row_bytes, got = 0;
    while (got < want) {
        ssize_t r = ::pread(fd, dst + got, want - got, off + got);
        if (r < 0) die(2, "read error on %s", name);
        if (r == 0) break;
        got += uint64_t(r);
    }
    if (got != want) die(2, "%s is shorter than the sample count", name);
}

// ---------------------------------------------------------------- TCP rendezvous

int tcp_listen_accept(int port)
{
    int s = ::socket(AF_INET, SOCK_STREAM, 0);
    int one = 1;
    ::setsockopt(s, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons(uint16_t(port));
    a.sin_addr.s_addr = htonl(INADDR_ANY);
    if (::bind(s, reinterpret_cast<sockaddr *>(&a), sizeof(a)) != 0) die(2, "cannot bind the peer port");
    if (::listen(s, 1) != 0) die(2, "listen failed");
    int c = ::accept(s, nullptr, nullptr);
    ::close(s);
    if (c < 0) die(2, "accept failed");
    return c;
}

int tcp_connect(const std::string &ip, int port, int timeout_s)
{
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons(uint16_t(port));
    if (::inet_pton(AF_INET, ip.c_str(), &a.sin_addr) != 1) die(1, "bad peer address %s", ip.c_str());
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        int s = ::socket(AF_INET, SOCK_STREAM, 0);
        if (::connect(s, reinterpret_cast<sockaddr *>(&a), sizeof(a)) == 0) return s;
        ::close(s);
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(timeout_s))
            die(2, "cannot reach the peer at %s", ip.c_str());
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
    }
}

void xfer(int s, void *buf, size_t n, bool send)
{
    auto *p = static_cast<uint8_t *>(buf);
    size_t done = 0;
    while (done < n) {
        ssize_t r = send ? ::send(s, p + done, n - done, 0) : ::recv(s, p + done, n - done, 0);
        if (r <= 0) die(2, "peer connection lost during the rendezvous");
        done += size_t(r);
    }
}

// ---------------------------------------------------------------- roles

struct Args {
    int bw = 32, scale = 12, role = 1, party = 0, B = 0;
    std::string keydir, sampledir, peer = "127.0.0.1";
};

uint64_t sample_count(const Args &a)
{
    const uint64_t row = uint64_t(NMAX) * FEAT * (a.bw / 8);
    for (int p : {0, 1}) {
        const std::string f = a.sampledir + "/x_share" + std::to_string(p) + ".dat";
        struct stat st;
        if (::stat(f.c_str(), &st) == 0) return uint64_t(st.st_size) / row;
    }
    die(2, "no x_share0.dat / x_share1.dat in %s", a.sampledir.c_str());
}

int dealer(const Args &a)
{
    const std::vector<int64_t> w = read_weights(env_str("DDG_WEIGHTS_BIN", a.sampledir + "/weights.bin"));
    const uint64_t N = sample_count(a);
    const long NC = env_long("DDG_NUM_CHUNKS", long((N + a.B - 1) / a.B));
    const uint64_t seed = uint64_t(env_long("DDG_SEED", 1));
    const int device = int(env_long("DDG_DEVICE", 0));
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    const uint64_t kb = ddg_forward_key_bytes(a.bw, a.scale, a.B);
    const uint64_t cb = ddg_key_chunk_bytes(a.bw, a.scale, a.B);
    if (!kb || !cb) die(2, "bad key layout: %s", ddg_last_error());
    void *d0 = nullptr, *d1 = nullptr, *h = nullptr;
    check_cuda(cudaMalloc(&d0, cb), "cudaMalloc");
    check_cuda(cudaMalloc(&d1, cb), "cudaMalloc");
    check_cuda(cudaMallocHost(&h, cb), "cudaMallocHost");
    int fds[2] = {-1, -1};
    for (int p : {0, 1})
        if (a.party == p || a.party == 2) {
            fds[p] = ::open(key_file(a.keydir, a.bw, a.scale, p).c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
            if (fds[p] < 0) die(2, "cannot create %s", key_file(a.keydir, a.bw, a.scale, p).c_str());
        }
    const auto t0 = std::chrono::steady_clock::now();
    for (long ck = 0; ck < NC; ck++) {
        // both parties' keys of micro-batch ck (the key region starts each chunk)
        check(ddg_dealer_forward(a.bw, a.scale, a.B, seed * 1000003ull + uint64_t(ck), w.data(), w.size(), device, d0,
                                 d1, nullptr),
              "dealer");
        for (int p : {0, 1}) {
            if (fds[p] < 0) continue;
            void *d = p == 0 ? d0 : d1;
            check(ddg_key_chunk_seal(d, a.bw, a.scale, a.B, uint64_t(ck), nullptr), "seal");
            check_cuda(cudaMemcpy(h, d, cb, cudaMemcpyDeviceToHost), "copy keys");
            if (::pwrite(fds[p], h, cb, off_t(uint64_t(ck) * cb)) != ssize_t(cb)) die(2, "key file write failed");
        }
    }
    for (int fd : fds)
        if (fd >= 0) ::close(fd);
    const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    FILE *m = std::fopen((a.keydir + "/meta.json").c_str(), "w");
    if (m) {
        const char *names[3] = {"dcf", "ot", "tt"};
        const char *be = names[relu_backend_env()];
        std::fprintf(m,
                     "{\n  \"B\": %d,\n  \"NC\": %ld,\n  \"N\": %llu,\n  \"bw\": %d,\n  \"scale\": %d,\n"
                     "  \"relu_backend\": \"%s\"\n}\n",
                     a.B, NC, (unsigned long long)N, a.bw, a.scale, be);
        std::fclose(m);
    }
    std::fprintf(stderr, "dealer: %ld chunk(s) of B=%d, %.1f MB per chunk and party, %.2f s\n", NC, a.B, cb / 1e6, s);
    cudaFree(d0), cudaFree(d1), cudaFreeHost(h);
    return 0;
}

struct ShareFiles {
    int x = -1, adj = -1, mask = -1, prot = -1;
};

ShareFiles open_shares(const Args &a, int p)
{
    ShareFiles f;
    auto op = [&](const std::string &name) {
        int fd = ::open((a.sampledir + "/" + name).c_str(), O_RDONLY);
        if (fd < 0) die(2, "cannot open %s/%s", a.sampledir.c_str(), name.c_str());
        return fd;
    };
    const std::string s = std::to_string(p);
    f.x = op("x_share" + s + ".dat"), f.adj = op("adj_share" + s + ".dat"), f.mask = op("mask_share" + s + ".dat");
    if (p == 1) f.prot = op("protein_emb.dat");  // public, held by party 1; party 0 enters zeros
    return f;
}

struct Staging {
    uint8_t *buf[4] = {};
    uint64_t row[4] = {};
};

Staging make_staging(int bw, int B)
{
    Staging s;
    const uint64_t e = uint64_t(bw / 8);
    const uint64_t rows[4] = {uint64_t(NMAX) * FEAT * e, uint64_t(NMAX) * NMAX * e, uint64_t(NMAX) * POOL * e,
                              uint64_t(PROT) * e};
    for (int i = 0; i < 4; i++) {
        s.row[i] = rows[i];
        check_cuda(cudaMallocHost(reinterpret_cast<void **>(&s.buf[i]), rows[i] * uint64_t(B)), "cudaMallocHost");
        std::memset(s.buf[i], 0, rows[i] * uint64_t(B));
    }
    return s;
}

void load_chunk(const ShareFiles &f, Staging &s, uint64_t first, uint64_t count, int B)
{
    read_rows(f.x, "x share", s.row[0], first, count, uint64_t(B), s.buf[0]);
    read_rows(f.adj, "adj share", s.row[1], first, count, uint64_t(B), s.buf[1]);
    read_rows(f.mask, "mask share", s.row[2], first, count, uint64_t(B), s.buf[2]);
    if (f.prot >= 0) read_rows(f.prot, "protein_emb.dat", s.row[3], first, count, uint64_t(B), s.buf[3]);
}

void print_affinities(const std::vector<double> &aff, uint64_t first, uint64_t count, uint64_t N)
{
    for (uint64_t i = 0; i < count; i++) {
        if (N == 1)
            std::printf("AFFINITY=%.6f\n", aff[i]);
        else
            std::printf("AFFINITY[%llu]=%.6f\n", (unsigned long long)(first + i), aff[i]);
    }
}

int evaluate(const Args &a)
{
    const std::vector<int64_t> w = read_weights(env_str("DDG_WEIGHTS_BIN", a.sampledir + "/weights.bin"));
    const uint64_t N = sample_count(a);
    const long NC = env_long("DDG_NUM_CHUNKS", long((N + a.B - 1) / a.B));
    if (uint64_t(NC) * uint64_t(a.B) < N) die(1, "DDG_NUM_CHUNKS x B is smaller than the sample count");
    const bool both = a.party == 2;
    const int device = int(env_long("DDG_DEVICE", both ? 0 : a.party));
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    const int nparty = both ? 2 : 1;
    ddg_party *P[2] = {};
    ddg_keystream *K[2] = {};
    ShareFiles F[2];
    Staging S[2];
    for (int i = 0; i < nparty; i++) {
        const int p = both ? i : a.party;
        check(ddg_party_create(&P[i], p, a.bw, a.scale, device), "party");
        check(ddg_party_set_weights(P[i], w.data(), w.size()), "weights");
        check(ddg_keystream_create(&K[i], P[i], a.B), "key stream");
        check(ddg_keystream_open_file(K[i], key_file(a.keydir, a.bw, a.scale, p).c_str(), int(NC)), "key file");
        check(ddg_keystream_set_verify(K[i], 1), "key verification");
        F[i] = open_shares(a, p);
        S[i] = make_staging(a.bw, a.B);
    }
    if (both) {
        check(ddg_pair_local(P[0], P[1]), "local pair");
    } else {
        // hand over the NCCL unique id: party 1 listens and creates it, party 0 connects
        const int port = int(env_long("DDG_PEER_PORT", 29650));
        uint8_t id[128];
        if (a.party == 1) {
            check(ddg_nccl_unique_id(id), "nccl id");
            int s = tcp_listen_accept(port);
            xfer(s, id, sizeof(id), true);
            ::close(s);
        } else {
            int s = tcp_connect(a.peer, port, int(env_long("DDG_PEER_TIMEOUT_S", 120)));
            xfer(s, id, sizeof(id), false);
            ::close(s);
        }
        check(ddg_party_connect_nccl(P[0], id, 2, a.party, 1 - a.party), "nccl connect");
    }
    std::vector<int64_t> raw(size_t(a.B));
    std::vector<double> aff(size_t(a.B));
    double total_ms = 0;
    for (long ck = 0; ck < NC; ck++) {
        const uint64_t first = uint64_t(ck) * uint64_t(a.B);
        const uint64_t count = first >= N ? 0 : (N - first < uint64_t(a.B) ? N - first : uint64_t(a.B));
        for (int i = 0; i < nparty; i++) load_chunk(F[i], S[i], first, count, a.B);
        const auto t0 = std::chrono::steady_clock::now();
        if (both) {
            const void *in0[4] = {S[0].buf[0], S[0].buf[1], S[0].buf[2], S[0].buf[3]};
            const void *in1[4] = {S[1].buf[0], S[1].buf[1], S[1].buf[2], S[1].buf[3]};
            check(ddg_forward_eval_pair_streamed(K[0], K[1], a.B, in0, in1, 1, raw.data(), aff.data()), "forward");
        } else {
            check(ddg_forward_eval_streamed(K[0], a.B, S[0].buf[0], S[0].buf[1], S[0].buf[2], S[0].buf[3], 1,
                                            raw.data(), aff.data()),
                  "forward");
        }
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        total_ms += ms;
        if (both || a.party == 0) print_affinities(aff, first, count, N);
        std::fprintf(stderr, "chunk %ld: %llu samples, %.2f ms\n", ck, (unsigned long long)count, ms);
    }
    std::fflush(stdout);
    std::fprintf(stderr, "online: %llu samples in %.2f ms (%.1f samples/s)\n", (unsigned long long)N, total_ms,
                 total_ms > 0 ? N / (total_ms / 1e3) : 0.0);
    for (int i = 0; i < nparty; i++) {
        ddg_keystream_destroy(K[i]);
        ddg_party_destroy(P[i]);
        for (uint8_t *b : S[i].buf) cudaFreeHost(b);
    }
    return 0;
}

}  // namespace

int main(int argc, char **argv)
{
    if (argc < 8 || argc > 9) {
        std::fprintf(stderr, "usage: %s <bw> <scale> <role 0=dealer|1=eval> <party 0|1|2> <keydir> <sampledir> <B> "
                             "[peer_ip]\n",
                     argv[0]);
        return 1;
    }
    Args a;
    a.bw = std::atoi(argv[1]), a.scale = std::atoi(argv[2]), a.role = std::atoi(argv[3]), a.party = std::atoi(argv[4]);
    a.keydir = argv[5], a.sampledir = argv[6], a.B = std::atoi(argv[7]);
    if (argc == 9) a.peer = argv[8];
    if ((a.bw != 32 && a.bw != 64) || a.B <= 0 || (a.role != 0 && a.role != 1) || a.party < 0 || a.party > 2)
        die(1, "bad arguments (bw 32|64, role 0|1, party 0|1|2, B > 0)");
    const long split = env_long("DDG_RELU_SPLIT", 3);
    check(ddg_relu_split(int(split)), "DDG_RELU_SPLIT");
    check(ddg_relu_backend(relu_backend_env()), "DDG_RELU_BACKEND");
    ::mkdir(a.keydir.c_str(), 0755);
    return a.role == 0 ? dealer(a) : evaluate(a);
}
