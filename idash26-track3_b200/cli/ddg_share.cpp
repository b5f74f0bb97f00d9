// ddg_share: the data owner's side of the offline pipeline in C++ -- fixed-
// point quantisation of a batch of drug graphs and their additive sharing
// into the two evaluators' share files (restates reference/share_data.py:
// 39-79 _to_ring / split_shares and :135-159 share_drug_graph_raw_adj, and
// reference/protein_plaintext.py:19-31 for the public protein vectors).
//
//   ddg_share <bw> <scale> <seed> <in_dir> <out_dir>
//
// <in_dir> holds the plaintext batch as little-endian float64, sample-major,
// no header (the batch size B follows from the file sizes):
//   x.f64        (B, 138, 94)   node features
//   adj.f64      (B, 138, 138)  raw 0/1 adjacency with self-loops on real atoms
//   mask.f64     (B, 138)       node mask (1 for real atoms)
//   protein.f64  (B, 128)       protein vectors (public)
// <out_dir> receives the evaluators' inputs, little-endian <u4 (bw 32) or
// <u8 (bw 64): x_share{0,1}.dat and mask_share{0,1}.dat at `scale` (the mask
// tiled to (138, 376) per sample, share_data.py:120-124), adj_share{0,1}.dat
// at scale 0 (the raw adjacency; the evaluators normalise it securely), and
// protein_emb.dat, the protein vectors at `scale`, unshared.  Quantisation is
// rint(x * 2^scale) (round half to even) reduced modulo 2^bw.  Shares:
// share0 = a pad, share1 = value - pad (mod 2^bw); the pads come from a
// counter-mode SplitMix64 stream per tensor keyed by <seed> (like the
// reference's numpy generator, reproducible from the seed and not a
// cryptographic generator: a deployment passes a secret seed).
// Exit status 0, 1 on usage, 2 on I/O or shape errors.
#include <sys/stat.h>

#include <cfenv>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace {

constexpr int NMAX = 138, FEAT = 94, POOL = 376, PROT = 128;

uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// pad word i of tensor t: SplitMix64 of a counter keyed by (seed, t)
uint64_t pad(uint64_t seed, int t, uint64_t i) { return splitmix64(splitmix64(seed * 4 + uint64_t(t)) ^ splitmix64(i)); }

bool read_f64(const std::string &path, std::vector<double> &v)
{
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    if (n < 0 || n % 8) {
        std::fclose(f);
        return false;
    }
    v.resize(size_t(n) / 8);
    const bool ok = std::fread(v.data(), 8, v.size(), f) == v.size();
    std::fclose(f);
    return ok;
}

uint64_t to_ring(double x, int scale, int bw)
{
    const int64_t fixed = int64_t(std::nearbyint(std::ldexp(x, scale)));
    const uint64_t u = uint64_t(fixed);
    return bw == 32 ? (u & 0xFFFFFFFFull) : u;
}

bool write_words(const std::string &path, const std::vector<uint64_t> &w, int bw)
{
    FILE *f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    bool ok = true;
    if (bw == 32) {
        std::vector<uint32_t> n(w.size());
        for (size_t i = 0; i < w.size(); i++) n[i] = uint32_t(w[i]);
        ok = std::fwrite(n.data(), 4, n.size(), f) == n.size();
    } else {
        ok = std::fwrite(w.data(), 8, w.size(), f) == w.size();
    }
    return std::fclose(f) == 0 && ok;
}

// share a ring tensor: share0 = pad, share1 = value - pad
bool write_pair(const std::string &dir, const char *name, const std::vector<uint64_t> &v, uint64_t seed, int t,
                int bw)
{
    const uint64_t mask = bw == 32 ? 0xFFFFFFFFull : ~0ull;
    std::vector<uint64_t> s0(v.size()), s1(v.size());
    for (size_t i = 0; i < v.size(); i++) {
        s0[i] = pad(seed, t, i) & mask;
        s1[i] = (v[i] - s0[i]) & mask;
    }
    return write_words(dir + "/" + name + "_share0.dat", s0, bw) && write_words(dir + "/" + name + "_share1.dat", s1, bw);
}

}  // namespace

int main(int argc, char **argv)
{
    if (argc != 6) {
        std::fprintf(stderr, "usage: ddg_share <bw> <scale> <seed> <in_dir> <out_dir>\n");
        return 1;
    }
    const int bw = std::atoi(argv[1]), scale = std::atoi(argv[2]);
    const uint64_t seed = std::strtoull(argv[3], nullptr, 10);
    const std::string in = argv[4], out = argv[5];
    if ((bw != 32 && bw != 64) || scale < 0 || scale >= bw - 1) {
        std::fprintf(stderr, "ddg_share: bw must be 32 or 64 and scale in [0, bw-1)\n");
        return 1;
    }
    std::fesetround(FE_TONEAREST);
    std::vector<double> x, adj, mask, prot;
    for (auto &p : {std::make_pair("x.f64", &x), std::make_pair("adj.f64", &adj), std::make_pair("mask.f64", &mask),
                    std::make_pair("protein.f64", &prot)}) {
        if (!read_f64(in + "/" + p.first, *p.second)) {
            std::fprintf(stderr, "ddg_share: cannot read %s/%s\n", in.c_str(), p.first);
            return 2;
        }
    }
    const size_t B = mask.size() / NMAX;
    if (B == 0 || mask.size() != B * NMAX || x.size() != B * NMAX * FEAT || adj.size() != B * NMAX * NMAX ||
        prot.size() != B * PROT) {
        std::fprintf(stderr, "ddg_share: inconsistent shapes (x %zu, adj %zu, mask %zu, protein %zu values)\n",
                     x.size(), adj.size(), mask.size(), prot.size());
        return 2;
    }
    mkdir(out.c_str(), 0755);
    std::vector<uint64_t> rx(x.size()), ra(adj.size()), rm(B * NMAX * POOL), rp(prot.size());
    for (size_t i = 0; i < x.size(); i++) rx[i] = to_ring(x[i], scale, bw);
    for (size_t i = 0; i < adj.size(); i++) ra[i] = to_ring(adj[i], 0, bw);
    for (size_t r = 0; r < B * NMAX; r++) {
        const uint64_t v = to_ring(mask[r], scale, bw);
        for (int c = 0; c < POOL; c++) rm[r * POOL + c] = v;
    }
    for (size_t i = 0; i < prot.size(); i++) rp[i] = to_ring(prot[i], scale, bw);
    // distinct pad streams per tensor (x 0, adj 1, mask 2), as the reference's sub-seeds seed + 0/1/2
    if (!write_pair(out, "x", rx, seed, 0, bw) || !write_pair(out, "adj", ra, seed, 1, bw) ||
        !write_pair(out, "mask", rm, seed, 2, bw) || !write_words(out + "/protein_emb.dat", rp, bw)) {
        std::fprintf(stderr, "ddg_share: cannot write the share files under %s\n", out.c_str());
        return 2;
    }
    std::printf("{\"batch\": %zu, \"bw\": %d, \"scale\": %d, \"nmax\": %d, \"pool_dim\": %d, \"adj_scale\": 0}\n", B,
                bw, scale, NMAX, POOL);
    return 0;
}
