// CPU check of the word-parallel AND-tree levels of the truth-table gates
// (idash26-track3_b200/csrc/tt_lanes.cuh), compiled as plain host C++ by
// tests/test_tt_lanes_cpu.py.
//
// For every plan compiled into the level kernel (bw 32 and 64 at scale 12;
// split ReLU, truncation carry and full-compare modes) and both parties, it
// plays the whole AND tree on random inputs: secret-shared digit bits as the
// level-1 table read leaves them, dealer triples (c = a b, c' = a b') with zero
// output masks, tt_open for each level, the XOR of both parties' openings, and
// tt_close.  The reconstructed part roots (and the cross combine) must equal
// the plaintext radix comparison folded over the same plan.
#include <cstdio>
#include <cstdlib>
#include <random>

#include "tt_lanes.cuh"

using namespace ddg;

namespace {

std::mt19937_64 rng(12345);
uint32_t rbit() { return uint32_t(rng() & 1u); }

struct Outcome {
    uint32_t hl, he, ll;
};

// plaintext fold of the digit bits over the plan's tree (node (2i+1, 2i) -> i,
// odd top node passes up), per part; the full-compare cross combine on top
template <int MODE, int NB>
Outcome plain(const uint32_t *lt, const uint32_t *eq)
{
    constexpr OtPlan P = digit_plan(NB, 12, MODE);
    uint32_t root_lt[2] = {0, 0}, root_eq[2] = {0, 0};
    for (int p = 0; p < 2; p++) {
        int k = P.nd[p];
        if (k == 0) continue;
        uint32_t l[OT_MAX_DIGITS], e[OT_MAX_DIGITS];
        for (int j = 0; j < k; j++) l[j] = lt[P.base[p] + j], e[j] = eq[P.base[p] + j];
        while (k > 1) {
            const int nk = (k + 1) / 2;
            for (int i = 0; i < k / 2; i++) {
                const uint32_t nl = l[2 * i + 1] ^ (e[2 * i + 1] & l[2 * i]), ne = e[2 * i + 1] & e[2 * i];
                l[i] = nl, e[i] = ne;
            }
            if (k & 1) l[k / 2] = l[k - 1], e[k / 2] = e[k - 1];
            k = nk;
        }
        root_lt[p] = l[0], root_eq[p] = e[0];
    }
    Outcome o{root_lt[0], root_eq[0], root_lt[1]};
    if (MODE == PLAN_TT_FULL) o.hl = root_lt[0] ^ (root_eq[0] & root_lt[1]);
    return o;
}

template <int MODE, int NB, int L>
void step(uint32_t (&st)[2], const uint32_t (&tw)[2][3], uint32_t (&w)[2])
{
    // close level L - 1 with both parties' openings, then open level L
    const uint32_t O = w[0] ^ w[1];
    st[0] = tt_close<MODE, NB, 12, 0, L>(st[0], tw[0], O);
    st[1] = tt_close<MODE, NB, 12, 1, L>(st[1], tw[1], O);
    constexpr OtPlan P = digit_plan(NB, 12, MODE);
    if constexpr (L <= P.levels) {
        w[0] = tt_open<MODE, NB, 12, L>(st[0], tw[0]);
        w[1] = tt_open<MODE, NB, 12, L>(st[1], tw[1]);
    }
}

template <int MODE, int NB>
int check(int trials)
{
    constexpr OtPlan P = digit_plan(NB, 12, MODE);
    static_assert(P.ok && P.state_bytes() == 4, "plan compiled into the level kernel");
    int bad = 0;
    for (int t = 0; t < trials; t++) {
        uint32_t lt[OT_MAX_DIGITS] = {}, eq[OT_MAX_DIGITS] = {};
        uint32_t st[2] = {0, 0};
        for (int g = 0; g < P.D; g++) {
            // eq of a digit whose table has no eq rows is never used: leave it 0
            lt[g] = rbit(), eq[g] = P.deq(g) ? rbit() : 0u;
            // bias towards equal digits so that the lower digits matter
            if (P.deq(g) && (rng() % 4) != 0) eq[g] = 1u, lt[g] = 0u;
            const uint32_t s0 = uint32_t(rng() & 3u);
            const uint32_t v = lt[g] | (eq[g] << 1);
            st[0] |= s0 << (2 * g);
            st[1] |= (s0 ^ v) << (2 * g);
        }
        uint32_t tw[2][3] = {{0, 0, 0}, {0, 0, 0}};
        for (int q = 0; q < P.ncomb; q++) {
            const uint32_t a = rbit(), b = rbit(), b2 = rbit();
            const uint32_t v = a | (b << 1) | (b2 << 2) | ((a & b) << 3) | ((a & b2) << 4);
            const uint32_t s0 = uint32_t(rng() & 31u), s1 = s0 ^ v;
            // at the plan's triple-bit positions (grouped by level where the plan packs them)
            for (int k = 0; k < 5; k++) {
                if (!P.comb[q].eq && (k == 2 || k == 4)) continue;  // no b', c' without an eq AND
                const int bit = P.tpos(q, k);
                tw[0][bit / 32] |= ((s0 >> k) & 1u) << (bit % 32);
                tw[1][bit / 32] |= ((s1 >> k) & 1u) << (bit % 32);
            }
        }
        uint32_t w[2] = {tt_open<MODE, NB, 12, 1>(st[0], tw[0]), tt_open<MODE, NB, 12, 1>(st[1], tw[1])};
        step<MODE, NB, 2>(st, tw, w);
        if constexpr (P.levels >= 2) step<MODE, NB, 3>(st, tw, w);
        if constexpr (P.levels >= 3) step<MODE, NB, 4>(st, tw, w);
        if constexpr (P.levels >= 4) step<MODE, NB, 5>(st, tw, w);
        if constexpr (P.levels >= 5) step<MODE, NB, 6>(st, tw, w);
        const uint32_t s = st[0] ^ st[1];
        const Outcome want = plain<MODE, NB>(lt, eq);
        const uint32_t hl = s & 1u, he = (s >> 1) & 1u, ll = (s >> (2 * P.base[1])) & 1u;
        bool ok = ll == want.ll;
        if (P.nd[0]) ok = ok && hl == want.hl && (MODE == PLAN_TT_FULL || he == want.he);
        if (!ok && bad++ < 5)
            std::printf("mode %d bw %d trial %d: got (%u %u %u) want (%u %u %u)\n", MODE, NB, t, hl, he, ll, want.hl,
                        want.he, want.ll);
    }
    std::printf("mode %d bw %d levels %d combines %d: %d of %d wrong\n", MODE, NB, P.levels, P.ncomb, bad, trials);
    // the plan's triple-bit positions: distinct, inside the triple words
    uint32_t seen[3] = {0u, 0u, 0u};
    const int nbits = 5 * P.ncomb + (MODE == PLAN_TT_FULL ? 1 : 0);
    for (int i = 0; i < nbits; i++) {
        if (i < 5 * P.ncomb && !P.comb[i / 5].eq && (i % 5 == 2 || i % 5 == 4)) continue;
        const int pos = i < 5 * P.ncomb ? P.tpos(i / 5, i % 5) : P.mu_bit();
        if (pos < 0 || pos >= 32 * P.tri_words() || ((seen[pos / 32] >> (pos % 32)) & 1u)) {
            std::printf("mode %d bw %d: triple bit %d at %d collides or overflows\n", MODE, NB, i, pos);
            bad++;
        } else {
            seen[pos / 32] |= 1u << (pos % 32);
        }
    }
    std::printf("positions mode %d bw %d packed %d:", MODE, NB, int(P.tpacked));
    for (int q = 0; q < P.ncomb; q++) std::printf(" %d %d", P.tpa[q], P.tpc[q]);
    std::printf(" %d\n", P.mu_bit());
    return bad;
}

// every truth-table plan (modes, both ring widths, every scale): the triple-bit
// positions distinct and inside the triple words, printed for the oracle check
int check_positions_all_scales()
{
    int bad = 0;
    for (int mode : {int(PLAN_TT_RELU), int(PLAN_TT_LRS), int(PLAN_TT_FULL)})
        for (int nb : {32, 64})
            for (int sc = 1; sc < nb - 1; sc++) {
                const OtPlan P = digit_plan(nb, sc, mode);
                std::printf("allpos %d %d %d %d %d:", mode, nb, sc, int(P.ok), int(P.tpacked));
                if (!P.ok) {
                    std::printf("\n");
                    continue;
                }
                uint32_t seen[3] = {0u, 0u, 0u};
                for (int q = 0; q < P.ncomb; q++)
                    for (int k = 0; k < 5; k++) {
                        if (!P.comb[q].eq && (k == 2 || k == 4)) continue;
                        const int pos = P.tpos(q, k);
                        if (pos < 0 || pos >= 32 * P.tri_words() || ((seen[pos / 32] >> (pos % 32)) & 1u)) bad++;
                        else seen[pos / 32] |= 1u << (pos % 32);
                    }
                if (mode == PLAN_TT_FULL) {
                    const int pos = P.mu_bit();
                    if (pos < 0 || pos >= 32 * P.tri_words() || ((seen[pos / 32] >> (pos % 32)) & 1u)) bad++;
                }
                for (int q = 0; q < P.ncomb; q++) std::printf(" %d %d", P.tpa[q], P.tpc[q]);
                std::printf(" %d\n", P.mu_bit());
            }
    if (bad) std::printf("all-scale positions: %d collide or overflow\n", bad);
    return bad;
}

}  // namespace

int main(int argc, char **argv)
{
    const int trials = argc > 1 ? std::atoi(argv[1]) : 20000;
    int bad = check_positions_all_scales();
    bad += check<PLAN_TT_RELU, 32>(trials);
    bad += check<PLAN_TT_RELU, 64>(trials);
    bad += check<PLAN_TT_LRS, 32>(trials);
    bad += check<PLAN_TT_LRS, 64>(trials);
    bad += check<PLAN_TT_FULL, 32>(trials);
    bad += check<PLAN_TT_FULL, 64>(trials);
    std::printf(bad ? "FAIL\n" : "ok\n");
    return bad ? 1 : 0;
}
