// Gate launchers (gates.cu).
#pragma once
#include "common.cuh"

namespace ddg {

int device_sms();
int gate_keygen(const GateLayout &L, uint64_t seed, uint32_t op, const void *rin, void *rout, void *k0, void *k1,
                cudaStream_t st);
int gate_round1(const GateLayout &L, const void *xhat, const void *key, uint32_t *bits_hi, uint32_t *bits_lo,
                cudaStream_t st);
// xhat2: a second addend of the opened input (an opening still held as both
// parties' shares), or null
int gate_round2(const GateLayout &L, int party, const void *xhat, const uint32_t *hi_own, const uint32_t *hi_peer,
                const uint32_t *lo_own, const uint32_t *lo_peer, const void *key, void *share, cudaStream_t st,
                const void *xhat2 = nullptr);

int aes_chain(uint64_t threads, int iters, uint32_t *out, cudaStream_t st, int variant = 0);

}  // namespace ddg
