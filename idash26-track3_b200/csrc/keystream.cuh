// Key chunks (4 KiB-padded forward key regions with an integrity trailer) and
// the double-buffered host->HBM key stream (keystream.cu).
#pragma once
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "forward.cuh"

namespace ddg {

struct ChunkTrailer {
    char magic[8];
    uint32_t bw, scale, batch, pad;
    uint64_t index, key_bytes, checksum;
    uint64_t reserved[2];
};
static_assert(sizeof(ChunkTrailer) == 64, "chunk trailer is 64 bytes");

uint64_t key_chunk_bytes(int bw, int s, int B);
int key_checksum(const void *d, uint64_t bytes, uint64_t *out, cudaStream_t st);
int chunk_seal(void *d_chunk, int bw, int s, int B, uint64_t index, cudaStream_t st);
int chunk_verify(const void *d_chunk, int bw, int s, int B, ChunkTrailer *out, cudaStream_t st);
int check_trailer(const ChunkTrailer &t, int bw, int s, int B);

struct KeyStream {
    Party *P = nullptr;
    int B = 0, device = 0;
    uint64_t chunk = 0;
    void *d_slot[2] = {};
    cudaStream_t copy = nullptr;
    cudaEvent_t ev_h2d[2] = {}, ev_free[2] = {}, ev_c0[2] = {};
    std::vector<const void *> host;   // ring of pinned host chunks
    // key-file source
    int fd = -1, file_chunks = 0;
    std::string path;
    void *staging[2] = {};
    std::thread io;
    std::mutex mu;
    std::condition_variable cv;
    bool quit = false, io_error = false;
    int64_t staged_upto = -1;
    int64_t consumed[2] = {-1, -1};
    // progress
    uint64_t next = 0;
    int64_t issued = -1;
    bool verify = false;
    int timeout_ms = 600000;
    uint64_t consumed_chunks = 0;
    double bytes_copied = 0, copy_ms = 0, read_ms = 0, wait_ms = 0;

    ~KeyStream();
    int init(Party *p, int B);
    int open_file(const char *path, int nchunks);
    int begin_forward();
    int end_forward(int status);

  private:
    void io_loop();
    void stop_io();
    int source_of(uint64_t j, const void **src);
    int issue(uint64_t j);
};

}  // namespace ddg
