"""include/ddg_backend.hpp, the Backend<T>-shaped C++ adapter over the C ABI,
compiles with a plain C++17 compiler, links against libddg.so and reports a
bad construction as a status code (no GPU needed: a wrong-size weights blob
fails before any device work, and without a device the party creation fails)."""
import os
import subprocess

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <cstdio>
#include <vector>
#include "ddg_backend.hpp"

struct Loopback : ddg_ref::Transport {
    int exchange(int, const void *, void *, uint64_t, void *) override { return 0; }
};

int main()
{
    std::vector<int64_t> tiny(3, 0);  // not a weights.bin blob
    ddg_ref::Backend be(0, 32, 12, 0, tiny.data(), tiny.size(), nullptr, 0);
    ddg_wire a{}, b{}, c{};
    Loopback lb;
    int64_t raw[1];
    double aff[1];
    // every call is well-formed C++ against the C ABI; none is run on a failed object
    if (be.status() == DDG_OK) {
        be.connect(&lb);
        be.secureAdjNormEval(1, nullptr, a);
        be.input(nullptr, 1, b);
        be.gcnLayerForward(0, 1, b, a, c);
        be.matmul(1, 94, a, b, c);
        be.matmul(c, 3, 1, b);
        be.fc_relu(c, 3, 1, b);
        be.mul(a, b, c);
        be.relu(a, b);
        be.truncateForward(a, b, true);
        be.maskedMaxPool(1, a, b);
        be.concatProtein(1, a, nullptr, b);
        be.output(1, a, raw, aff);
    }
    std::printf("%d %llu\n", be.status(), (unsigned long long)be.keyBuf.offset);
    return be.status() == DDG_OK ? 1 : 0;
}
"""


def test_backend_adapter_compiles_links_and_reports_status(tmp_path, ddg):
    src = tmp_path / "adapter.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "adapter"
    libdir = os.path.dirname(ddg.LIB_PATH)
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-I" + os.path.join(REPO, "include"),
                        str(src), "-o", str(exe), "-L" + libdir, "-lddg", "-Wl,-rpath," + libdir],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    status, offset = r.stdout.split()
    assert int(status) in (1, 2) and int(offset) == 0  # DDG_ERR_ARG (weights) or DDG_ERR_CUDA (no device)
