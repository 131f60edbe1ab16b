/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the selective-scan engine.
 *
 * A plain restatement of the reference's scalar recurrences
 * (kernel/arm-scan-core/src/scalar.rs, mamba3/scalar.rs, mamba3/mimo.rs),
 * built as liboracle.so.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load it, as the checker or as the timed CPU
 * baseline ("port").  The shipped library (armhackathon_b200/libb200scan.so)
 * never links it.
 *
 * Pinning: the f64 instantiation is checked against the reference's own
 * golden vectors (the npz fixtures under tests/golden, produced from the
 * reference's fixtures by tests/golden/make_fixtures.py) in
 * tests/test_oracle_golden.py.
 *
 * Threading stands in for the reference's rayon row parallelism
 * (kernel/arm-scan-core/src/parallel.rs:24-85): rows are split into
 * contiguous ranges, one std::thread per range.
 */
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <thread>
#include <vector>

extern "C" {
typedef struct { size_t batch, dim, len, state, groups; } oracle_m1_dims;
typedef struct { size_t batch, heads, dv, dqk, len, rank; } oracle_m3_dims;
}

template <class F>
static void oracle_parallel_rows(size_t nrows, int nthreads, F&& body) {
    size_t nt = nthreads > 1 ? (size_t)nthreads : 1;
    if (nt > nrows) nt = nrows;
    if (nt <= 1) { body((size_t)0, nrows); return; }
    std::vector<std::thread> pool;
    const size_t per = (nrows + nt - 1) / nt;
    for (size_t i = 0; i < nt; ++i) {
        const size_t r0 = i * per, r1 = r0 + per < nrows ? r0 + per : nrows;
        if (r0 >= r1) break;
        pool.emplace_back([&body, r0, r1] { body(r0, r1); });
    }
    for (auto& th : pool) th.join();
}

#define ROWS_BEGIN(n) oracle_parallel_rows((n), nthreads, [&](size_t r0, size_t r1) {
#define ROWS_END });

#define T float
#define FN(x) x##_f32
#define EXP expf
#define LOG1P log1pf
#include "scan_oracle_body.h"
#undef T
#undef FN
#undef EXP
#undef LOG1P

#define T double
#define FN(x) x##_f64
#define EXP exp
#define LOG1P log1p
#include "scan_oracle_body.h"
#undef T
#undef FN
#undef EXP
#undef LOG1P

extern "C" unsigned oracle_hw_threads(void) { return std::thread::hardware_concurrency(); }
