// Host-side check of the CTA-pair kernels' stream-K schedule (pair_work and
// streamk_split in gemm_common.cuh), compiled and run on the CPU by
// tests/test_gemm_plan.py: for every (tiles, k-blocks, pairs) case given on
// the command line, every k-block of every tile is run by exactly one pair,
// in one contiguous range per (pair, tile); a split tile is shared by exactly
// two pairs, p (its first k-blocks, on p's list right after its whole-wave
// tiles) and p + 1 (the rest, the last item on p + 1's list), which is the
// hand-off the kernel implements; and the pairs' k-block counts differ by at
// most one within the stream-K region.  Prints "OK <cases>" or the first violation.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../minixla_b200/csrc/gemm_common.cuh"

using namespace mxb;

static int check(int tiles, int nk, int pairs) {
    FusedParams p{};
    p.num_tiles = tiles;
    p.num_kb = nk;
    const StreamKSplit sk = streamk_split(tiles, nk, pairs);
    p.sk_dp_tiles = sk.dp_tiles;
    p.sk_q = sk.q;
    p.sk_extra = sk.extra;
    const int launched = tiles < pairs ? tiles : pairs;
    if (sk.q > 0 && (sk.q < nk || sk.dp_tiles % launched != 0)) {
        printf("FAIL tiles=%d nk=%d pairs=%d: q=%d dp=%d\n", tiles, nk, pairs, sk.q, sk.dp_tiles);
        return 1;
    }
    std::vector<int> owner(static_cast<size_t>(tiles) * nk, -1);
    std::vector<int> head_of(tiles, -1), tail_of(tiles, -1);
    std::vector<long long> work(launched, 0);
    for (int pr = 0; pr < launched; ++pr) {
        PairWork w;
        int n = 0, n_dp_seen = 0;
        for (int idx = 0; pair_work(p, pr, launched, idx, w); ++idx, ++n) {
            if (w.t < 0 || w.t >= tiles || w.kb0 < 0 || w.kb1 > nk || w.kb0 >= w.kb1) {
                printf("FAIL tiles=%d nk=%d pairs=%d: pair %d item %d bad (%d,%d,%d)\n", tiles, nk, pairs, pr, idx,
                       w.t, w.kb0, w.kb1);
                return 1;
            }
            for (int kb = w.kb0; kb < w.kb1; ++kb) {
                int& o = owner[static_cast<size_t>(w.t) * nk + kb];
                if (o != -1) {
                    printf("FAIL tiles=%d nk=%d pairs=%d: tile %d kb %d twice\n", tiles, nk, pairs, w.t, kb);
                    return 1;
                }
                o = pr;
            }
            if (w.t >= sk.dp_tiles || sk.q == 0) work[pr] += w.kb1 - w.kb0;
            if (sk.q > 0 && w.t < sk.dp_tiles) {
                if (idx != n_dp_seen) {  // the whole-wave tiles come first
                    printf("FAIL tiles=%d nk=%d pairs=%d: pair %d wave tile at item %d\n", tiles, nk, pairs, pr, idx);
                    return 1;
                }
                ++n_dp_seen;
            }
            const bool whole = w.kb0 == 0 && w.kb1 == nk;
            if (whole != (w.kind == kWorkFull) || (w.kind == kWorkHead && (w.kb0 != 0 || idx != n_dp_seen)) ||
                (w.kind == kWorkTail && w.kb1 != nk)) {
                printf("FAIL tiles=%d nk=%d pairs=%d: pair %d item %d kind %d (%d,%d)\n", tiles, nk, pairs, pr, idx,
                       w.kind, w.kb0, w.kb1);
                return 1;
            }
            if (w.kind == kWorkHead) head_of[w.t] = pr;
            if (w.kind == kWorkTail) tail_of[w.t] = pr;
        }
        // a tail is the last item of its pair's list
        PairWork last;
        if (n > 0 && pair_work(p, pr, launched, n - 1, last)) {
            for (int idx = 0; idx < n - 1; ++idx) {
                PairWork w;
                pair_work(p, pr, launched, idx, w);
                if (w.kind == kWorkTail) {
                    printf("FAIL tiles=%d nk=%d pairs=%d: pair %d tail not last\n", tiles, nk, pairs, pr);
                    return 1;
                }
            }
        }
    }
    for (size_t i = 0; i < owner.size(); ++i)
        if (owner[i] == -1) {
            printf("FAIL tiles=%d nk=%d pairs=%d: tile %zu kb %zu never run\n", tiles, nk, pairs, i / nk, i % nk);
            return 1;
        }
    for (int t = 0; t < tiles; ++t) {
        if ((head_of[t] == -1) != (tail_of[t] == -1) || (head_of[t] != -1 && tail_of[t] != head_of[t] + 1)) {
            printf("FAIL tiles=%d nk=%d pairs=%d: tile %d head %d tail %d\n", tiles, nk, pairs, t, head_of[t],
                   tail_of[t]);
            return 1;
        }
    }
    if (sk.q > 0) {
        long long lo = work[0], hi = work[0];
        for (long long x : work) {
            lo = x < lo ? x : lo;
            hi = x > hi ? x : hi;
        }
        if (hi - lo > 1) {
            printf("FAIL tiles=%d nk=%d pairs=%d: stream-K work %lld..%lld\n", tiles, nk, pairs, lo, hi);
            return 1;
        }
    }
    return 0;
}

int main(int argc, char** argv) {
    int cases = 0;
    for (int i = 1; i + 2 < argc; i += 3) {
        if (check(atoi(argv[i]), atoi(argv[i + 1]), atoi(argv[i + 2]))) return 1;
        ++cases;
    }
    printf("OK %d\n", cases);
    return 0;
}
