// Host-only check of the pipelined batch schedule (csrc/engine.hpp pipeline_pieces /
// pipeline_growth): two ranks that learned different growth factors before joining a gather, or
// from calls that gather nothing, still cut identical pieces once joined. Prints one line per
// case and "ok" at the end; any failed check prints "FAIL ..." and exits 1.
#include <cstdio>
#include <vector>

#include "engine.hpp"

static int fails = 0;
static void check(bool ok, const char *what, unsigned images) {
    if (!ok) {
        std::printf("FAIL %s (images %u)\n", what, images);
        fails++;
    }
}

int main() {
    const unsigned sizes[] = {512, 513, 1000, 2048, 2101, 4096, 65536};
    for (unsigned images : sizes) {
        for (double g : {uq::kRampedPieces, 1.15, 1.25, 2.7, 3.0}) {
            const std::vector<uint32_t> p = uq::pipeline_pieces(images, g);
            unsigned sum = 0;
            for (uint32_t n : p) sum += n;
            check(sum == images, "pieces cover the batch", images);
            check(p.size() <= uq::kMaxPieces, "at most kMaxPieces", images);
            for (uint32_t n : p) check(n > 0, "no empty piece", images);
        }
        // rank 0 learned 2.7 (decoder calls), rank 1 learned 1.2 (before joining)
        const auto r0 = uq::pipeline_pieces(images, uq::pipeline_growth(true, 2.7, 0.0));
        const auto r1 = uq::pipeline_pieces(images, uq::pipeline_growth(true, 1.2, 0.0));
        check(r0 == r1, "joined ranks cut identical pieces", images);
        check(r0 == uq::pipeline_pieces(images, uq::kInitialPieceGrowth), "joined ranks use the initial growth",
              images);
        check(uq::pipeline_growth(false, 2.7, 0.0) == 2.7, "a session alone uses what it learned", images);
        check(uq::pipeline_growth(true, 2.7, 1.5) == 1.5, "UNOQ_PIPE_GROWTH wins", images);
        // copy-bound calls: the ramped schedule starts and ends on a quarter of its middle size
        const auto rp = uq::pipeline_pieces(images, uq::kRampedPieces);
        if (images >= 768) {
            check(rp.size() >= 5 && rp.front() == rp.back() && rp[1] == rp[rp.size() - 2] && rp.front() < rp[1] &&
                      rp[1] < rp[2],
                  "ramped schedule: quarter and half pieces at both ends", images);
        }
        std::printf("images %u: %zu pieces, first %u, last %u; ramped %zu pieces, first %u, last %u\n", images,
                    r0.size(), r0.front(), r0.back(), rp.size(), rp.front(), rp.back());
    }
    if (fails) return 1;
    std::printf("ok\n");
    return 0;
}
