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
        for (double g : {uq::kCopyBoundPieces, 1.15, 1.25, 2.7, 3.0}) {
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
        // copy-bound calls: a first piece of 192 images (a quarter of smaller batches), then equal
        // pieces (differing by at most one image) of about 352, none below the break-even size
        // that keeps compute in step with the uploads unless the batch is too small for more
        const auto rp = uq::pipeline_pieces(images, uq::kCopyBoundPieces);
        check(rp.front() == (images / 4 < uq::kCopyBoundFirst ? images / 4 : uq::kCopyBoundFirst),
              "copy-bound schedule: first piece", images);
        uint32_t lo = ~0u, hi = 0;
        for (size_t i = 1; i < rp.size(); i++) lo = rp[i] < lo ? rp[i] : lo, hi = rp[i] > hi ? rp[i] : hi;
        check(rp.size() >= 2 && hi - lo <= 1, "copy-bound schedule: equal pieces after the first", images);
        check(rp.size() == uq::kMaxPieces || (lo >= uq::kCopyBoundPiece * 2 / 3 && hi <= uq::kCopyBoundPiece * 3 / 2) ||
                  rp.size() == 2,
              "copy-bound schedule: pieces near the break-even size", images);
        std::printf("images %u: %zu pieces, first %u, last %u; copy-bound %zu pieces, first %u, then %u\n", images,
                    r0.size(), r0.front(), r0.back(), rp.size(), rp.front(), rp[1]);
    }
    // learning: MobileNetV4-like timings (0.28 ms per piece + 1.93 us per image of compute against
    // 2.725 us per image of upload) stay copy-bound, and enter it from a growing call of 1,024
    // images whose largest piece alone looks compute-bound; the fitted model recovers the fixed
    // cost and slope. YOLO-like timings (0.95 ms + 8.16 us against 5.59 us) keep growing pieces.
    auto mnv4 = [](double n) { return (float)(0.28 + 1.93e-3 * n); };
    auto up_m = [](double n) { return (float)(2.725e-3 * n); };
    const uq::PieceChoice a = uq::learn_pieces(uq::kCopyBoundPieces, 355, up_m(355), mnv4(355), 192, mnv4(192));
    check(a.growth < 1.0 && a.model.fixed > 0.27 && a.model.fixed < 0.29 && a.model.slope > 1.9e-3 &&
              a.model.slope < 1.96e-3 && a.model.up > 2.7e-3 && a.model.up < 2.75e-3,
          "copy-bound call stays copy-bound with the fitted model", 4096);
    const uq::PieceChoice b = uq::learn_pieces(1.25, 304, up_m(304), mnv4(304) * 1.0f, 64, mnv4(64));
    check(b.growth < 1.0, "a growing call whose pieces are small enters the copy-bound schedule", 1024);
    auto yolo = [](double n) { return (float)(0.95 + 8.16e-3 * n); };
    const uq::PieceChoice c = uq::learn_pieces(1.25, 598, (float)(5.59e-3 * 598), yolo(598), 64, yolo(64));
    check(c.growth > 1.8 && c.growth < 2.1, "compute-bound call grows by 1.1 x compute / upload", 1024);
    const uq::PieceChoice d = uq::learn_pieces(1.25, 400, 1.0f, 0.8f, 0, 0.f);
    check(d.growth < 1.0 && d.model.up == 0.0, "one piece size: the largest piece's average decides, no model", 400);
    const uq::PieceChoice e = uq::learn_pieces(uq::kCopyBoundPieces, 355, 1.0f, 1.2f, 0, 0.f);
    check(e.growth >= 1.15, "compute above upload leaves the copy-bound schedule", 355);
    // planning on the MobileNetV4 model: the least simulated end time, which beats the model-free
    // rule and the ramped schedule it replaced (quarter and half pieces at both ends)
    for (unsigned images : {512u, 1024u, 2048u, 4096u, 8192u}) {
        const auto planned = uq::pipeline_pieces(images, uq::kCopyBoundPieces, a.model);
        unsigned sum = 0;
        for (uint32_t n : planned) sum += n;
        check(sum == images && planned.size() <= uq::kMaxPieces, "planned pieces cover the batch", images);
        const double e_plan = uq::pipeline_end(planned, a.model);
        const double e_rule = uq::pipeline_end(uq::pipeline_pieces(images, uq::kCopyBoundPieces), a.model);
        const uint32_t mid = images / 8 < 256 ? 256 : images / 8 > 1024 ? 1024 : images / 8;
        std::vector<uint32_t> ramp{mid / 4, mid / 2};
        const uint32_t rest = images - 3 * mid / 2;
        uint32_t m = (rest + mid / 2) / mid;
        m = m < 1 ? 1 : m;
        for (uint32_t i = 0; i < m; i++) ramp.push_back(rest / m + (i < rest % m ? 1 : 0));
        ramp.push_back(mid / 2);
        ramp.push_back(mid / 4);
        const double e_ramp = uq::pipeline_end(ramp, a.model);
        check(e_plan <= e_rule + 1e-9 && e_plan < e_ramp, "planned schedule ends first", images);
        std::printf("MobileNetV4 model, %u images: planned %zu pieces (first %u, then %u) %.2f ms, rule %.2f ms, ramped %.2f ms, upload %.2f ms\n",
                    images, planned.size(), planned[0], planned[1], e_plan, e_rule, e_ramp, a.model.up * images);
    }
    // planning on a YOLO26n-like model (compute-bound, outputs of 171 KB per image read back):
    // growing pieces, ending sooner than the growth-factor rule the session would use otherwise
    uq::PieceModel ym;
    ym.fixed = 0.95, ym.slope = 8.16e-3, ym.up = 5.59e-3, ym.down = 3.11e-3;
    for (unsigned images : {512u, 1024u, 2048u}) {
        const auto planned = uq::pipeline_pieces(images, 1.93, ym);
        unsigned sum = 0;
        for (uint32_t n : planned) sum += n;
        check(sum == images && planned.size() <= uq::kMaxPieces, "planned pieces cover the batch", images);
        const double e_plan = uq::pipeline_end(planned, ym), e_rule = uq::pipeline_end(uq::pipeline_pieces(images, 1.93), ym);
        check(e_plan <= e_rule, "planned compute-bound schedule ends no later", images);
        std::printf("YOLO26n model, %u images: planned %zu pieces (first %u, last %u) %.2f ms, growth rule %.2f ms\n",
                    images, planned.size(), planned.front(), planned.back(), e_plan, e_rule);
    }
    for (unsigned images : {128u, 1000u, 4096u})
        for (double g : {1.2, 2.0, 3.2})
            for (uint32_t tail : {0u, 64u}) {
                const auto gp = uq::growing_pieces(images, 64, g, tail);
                unsigned sum = 0;
                for (uint32_t n : gp) sum += n;
                check(gp.empty() || (sum == images && gp.size() <= uq::kMaxPieces), "growing pieces cover the batch", images);
            }
    if (fails) return 1;
    std::printf("ok\n");
    return 0;
}
