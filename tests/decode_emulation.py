"""The GPU decoder's contract (include/unoq_cuda.h UgYoloDecode / UgDetectionRecord) restated in
numpy, for tests: from a packed int8 head output and the installed tables, the records that
ug_detect_batch must return, bit for bit. Follows the reference decode (modern.py:75-103):
stage 1 = argsort(-best score, stable)[:candidates], stage 2 = argsort(-flat, stable)[:k]."""
import numpy as np

from unoq_dsp.native import NO_ANCHOR, RECORD_DTYPE


def level_arrays(config):
    levels = []
    for l in range(config.levels):
        lv = config.level[l]
        levels.append({"box": lv.box_offset, "score": lv.score_offset, "h": lv.height, "w": lv.width,
                       "stride": np.float32(lv.stride), "distance": np.array(lv.distance[:], dtype="f4"),
                       "scores": np.array(lv.score[:], dtype="f4"), "rank": np.array(lv.rank[:], dtype=np.int64)})
    return levels


def emulate(config, packed, k):
    """packed: (N, output_bytes) int8 -> (N, k) RECORD_DTYPE."""
    packed = np.asarray(packed).reshape(len(packed), -1).view(np.int8)
    C, levels = config.classes, level_arrays(config)
    out = np.zeros((len(packed), k), dtype=RECORD_DTYPE)
    out["anchor"] = NO_ANCHOR
    for n, img in enumerate(packed):
        codes, where = [], []
        for l, lv in enumerate(levels):
            cells = lv["h"] * lv["w"]
            q = img[lv["score"]:lv["score"] + cells * C].reshape(cells, C).astype(np.int64)
            codes.append(lv["rank"][q + 128])
            where += [(l, cell) for cell in range(cells)]
        codes = np.concatenate(codes)
        best = codes.max(1)
        first = np.lexsort((np.arange(len(best)), -best))[:min(config.candidates, len(best))]
        flat = codes[first].reshape(-1)
        second = np.lexsort((np.arange(flat.size), -flat))[:min(k, flat.size)]
        for r, j in enumerate(second):
            i, c = divmod(int(j), C)
            a = int(first[i])
            l, cell = where[a]
            lv = levels[l]
            q = int(img[lv["score"] + cell * C + c])
            d = lv["distance"][img[lv["box"] + 4 * cell:lv["box"] + 4 * cell + 4].astype(np.int64) + 128]
            gx, gy = np.float32(cell % lv["w"]) + np.float32(.5), np.float32(cell // lv["w"]) + np.float32(.5)
            st = lv["stride"]
            out[n, r] = (a, c, lv["scores"][q + 128], ((gx - d[0]) * st, (gy - d[1]) * st, (gx + d[2]) * st,
                                                       (gy + d[3]) * st), 0)
    return out


def packed_specs(outputs):
    """Give a contract's output specs back-to-back packed offsets (the model compiler's layout)."""
    at, specs = 0, []
    for spec in outputs:
        spec = dict(spec, packed_offset=at, bytes=int(np.prod(spec["shape"])))
        at += spec["bytes"]
        specs.append(spec)
    return specs, at


def pack(raw, specs, total):
    buf = np.zeros(total, dtype=np.int8)
    for spec in specs:
        buf[spec["packed_offset"]:spec["packed_offset"] + spec["bytes"]] = np.asarray(raw[spec["name"]]).reshape(-1)
    return buf
