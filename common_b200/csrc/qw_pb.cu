// qw_pb.cu -- weights from the reference's own protobuf format (host code).
//
// The reference stores state dictionaries as protobuf CollectionLibraryData messages
// (engine/ml/src/main/proto/collections.proto):
//   CollectionLibraryData { repeated CollectionLibraryEntry collections = 1; }
//   CollectionLibraryEntry { string key = 1; CollectionData collection = 2; }
//   CollectionData { TraversalPolicyData traversal_policy = 1; repeated double data = 2;
//                    repeated float data_32 = 3; }
//   TraversalPolicyData { repeated int32 dims = 1; int32 traversal_axis = 2; }
// and StateDictionary(weightsDirectory) reads every non-hidden file of a directory
// (StateDictionary.java:119-150), decoding each entry with CollectionEncoder.decode (data when present,
// else data_32; an entry with no dimensions is null and skipped).  This is a small reader of the
// protobuf wire format for exactly these messages (packed or unpacked repeated fields), over a
// memory-mapped file, handing every entry to qw_load_tensor.
#include <dirent.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <utility>
#include <string>
#include <vector>

#include "../../include/qwen3_b200.h"

namespace qw {
void model_set_error(qw_model *m, const std::string &msg);  // qw_model.cu
}

namespace {

struct Wire {
    const uint8_t *p, *end;
    bool ok = true;

    bool more() const { return ok && p < end; }
    uint64_t varint() {
        uint64_t v = 0;
        for (int s = 0; s < 64; s += 7) {
            if (p >= end) { ok = false; return 0; }
            const uint8_t b = *p++;
            v |= (uint64_t)(b & 0x7F) << s;
            if (!(b & 0x80)) return v;
        }
        ok = false;
        return 0;
    }
    Wire sub() {  // a length-delimited field as its own reader
        const uint64_t n = varint();
        Wire w{p, p};
        if (!ok || n > (uint64_t)(end - p)) { ok = false; return w; }
        w.end = p + n;
        p += n;
        return w;
    }
    void skip(int wt) {
        switch (wt) {
            case 0: varint(); break;
            case 1: if (end - p < 8) ok = false; else p += 8; break;
            case 2: sub(); break;
            case 5: if (end - p < 4) ok = false; else p += 4; break;
            default: ok = false;
        }
    }
};

struct Entry {
    std::string key;
    std::vector<int64_t> dims;
    // byte ranges of the values in the mapped file, little-endian: packed chunks (a repeated field may be
    // split over several) and unpacked single values alike
    std::vector<std::pair<const uint8_t *, size_t>> r64, r32;
    size_t b64 = 0, b32 = 0;
};

bool parse_policy(Wire w, Entry &e) {
    while (w.more()) {
        const uint64_t tag = w.varint();
        const int field = (int)(tag >> 3), wt = (int)(tag & 7);
        if (field == 1 && wt == 2) {
            Wire pk = w.sub();
            while (pk.more()) e.dims.push_back((int64_t)(int32_t)pk.varint());
            if (!pk.ok) return false;
        } else if (field == 1 && wt == 0) {
            e.dims.push_back((int64_t)(int32_t)w.varint());
        } else {
            w.skip(wt);  // traversal_axis and anything unknown
        }
    }
    return w.ok;
}

bool parse_collection(Wire w, Entry &e) {
    while (w.more()) {
        const uint64_t tag = w.varint();
        const int field = (int)(tag >> 3), wt = (int)(tag & 7);
        if (field == 1 && wt == 2) {
            if (!parse_policy(w.sub(), e)) return false;
        } else if (field == 2 && (wt == 2 || wt == 1)) {
            const uint8_t *a = w.p;
            size_t n = 8;
            if (wt == 2) { Wire d = w.sub(); a = d.p; n = (size_t)(d.end - d.p); }
            else w.skip(1);
            if (!w.ok || n % 8) return false;
            e.r64.emplace_back(a, n);
            e.b64 += n;
        } else if (field == 3 && (wt == 2 || wt == 5)) {
            const uint8_t *a = w.p;
            size_t n = 4;
            if (wt == 2) { Wire d = w.sub(); a = d.p; n = (size_t)(d.end - d.p); }
            else w.skip(5);
            if (!w.ok || n % 4) return false;
            e.r32.emplace_back(a, n);
            e.b32 += n;
        } else {
            w.skip(wt);
        }
    }
    return w.ok;
}

// Entries of one file, parsed completely before any is used: a file the protobuf parser rejects contributes
// nothing, as CollectionLibraryData.parseFrom throwing does in StateDictionary.loadWeights.
bool parse_library(Wire w, std::vector<Entry> &out) {
    while (w.more()) {
        const uint64_t tag = w.varint();
        const int field = (int)(tag >> 3), wt = (int)(tag & 7);
        if (!(field == 1 && wt == 2)) { w.skip(wt); continue; }
        Wire ew = w.sub();
        Entry e;
        bool have = false;
        while (ew.more()) {
            const uint64_t t2 = ew.varint();
            const int f2 = (int)(t2 >> 3), wt2 = (int)(t2 & 7);
            if (f2 == 1 && wt2 == 2) {
                Wire k = ew.sub();
                e.key.assign((const char *)k.p, (size_t)(k.end - k.p));
            } else if (f2 == 2 && wt2 == 2) {
                if (!parse_collection(ew.sub(), e)) return false;
                have = true;
            } else {
                ew.skip(wt2);
            }
        }
        if (!ew.ok || !w.ok) return false;
        if (have && !e.dims.empty()) out.push_back(std::move(e));  // else CollectionEncoder.decode returns null
    }
    return w.ok;
}

// One file.  Following StateDictionary.loadWeights, a file that cannot be read or parsed, or an entry whose
// value count does not match its shape, ends that file with a warning (entries before it stay loaded) and
// loading goes on with the next file; a known key whose shape does not fit the model is an error.
qw_status load_file(qw_model *m, const std::string &path, int32_t *loaded, std::string &warn) {
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) { warn += "cannot open " + path + "; "; return QW_OK; }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); warn += "cannot stat " + path + "; "; return QW_OK; }
    if (st.st_size == 0) { close(fd); return QW_OK; }
    void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { warn += "cannot map " + path + "; "; return QW_OK; }
    std::vector<Entry> entries;
    qw_status s = QW_OK;
    if (!parse_library(Wire{(const uint8_t *)map, (const uint8_t *)map + st.st_size}, entries)) {
        warn += "malformed CollectionLibraryData in " + path + "; ";
        entries.clear();
    }
    std::vector<double> al64;
    std::vector<float> al32;
    for (Entry &e : entries) {
        // CollectionEncoder.decode: `data` (doubles) when present, else `data_32`
        const void *ptr;
        qw_dtype dt;
        size_t n;
        if (e.b64) {
            dt = QW_DTYPE_F64;
            al64.resize(e.b64 / 8);
            uint8_t *o = (uint8_t *)al64.data();
            for (auto &r : e.r64) { memcpy(o, r.first, r.second); o += r.second; }
            ptr = al64.data();
            n = al64.size();
        } else {
            dt = QW_DTYPE_F32;
            al32.resize(e.b32 / 4);
            uint8_t *o = (uint8_t *)al32.data();
            for (auto &r : e.r32) { memcpy(o, r.first, r.second); o += r.second; }
            ptr = al32.data();
            n = al32.size();
        }
        int64_t numel = 1;
        for (int64_t d : e.dims) numel = d < 0 ? -1 : numel * d;
        if (numel < 0 || (size_t)numel != n) {
            warn += "'" + e.key + "' in " + path + ": " + std::to_string(n) + " values for shape of " +
                    std::to_string(numel) + "; ";
            break;
        }
        const qw_status ls = qw_load_tensor(m, e.key.c_str(), dt, e.dims.data(), (int32_t)e.dims.size(), ptr);
        if (ls == QW_ERR_KEY) continue;  // a tensor this model does not use
        if (ls) { s = ls; break; }
        (*loaded)++;
    }
    munmap(map, (size_t)st.st_size);
    return s;
}

}  // namespace

extern "C" qw_status qw_load_state_dict_pb(qw_model *m, const char *path, int32_t *loaded_out) {
    if (!m || !path) return QW_ERR_ARG;
    int32_t loaded = 0;
    std::string warn;
    qw_status s = QW_OK;
    struct stat st;
    if (stat(path, &st) != 0) {
        qw::model_set_error(m, std::string("load_state_dict_pb: no such file or directory: ") + path);
        return QW_ERR_ARG;
    }
    if (S_ISDIR(st.st_mode)) {
        DIR *d = opendir(path);
        std::vector<std::string> names;
        if (d) {
            while (struct dirent *de = readdir(d))
                if (de->d_name[0] != '.') names.push_back(de->d_name);
            closedir(d);
        }
        std::sort(names.begin(), names.end());
        for (const auto &n : names) {
            const std::string f = std::string(path) + "/" + n;
            struct stat fs;
            if (stat(f.c_str(), &fs) != 0 || !S_ISREG(fs.st_mode)) continue;
            s = load_file(m, f, &loaded, warn);
            if (s) break;
        }
    } else {
        s = load_file(m, path, &loaded, warn);
    }
    if (loaded_out) *loaded_out = loaded;
    if (!s && !warn.empty()) {
        fprintf(stderr, "qw_load_state_dict_pb: skipped %s\n", warn.c_str());
        qw::model_set_error(m, "load_state_dict_pb skipped: " + warn);
    }
    return s;
}
