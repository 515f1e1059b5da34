// handoff.cpp - the hand-off table (include/strata_kv/handoff.hpp).
//
// Decisions (claim, publish, release, reclaim, cancel) run under the arena file's exclusive flock plus a
// process mutex (a flock belongs to an open file description, so two threads on one handle would share it);
// header reads for readers and diagnostics take a shared flock.  Payload bytes are written with no lock held.
#include "strata_kv/handoff.hpp"

#include <atomic>
#include <cerrno>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <filesystem>
#include <fstream>
#include <sstream>

#include <fcntl.h>
#include <signal.h>
#include <sys/file.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/statvfs.h>
#include <unistd.h>

namespace strata::core {
namespace {

const char kArenaMagic[] = "STRATA-HARENA-V1";   // 16 bytes on disk, no terminator
const char kSlotMagic[] = "STRATA-HSLOT-V1";     // 15 bytes + the terminator = 16 on disk

bool fail(std::string& err, const std::string& why) {
    err = "handoff arena: " + why;
    return false;
}
std::string hex16(uint64_t v) {
    char b[20];
    std::snprintf(b, sizeof b, "%016llx", (unsigned long long) v);
    return b;
}
std::string num(uint64_t v) { return std::to_string(v); }
const char* state_name(uint32_t s) {
    return s == kHandoffFree ? "FREE" : s == kHandoffClaimed ? "CLAIMED" : s == kHandoffReady ? "READY" : "UNKNOWN";
}
uint64_t me_pid() { return (uint64_t) (uint32_t) ::getpid(); }

uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
/// A fresh, non-zero nonce: time, pid and a process counter mixed.
uint64_t fresh_nonce() {
    static std::atomic<uint64_t> counter{0};
    timespec ts{};
    clock_gettime(CLOCK_REALTIME, &ts);
    const uint64_t v = splitmix64(((uint64_t) ts.tv_sec * 1000000000ull + (uint64_t) ts.tv_nsec) ^ (me_pid() << 32) ^
                                  (counter.fetch_add(1) * 0xD1B54A32D192ED03ull));
    return v ? v : 1;
}

bool pread_all(int fd, void* p, uint64_t n, uint64_t off) {
    uint64_t done = 0;
    while (done < n) {
        const ssize_t r = ::pread(fd, static_cast<uint8_t*>(p) + done, n - done, (off_t) (off + done));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        done += (uint64_t) r;
    }
    return true;
}
bool pwrite_all(int fd, const void* p, uint64_t n, uint64_t off) {
    uint64_t done = 0;
    while (done < n) {
        const ssize_t r = ::pwrite(fd, static_cast<const uint8_t*>(p) + done, n - done, (off_t) (off + done));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        done += (uint64_t) r;
    }
    return true;
}

bool slot_header_sane(const HandoffSlotHeader& h) {
    return std::memcmp(h.magic, kSlotMagic, 16) == 0 && h.version == kHandoffVersion &&
           h.header_bytes == kHandoffHeaderBytes;
}

/// Why an arena header's tier table cannot describe its file, or "" when it can: the tiers lie back to back from
/// byte 4096 in order, each count x (4096-byte header + slot bytes) without overflow, the slot counts add up to
/// slot_total (an int slot index reaches them all), and the last tier ends at arena_bytes.  A reader checks this
/// before it computes any slot address from the header of a file another process wrote.
std::string tier_layout_error(const HandoffArenaHeader& h) {
    uint64_t at = kHandoffHeaderBytes, slots = 0;
    for (uint32_t t = 0; t < h.tier_count; ++t) {
        if (h.tier_slot_off[t] != at) return "tier " + num(t) + " starts at byte " + num(h.tier_slot_off[t]) + ", not " + num(at);
        uint64_t region = 0;
        if (__builtin_add_overflow(h.tier_slot_bytes[t], kHandoffHeaderBytes, &region) ||
            __builtin_mul_overflow(region, h.tier_slot_count[t], &region) || __builtin_add_overflow(at, region, &at) ||
            __builtin_add_overflow(slots, h.tier_slot_count[t], &slots))
            return "tier " + num(t) + "'s size overflows";
    }
    if (slots != h.slot_total) return "the tiers hold " + num(slots) + " slots, the header says " + num(h.slot_total);
    if (slots > (uint64_t) INT32_MAX) return "more slots than an int index reaches";
    if (at != h.arena_bytes) return "the tiers end at byte " + num(at) + ", the header says " + num(h.arena_bytes);
    return {};
}

std::string tier_list(const uint64_t* v, uint32_t n) {
    std::string s;
    for (uint32_t i = 0; i < n; ++i) s += (i ? "," : "") + num(v[i]);
    return s;
}
std::string gib(uint64_t bytes) {
    char b[32];
    std::snprintf(b, sizeof b, "%.2f GiB", (double) bytes / (double) (1ull << 30));
    return b;
}

}  // namespace

// ------------------------------------------------------------------------------------------------ processes

uint64_t handoff_now_ms() {
    timespec ts{};
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t) ts.tv_sec * 1000ull + (uint64_t) ts.tv_nsec / 1000000ull;
}

bool handoff_pid_alive(uint64_t pid) {
    if (pid == 0 || pid > (uint64_t) INT_MAX) return false;
    return ::kill((pid_t) pid, 0) == 0 || errno == EPERM;
}

uint64_t handoff_proc_start_time(uint64_t pid) {
    if (pid == 0) return 0;
    std::ifstream f("/proc/" + std::to_string(pid) + "/stat");
    if (!f) return 0;
    std::string line;
    std::getline(f, line);
    const size_t close = line.rfind(')');
    if (close == std::string::npos) return 0;
    std::istringstream rest(line.substr(close + 1));
    std::string field;
    // after the command name: field 3 (state) onwards; the start time is field 22
    for (int i = 3; i <= 22; ++i)
        if (!(rest >> field)) return 0;
    return std::strtoull(field.c_str(), nullptr, 10);
}

bool handoff_claim_alive(uint64_t pid, uint64_t start_time) {
    if (!handoff_pid_alive(pid)) return false;
    if (start_time == 0) return true;   // unknown must never read as dead
    return handoff_proc_start_time(pid) == start_time;
}

// ------------------------------------------------------------------------------------------------ identity

std::string handoff_split_spec(const HandoffSplit& split) {
    std::string s = "main=" + std::to_string(split.main_lo) + ".." + std::to_string(split.main_hi);
    for (size_t i = 0; i < split.stages.size(); ++i)
        s += "|s" + std::to_string(i + 1) + "=" + std::to_string(split.stages[i].layer_lo) + ".." +
             std::to_string(split.stages[i].layer_hi);
    s += "|n=" + std::to_string(1 + split.stages.size());
    s += std::string("|draft=") + (split.stages.empty() ? "main" : split.draft_on_last ? "last" : "main");
    return s;
}

uint64_t handoff_geom_hash(const std::array<int64_t, 18>& geometry, const std::string& split_spec) {
    uint8_t key[18 * 8];
    for (size_t i = 0; i < 18; ++i)
        for (int b = 0; b < 8; ++b) key[i * 8 + (size_t) b] = (uint8_t) ((uint64_t) geometry[i] >> (8 * b));
    const uint64_t h = fnv1a64(key, sizeof key);
    return fnv1a64(reinterpret_cast<const uint8_t*>(split_spec.data()), split_spec.size(), h);
}

std::string handoff_arena_path(const std::string& dir, uint64_t pack_hash, const std::string& split_spec,
                               const std::string& instance) {
    return dir + "/" + hex16(pack_hash) + "-" + split_spec + "/" + instance + "/arena";
}

// ------------------------------------------------------------------------------------------------ sizing

bool handoff_size_arena(const std::vector<HandoffTierSpec>& tiers, const std::vector<uint64_t>& priced,
                        HandoffSizing& out, std::string& err) {
    if (tiers.empty()) return fail(err, "no tiers: an arena needs at least one tier");
    if (tiers.size() > (size_t) kHandoffMaxTiers)
        return fail(err, num(tiers.size()) + " tiers, but the header holds at most " + num(kHandoffMaxTiers) + " tiers");
    if (priced.size() != tiers.size()) return fail(err, "one priced payload per tier is required");
    for (size_t i = 0; i < tiers.size(); ++i) {
        if (tiers[i].slot_count == 0)
            return fail(err, "tier " + num(i) + " (" + num(tiers[i].max_tokens) + " tokens) has 0 slots");
        if (tiers[i].max_tokens == 0) return fail(err, "tier " + num(i) + " has 0 tokens");
        if (i && tiers[i].max_tokens <= tiers[i - 1].max_tokens)
            return fail(err, "tiers must ascend by token count (" + num(tiers[i - 1].max_tokens) + " then " +
                                 num(tiers[i].max_tokens) + ")");
    }
    HandoffSizing s;
    s.tiers = tiers;
    s.payload_bytes = priced;
    uint64_t at = kHandoffHeaderBytes;
    for (size_t i = 0; i < tiers.size(); ++i) {
        const uint64_t slot = handoff_round_up_64(priced[i]) + kHandoffSlackBytes;
        if (slot < priced[i]) return fail(err, "slot size overflow");
        s.slot_bytes.push_back(slot);
        s.slot_off.push_back(at);
        const uint64_t group = tiers[i].slot_count * (kHandoffHeaderBytes + slot);
        if (group / tiers[i].slot_count != kHandoffHeaderBytes + slot || at + group < at)
            return fail(err, "arena size overflow");
        at += group;
        s.slot_total += tiers[i].slot_count;
    }
    s.arena_bytes = at;
    s.max_tokens = tiers.back().max_tokens;
    std::string counts, toks;
    for (size_t i = 0; i < tiers.size(); ++i) {
        counts += (i ? "," : "") + num(tiers[i].slot_count);
        toks += (i ? "," : "") + num(tiers[i].max_tokens);
    }
    s.describe = "slots " + counts + " (tiers " + toks + "), max " + num(s.max_tokens) + " tokens, arena " +
                 gib(s.arena_bytes) + " (" + num(s.arena_bytes) + " B)";
    out = std::move(s);
    return true;
}

bool handoff_size_arena(const std::vector<HandoffTierSpec>& tiers, const HandoffPricer& pricer, HandoffSizing& out,
                        std::string& err) {
    if (tiers.empty()) return fail(err, "no tiers: an arena needs at least one tier");
    if (tiers.size() > (size_t) kHandoffMaxTiers)
        return fail(err, num(tiers.size()) + " tiers, but the header holds at most " + num(kHandoffMaxTiers) + " tiers");
    std::vector<uint64_t> priced(tiers.size());
    for (size_t i = 0; i < tiers.size(); ++i) {
        if (tiers[i].slot_count == 0)
            return fail(err, "tier " + num(i) + " (" + num(tiers[i].max_tokens) + " tokens) has 0 slots");
        if (i && tiers[i].max_tokens <= tiers[i - 1].max_tokens)
            return fail(err, "tiers must ascend by token count (" + num(tiers[i - 1].max_tokens) + " then " +
                                 num(tiers[i].max_tokens) + ")");
        std::string why;
        if (!pricer || !pricer(tiers[i].max_tokens, priced[i], why))
            return fail(err, "pricing tier " + num(i) + " (" + num(tiers[i].max_tokens) + " tokens): " + why);
    }
    return handoff_size_arena(tiers, priced, out, err);
}

// ------------------------------------------------------------------------------------------------ payload

HandoffPayload::~HandoffPayload() { unbind(); }
HandoffPayload::HandoffPayload(HandoffPayload&& o) noexcept { *this = std::move(o); }
HandoffPayload& HandoffPayload::operator=(HandoffPayload&& o) noexcept {
    if (this != &o) {
        unbind();
        data = std::exchange(o.data, nullptr);
        bytes = std::exchange(o.bytes, 0);
        index = o.index;
        tier = o.tier;
        nonce = o.nonce;
        client_id = o.client_id;
        request_id = o.request_id;
        tokens = o.tokens;
        payload_bytes = o.payload_bytes;
        payload_hash = o.payload_hash;
        seq = o.seq;
        map_ = std::exchange(o.map_, nullptr);
        map_bytes_ = std::exchange(o.map_bytes_, 0);
    }
    return *this;
}
void HandoffPayload::bind_mapping(void* map, uint64_t map_bytes, const uint8_t* d, uint64_t n) {
    unbind();
    map_ = map;
    map_bytes_ = map_bytes;
    data = d;
    bytes = n;
}
void HandoffPayload::unbind() {
    if (map_) ::munmap(map_, map_bytes_);
    map_ = nullptr;
    map_bytes_ = 0;
    data = nullptr;
    bytes = 0;
}

// ------------------------------------------------------------------------------------------------ the arena

struct HandoffArena::Locked {
    const HandoffArena& a;
    bool ok = false;
    Locked(const HandoffArena& arena, bool exclusive) : a(arena) {
        a.mu_.lock();
        int r;
        do {
            r = ::flock(a.fd_, exclusive ? LOCK_EX : LOCK_SH);
        } while (r != 0 && errno == EINTR);
        ok = r == 0;
    }
    ~Locked() {
        if (ok) ::flock(a.fd_, LOCK_UN);
        a.mu_.unlock();
    }
};

HandoffArena::HandoffArena() {
    if (const char* v = std::getenv("STRATA_HANDOFF_LEASE_MS")) lease_ms_ = std::strtoull(v, nullptr, 10);
}
HandoffArena::~HandoffArena() { close_(); }
HandoffArena::HandoffArena(HandoffArena&& o) noexcept { *this = std::move(o); }
HandoffArena& HandoffArena::operator=(HandoffArena&& o) noexcept {
    if (this != &o) {
        close_();
        fd_ = std::exchange(o.fd_, -1);
        writer_ = std::exchange(o.writer_, false);
        path_ = std::move(o.path_);
        hdr_ = o.hdr_;
        o.hdr_ = HandoffArenaHeader{};
        lease_ms_ = o.lease_ms_;
        client_pids_ = std::move(o.client_pids_);
    }
    return *this;
}

void HandoffArena::close_() {
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
    writer_ = false;
    path_.clear();
    hdr_ = HandoffArenaHeader{};
}

uint64_t HandoffArena::tier_max_tokens(uint32_t t) const { return t < hdr_.tier_count ? hdr_.tier_max_tokens[t] : 0; }
uint64_t HandoffArena::tier_slot_bytes(uint32_t t) const { return t < hdr_.tier_count ? hdr_.tier_slot_bytes[t] : 0; }
uint64_t HandoffArena::tier_slot_count(uint32_t t) const { return t < hdr_.tier_count ? hdr_.tier_slot_count[t] : 0; }
uint64_t HandoffArena::tier_slot_off(uint32_t t) const { return t < hdr_.tier_count ? hdr_.tier_slot_off[t] : 0; }

bool HandoffArena::locate_(int index, uint64_t& base, uint32_t& tier, uint64_t& capacity) const {
    if (index < 0) return false;
    uint64_t seen = 0;
    for (uint32_t t = 0; t < hdr_.tier_count; ++t) {
        const uint64_t n = hdr_.tier_slot_count[t];
        if ((uint64_t) index < seen + n) {
            base = hdr_.tier_slot_off[t] + ((uint64_t) index - seen) * (kHandoffHeaderBytes + hdr_.tier_slot_bytes[t]);
            tier = t;
            capacity = hdr_.tier_slot_bytes[t];
            return true;
        }
        seen += n;
    }
    return false;
}

bool HandoffArena::load_slot_(int index, HandoffSlotHeader& h, uint64_t& base, uint64_t& capacity) const {
    uint32_t tier = 0;
    if (fd_ < 0 || !locate_(index, base, tier, capacity)) return false;
    return pread_all(fd_, &h, sizeof h, base);
}

bool HandoffArena::store_(uint64_t off, const void* p, uint64_t n) const { return pwrite_all(fd_, p, n, off); }

bool HandoffArena::reset_slot_(uint64_t base, uint32_t tier, uint32_t flags) const {
    HandoffSlotHeader s{};
    std::memcpy(s.magic, kSlotMagic, 16);
    s.version = kHandoffVersion;
    s.header_bytes = (uint32_t) kHandoffHeaderBytes;
    s.state = kHandoffFree;
    s.flags = flags;
    s.tier = tier;
    return store_(base, &s, sizeof s);
}

bool HandoffArena::open_writer(const std::string& path, const HandoffSizing& sz, uint64_t pack_hash,
                               uint64_t geom_hash, std::string& err, bool allow_existing_writer) {
    if (pack_hash == 0) return fail(err, "the pack hash must be non-zero");
    if (geom_hash == 0) return fail(err, "the geometry hash must be non-zero");
    const size_t nt = sz.tiers.size();
    if (nt == 0 || nt > (size_t) kHandoffMaxTiers || sz.slot_bytes.size() != nt || sz.slot_off.size() != nt)
        return fail(err, "the sizing is malformed (tier tables of different lengths)");
    uint64_t at = kHandoffHeaderBytes, total = 0;
    for (size_t i = 0; i < nt; ++i) {
        if (sz.slot_off[i] != at)
            return fail(err, "the sizing puts tier " + num(i) + " at byte " + num(sz.slot_off[i]) + " but the layout says " +
                                 num(at));
        at += sz.tiers[i].slot_count * (kHandoffHeaderBytes + sz.slot_bytes[i]);
        total += sz.tiers[i].slot_count;
    }
    if (at != sz.arena_bytes)
        return fail(err, "the sizing's arena_bytes " + num(sz.arena_bytes) + " does not add up: its layout is " +
                             num(at) + " bytes");
    close_();
    namespace fs = std::filesystem;
    const fs::path p(path);
    std::error_code ec;
    if (p.has_parent_path()) fs::create_directories(p.parent_path(), ec);
    if (ec) return fail(err, "cannot create " + p.parent_path().string() + ": " + ec.message());
    const uint64_t me = me_pid(), my_start = handoff_proc_start_time(me_pid());
    struct stat st{};
    if (::stat(path.c_str(), &st) == 0) {
        fd_ = ::open(path.c_str(), O_RDWR | O_CLOEXEC);
        if (fd_ < 0) return fail(err, "cannot open " + path + ": " + std::strerror(errno));
        HandoffArenaHeader h{};
        bool ok = true;
        {
            Locked lk(*this, true);
            if (!lk.ok || !pread_all(fd_, &h, sizeof h, 0)) ok = fail(err, "cannot read the header of " + path);
            else if (std::memcmp(h.magic, kArenaMagic, 16) != 0) ok = fail(err, path + " is not a handoff arena (bad magic)");
            else if (h.version != kHandoffVersion)
                ok = fail(err, path + " is arena version " + num(h.version) + "; this build reads version 1");
            else if (h.header_bytes != kHandoffHeaderBytes)
                ok = fail(err, path + " has header_bytes " + num(h.header_bytes) + ", not 4096");
            else if (::fstat(fd_, &st) != 0 || (uint64_t) st.st_size != h.arena_bytes)
                ok = fail(err, path + " is " + num((uint64_t) st.st_size) + " bytes but its header says " + num(h.arena_bytes));
            else if (h.arena_bytes != sz.arena_bytes)
                ok = fail(err, "the arena at " + path + " holds " + num(h.arena_bytes) + " bytes; this tier table needs " +
                                   num(sz.arena_bytes));
            else if (h.pack_hash != pack_hash)
                ok = fail(err, "pack hash " + hex16(h.pack_hash) + " of " + path + " differs from this instance's " +
                                   hex16(pack_hash));
            else if (h.geom_hash != geom_hash)
                ok = fail(err, "geometry hash " + hex16(h.geom_hash) + " of " + path + " differs from this instance's " +
                                   hex16(geom_hash));
            else {
                bool same = h.tier_count == nt && h.slot_total == total;
                for (size_t i = 0; same && i < nt; ++i)
                    same = h.tier_max_tokens[i] == sz.tiers[i].max_tokens && h.tier_slot_count[i] == sz.tiers[i].slot_count &&
                           h.tier_slot_bytes[i] == sz.slot_bytes[i] && h.tier_slot_off[i] == sz.slot_off[i];
                if (!same) ok = fail(err, "the tier table of " + path + " differs from this sizing");
            }
            if (ok && h.created_pid != me) {
                if (handoff_claim_alive(h.created_pid, h.created_start)) {
                    if (!allow_existing_writer)
                        ok = fail(err, "one arena per prefill instance: " + path + " belongs to the live pid " +
                                           num(h.created_pid));
                } else {
                    // the creator is gone: nothing of a dead instance's table survives a restart
                    h.created_pid = me;
                    h.created_start = my_start;
                    hdr_ = h;
                    ok = store_(0, &h, sizeof h);
                    for (uint64_t i = 0; ok && i < h.slot_total; ++i) {
                        uint64_t base = 0, cap = 0;
                        uint32_t tier = 0;
                        ok = locate_((int) i, base, tier, cap) && reset_slot_(base, tier, 0);
                    }
                    if (!ok) fail(err, "cannot rebuild the slot table of " + path);
                }
            }
        }
        if (!ok) {
            close_();
            return false;
        }
        hdr_ = h;
    } else {
        struct statvfs sv{};
        const std::string dir = p.has_parent_path() ? p.parent_path().string() : ".";
        if (::statvfs(dir.c_str(), &sv) != 0) return fail(err, "cannot statvfs " + dir + ": " + std::strerror(errno));
        const uint64_t avail = (uint64_t) sv.f_bavail * (uint64_t) (sv.f_frsize ? sv.f_frsize : sv.f_bsize);
        if (sz.arena_bytes > avail)
            return fail(err, "the arena needs " + num(sz.arena_bytes) + " bytes but " + dir + " has " + num(avail) +
                                 " bytes free");
        fd_ = ::open(path.c_str(), O_RDWR | O_CREAT | O_EXCL | O_CLOEXEC, 0644);
        if (fd_ < 0) return fail(err, "cannot create " + path + ": " + std::strerror(errno));
        if (::ftruncate(fd_, (off_t) sz.arena_bytes) != 0) {
            const std::string why = std::strerror(errno);
            close_();
            ::unlink(path.c_str());
            return fail(err, "cannot size " + path + " to " + num(sz.arena_bytes) + " bytes: " + why);
        }
        HandoffArenaHeader h{};
        std::memcpy(h.magic, kArenaMagic, 16);
        h.version = kHandoffVersion;
        h.header_bytes = (uint32_t) kHandoffHeaderBytes;
        h.tier_count = (uint32_t) nt;
        h.slot_total = total;
        h.arena_bytes = sz.arena_bytes;
        h.pack_hash = pack_hash;
        h.geom_hash = geom_hash;
        h.created_pid = me;
        h.created_start = my_start;
        for (size_t i = 0; i < nt; ++i) {
            h.tier_max_tokens[i] = sz.tiers[i].max_tokens;
            h.tier_slot_count[i] = sz.tiers[i].slot_count;
            h.tier_slot_bytes[i] = sz.slot_bytes[i];
            h.tier_slot_off[i] = sz.slot_off[i];
        }
        hdr_ = h;
        bool ok = true;
        {
            Locked lk(*this, true);
            ok = lk.ok && store_(0, &h, sizeof h);
            for (uint64_t i = 0; ok && i < total; ++i) {
                uint64_t base = 0, cap = 0;
                uint32_t tier = 0;
                ok = locate_((int) i, base, tier, cap) && reset_slot_(base, tier, 0);
            }
        }
        if (!ok) {
            close_();
            ::unlink(path.c_str());
            return fail(err, "cannot write the header of " + path);
        }
    }
    writer_ = true;
    path_ = path;
    return true;
}

void HandoffArena::note_client_pid(uint64_t client_id, uint64_t pid) {
    std::lock_guard<std::mutex> lock(mu_);
    for (auto& cp : client_pids_)
        if (cp.first == client_id) {
            cp.second = pid;
            return;
        }
    client_pids_.emplace_back(client_id, pid);
}

std::vector<HandoffReclaim> HandoffArena::reclaim(std::string* err) {
    if (fd_ < 0) {
        if (err) *err = "handoff arena: reclaim on an arena that is not open";
        return {};
    }
    if (!writer_) {
        if (err) *err = "handoff arena: only the writer reclaims slots";
        return {};
    }
    Locked lk(*this, true);
    if (!lk.ok) {
        if (err) *err = "handoff arena: cannot lock " + path_;
        return {};
    }
    return reclaim_locked_(err);
}

std::vector<HandoffReclaim> HandoffArena::reclaim_locked_(std::string*) {
    std::vector<HandoffReclaim> out;
    const uint64_t now = handoff_now_ms();
    auto expired = [&](uint64_t since) { return now >= since && now - since > lease_ms_; };
    for (uint64_t i = 0; i < hdr_.slot_total; ++i) {
        HandoffSlotHeader h{};
        uint64_t base = 0, cap = 0;
        if (!load_slot_((int) i, h, base, cap) || !slot_header_sane(h)) continue;
        std::string why;
        uint64_t since = h.claimed_ms;
        if (h.state == kHandoffClaimed) {
            if (!handoff_claim_alive(h.owner_pid, h.owner_start))
                why = "the owner pid " + num(h.owner_pid) + " is gone";
            else if (expired(h.claimed_ms))
                why = "the claim's lease of " + num(lease_ms_) + " ms expired";
        } else if (h.state == kHandoffReady) {
            since = h.published_ms ? h.published_ms : h.claimed_ms;
            uint64_t pid = 0;
            for (const auto& cp : client_pids_)
                if (cp.first == h.client_id) pid = cp.second;
            if (pid && !handoff_pid_alive(pid))
                why = "the reader (client " + num(h.client_id) + ", pid " + num(pid) + ") is gone";
            else if (expired(since))
                why = "the READY slot's lease of " + num(lease_ms_) + " ms expired unread";
        }
        if (why.empty()) continue;
        HandoffReclaim r;
        r.index = (int) i;
        r.was_state = h.state;
        r.flags = h.flags;
        r.owner_pid = h.owner_pid;
        r.client_id = h.client_id;
        r.nonce = h.nonce;
        r.payload_bytes = h.payload_bytes;
        r.age_ms = now >= since ? now - since : 0;
        r.why = why;
        if (reset_slot_(base, h.tier, kHandoffFlagAbandoned)) out.push_back(std::move(r));
    }
    return out;
}

std::string HandoffArena::free_slots_locked_() const {
    uint64_t free = 0;
    for (uint64_t i = 0; i < hdr_.slot_total; ++i) {
        HandoffSlotHeader h{};
        uint64_t base = 0, cap = 0;
        if (load_slot_((int) i, h, base, cap) && slot_header_sane(h) && h.state == kHandoffFree) ++free;
    }
    return num(free) + "/" + num(hdr_.slot_total);
}

std::string HandoffArena::free_slots(std::string* err) const {
    if (fd_ < 0) {
        if (err) *err = "handoff arena: not open";
        return "0/0";
    }
    Locked lk(*this, false);
    return free_slots_locked_();
}

bool HandoffArena::claim(uint32_t tier, uint64_t client_id, uint64_t request_id, HandoffClaim& out, std::string& err) {
    out = HandoffClaim{};
    if (fd_ < 0) return fail(err, "the arena is not open");
    if (!writer_) return fail(err, "a reader never claims a slot");
    if (tier >= hdr_.tier_count)
        return fail(err, "tier " + num(tier) + " is not in this arena (it has " + num(hdr_.tier_count) + " tiers)");
    Locked lk(*this, true);
    if (!lk.ok) return fail(err, "cannot lock " + path_);
    reclaim_locked_(nullptr);
    for (uint64_t i = 0; i < hdr_.slot_total; ++i) {
        uint64_t base = 0, cap = 0;
        uint32_t t = 0;
        if (!locate_((int) i, base, t, cap) || t < tier) continue;   // the smallest group >= the job's tier
        HandoffSlotHeader h{};
        if (!pread_all(fd_, &h, sizeof h, base) || !slot_header_sane(h) || h.state != kHandoffFree) continue;
        HandoffSlotHeader c{};
        std::memcpy(c.magic, kSlotMagic, 16);
        c.version = kHandoffVersion;
        c.header_bytes = (uint32_t) kHandoffHeaderBytes;
        c.state = kHandoffClaimed;
        c.tier = t;
        c.owner_pid = me_pid();
        c.owner_start = handoff_proc_start_time(me_pid());
        c.nonce = fresh_nonce();
        c.client_id = client_id;
        c.request_id = request_id;
        c.pack_hash = hdr_.pack_hash;
        c.geom_hash = hdr_.geom_hash;
        c.claimed_ms = handoff_now_ms();
        if (!store_(base, &c, sizeof c)) return fail(err, "cannot write slot " + num(i) + "'s claim");
        out.index = (int) i;
        out.base = base;
        out.payload_off = base + kHandoffHeaderBytes;
        out.capacity = cap;
        out.tier = t;
        out.nonce = c.nonce;
        return true;
    }
    return fail(err, "no free handoff slot for a tier-" + num(tier) + " job (" + free_slots_locked_() + " slots free)");
}

bool HandoffArena::write_payload(const HandoffClaim& c, uint64_t offset, const void* data, uint64_t bytes,
                                 std::string& err) {
    if (fd_ < 0 || !writer_) return fail(err, "only the writer writes payloads");
    if (c.index < 0 || c.capacity == 0) return fail(err, "not a claimed slot");
    if (offset > c.capacity || bytes > c.capacity - offset)
        return fail(err, "the write ends at byte " + num(offset + bytes) + ", past the slot's capacity of " +
                             num(c.capacity));
    if (!pwrite_all(fd_, data, bytes, c.payload_off + offset))
        return fail(err, std::string("pwrite into slot ") + num((uint64_t) c.index) + " failed: " + std::strerror(errno));
    return true;
}

bool HandoffArena::publish(const HandoffClaim& c, uint64_t tokens, uint64_t payload_bytes, uint64_t payload_hash,
                           std::string& err) {
    if (fd_ < 0 || !writer_) return fail(err, "only the writer publishes");
    if (payload_bytes > c.capacity)
        return fail(err, "a payload of " + num(payload_bytes) + " bytes does not fit the slot's capacity of " +
                             num(c.capacity));
    Locked lk(*this, true);
    if (!lk.ok) return fail(err, "cannot lock " + path_);
    HandoffSlotHeader h{};
    uint64_t base = 0, cap = 0;
    if (!load_slot_(c.index, h, base, cap) || !slot_header_sane(h) || h.state != kHandoffClaimed ||
        h.nonce != c.nonce || h.owner_pid != me_pid())
        return fail(err, "the claim is gone: slot " + num((uint64_t) c.index) + " is " + state_name(h.state) +
                             " with nonce " + hex16(h.nonce));
    if (h.flags & kHandoffFlagCancelled) return fail(err, "the job in slot " + num((uint64_t) c.index) + " was cancelled");
    uint64_t block[6] = {tokens, payload_bytes, payload_hash, h.claimed_ms, std::max(handoff_now_ms(), h.claimed_ms), 1};
    if (!store_(base + kSlotPublishBlockOffset, block, sizeof block)) return fail(err, "cannot write the publish block");
    std::atomic_thread_fence(std::memory_order_release);
    const uint32_t state_flags[2] = {kHandoffReady, h.flags};
    if (!store_(base + kSlotStateOffset, state_flags, sizeof state_flags)) return fail(err, "cannot write the READY state");
    return true;
}

bool HandoffArena::release(int index, uint64_t nonce, std::string& err) {
    if (fd_ < 0 || !writer_) return fail(err, "only the writer releases a slot");
    Locked lk(*this, true);
    HandoffSlotHeader h{};
    uint64_t base = 0, cap = 0;
    if (!lk.ok || !load_slot_(index, h, base, cap) || !slot_header_sane(h))
        return fail(err, "slot " + num((uint64_t) index) + " cannot be read");
    if (h.state == kHandoffFree || h.nonce != nonce)
        return fail(err, "slot " + num((uint64_t) index) + " is " + state_name(h.state) + " with nonce " + hex16(h.nonce) +
                             ", not " + hex16(nonce));
    return reset_slot_(base, h.tier, 0) || fail(err, "cannot free slot " + num((uint64_t) index));
}

bool HandoffArena::abort_claim(int index, uint64_t nonce, std::string& err) {
    if (fd_ < 0 || !writer_) return fail(err, "only the writer aborts a claim");
    Locked lk(*this, true);
    HandoffSlotHeader h{};
    uint64_t base = 0, cap = 0;
    if (!lk.ok || !load_slot_(index, h, base, cap) || !slot_header_sane(h))
        return fail(err, "slot " + num((uint64_t) index) + " cannot be read");
    if (h.state == kHandoffFree || h.nonce != nonce)
        return fail(err, "slot " + num((uint64_t) index) + " is " + state_name(h.state) + " with nonce " + hex16(h.nonce) +
                             ", not " + hex16(nonce));
    return reset_slot_(base, h.tier, kHandoffFlagPartial) || fail(err, "cannot free slot " + num((uint64_t) index));
}

bool HandoffArena::cancel(int index, uint64_t nonce, std::string& err) {
    if (fd_ < 0 || !writer_) return fail(err, "only the writer cancels a job");
    Locked lk(*this, true);
    HandoffSlotHeader h{};
    uint64_t base = 0, cap = 0;
    if (!lk.ok || !load_slot_(index, h, base, cap) || !slot_header_sane(h))
        return fail(err, "slot " + num((uint64_t) index) + " cannot be read");
    if (h.state != kHandoffClaimed || h.nonce != nonce)
        return fail(err, "slot " + num((uint64_t) index) + " is " + state_name(h.state) + " with nonce " + hex16(h.nonce) +
                             ", not " + hex16(nonce));
    const uint32_t flags = h.flags | kHandoffFlagCancelled;
    return store_(base + kSlotFlagsOffset, &flags, sizeof flags) || fail(err, "cannot flag the cancel");
}

bool HandoffArena::open_reader(const std::string& path, uint64_t pack_hash, uint64_t geom_hash, std::string& err) {
    close_();
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) return fail(err, "cannot open " + path + ": " + std::strerror(errno));
    HandoffArenaHeader h{};
    struct stat st{};
    bool ok = true;
    {
        Locked lk(*this, false);
        if (!lk.ok || !pread_all(fd_, &h, sizeof h, 0)) ok = fail(err, "cannot read the header of " + path);
    }
    if (ok && std::memcmp(h.magic, kArenaMagic, 16) != 0) ok = fail(err, path + " is not a handoff arena (bad magic)");
    else if (ok && h.version != kHandoffVersion)
        ok = fail(err, path + " is arena version " + num(h.version) + "; this build reads version 1");
    else if (ok && h.header_bytes != kHandoffHeaderBytes)
        ok = fail(err, path + " has header_bytes " + num(h.header_bytes) + ", not 4096");
    else if (ok && (::fstat(fd_, &st) != 0 || (uint64_t) st.st_size != h.arena_bytes))
        ok = fail(err, path + " is " + num((uint64_t) st.st_size) + " bytes but its header says " + num(h.arena_bytes));
    else if (ok && (h.tier_count == 0 || h.tier_count > (uint32_t) kHandoffMaxTiers))
        ok = fail(err, path + " has an impossible tier count " + num(h.tier_count));
    else if (ok && h.pack_hash != pack_hash)
        ok = fail(err, "pack hash " + hex16(h.pack_hash) + " of " + path + " differs from this instance's " +
                           hex16(pack_hash));
    else if (ok && h.geom_hash != geom_hash)
        ok = fail(err, "geometry hash " + hex16(h.geom_hash) + " of " + path + " differs from this instance's " +
                           hex16(geom_hash));
    else if (ok) {
        const std::string why = tier_layout_error(h);
        if (!why.empty()) ok = fail(err, path + " has an inconsistent tier table: " + why);
    }
    if (!ok) {
        close_();
        return false;
    }
    hdr_ = h;
    writer_ = false;
    path_ = path;
    return true;
}

bool HandoffArena::read_slot(int index, uint64_t expect_nonce, uint64_t client_id, HandoffPayload& out,
                             std::string& err) {
    out.unbind();
    if (fd_ < 0) return fail(err, "the arena is not open");
    if (writer_) return fail(err, "a writer handle does not read slots; open the arena as a reader");
    HandoffSlotHeader h{};
    uint64_t base = 0, cap = 0;
    {
        Locked lk(*this, false);
        if (!lk.ok || !load_slot_(index, h, base, cap))
            return fail(err, "slot " + std::to_string(index) + " is not in this arena");
    }
    const std::string s = "slot " + std::to_string(index);
    if (!slot_header_sane(h)) return fail(err, s + " has an incompatible header");
    if (h.state != kHandoffReady) return fail(err, s + " is " + state_name(h.state) + ", not READY");
    if (h.client_id != client_id)
        return fail(err, s + " is addressed to client " + num(h.client_id) + ", not " + num(client_id));
    if (h.nonce != expect_nonce) return fail(err, s + " holds nonce " + hex16(h.nonce) + ", not " + hex16(expect_nonce));
    if (h.pack_hash != hdr_.pack_hash)
        return fail(err, s + " was written for pack " + hex16(h.pack_hash) + "; this arena is pack " + hex16(hdr_.pack_hash));
    if (h.geom_hash != hdr_.geom_hash)
        return fail(err, s + " was written for geometry hash " + hex16(h.geom_hash) + "; this arena's is " +
                             hex16(hdr_.geom_hash));
    if (h.seq != 1) return fail(err, s + " carries seq " + num(h.seq) + "; a version-1 payload is one window (seq 1)");
    if (h.payload_bytes > cap)
        return fail(err, s + " declares " + num(h.payload_bytes) + " payload bytes in a " + num(cap) + "-byte slot");
    const uint64_t page = (uint64_t) ::sysconf(_SC_PAGESIZE);
    const uint64_t off = base + kHandoffHeaderBytes;
    struct stat st{};
    if (::fstat(fd_, &st) != 0 || (uint64_t) st.st_size < off + h.payload_bytes)
        return fail(err, "the arena file is shorter than " + s + "'s payload");
    const uint64_t aligned = off & ~(page - 1);
    const uint64_t len = (off - aligned) + std::max<uint64_t>(h.payload_bytes, 1);
    void* map = ::mmap(nullptr, len, PROT_READ, MAP_SHARED, fd_, (off_t) aligned);
    if (map == MAP_FAILED) return fail(err, "cannot map " + s + ": " + std::strerror(errno));
    out.bind_mapping(map, len, static_cast<const uint8_t*>(map) + (off - aligned), h.payload_bytes);
    out.index = index;
    out.tier = h.tier;
    out.nonce = h.nonce;
    out.client_id = h.client_id;
    out.request_id = h.request_id;
    out.tokens = h.tokens;
    out.payload_bytes = h.payload_bytes;
    out.payload_hash = h.payload_hash;
    out.seq = h.seq;
    return true;
}

uint64_t HandoffArena::payload_hash_of(const HandoffPayload& p) {
    return p.valid() ? fnv1a64(p.data, p.payload_bytes) : 0;
}

bool HandoffArena::slot_info(int index, HandoffSlotInfo& out) const {
    if (fd_ < 0) return false;
    HandoffSlotHeader h{};
    uint64_t base = 0, cap = 0;
    {
        Locked lk(*this, false);
        if (!lk.ok || !load_slot_(index, h, base, cap)) return false;
    }
    out = HandoffSlotInfo{};
    out.index = index;
    out.base = base;
    out.capacity = cap;
    out.state = h.state;
    out.flags = h.flags;
    out.tier = h.tier;
    out.owner_pid = h.owner_pid;
    out.owner_start = h.owner_start;
    out.nonce = h.nonce;
    out.client_id = h.client_id;
    out.request_id = h.request_id;
    out.pack_hash = h.pack_hash;
    out.geom_hash = h.geom_hash;
    out.tokens = h.tokens;
    out.payload_bytes = h.payload_bytes;
    out.payload_hash = h.payload_hash;
    out.claimed_ms = h.claimed_ms;
    out.published_ms = h.published_ms;
    out.seq = h.seq;
    return true;
}

std::string HandoffArena::describe() const {
    return "slots " + tier_list(hdr_.tier_slot_count, hdr_.tier_count) + " (tiers " +
           tier_list(hdr_.tier_max_tokens, hdr_.tier_count) + "), max " + num(max_tokens()) + " tokens, arena " +
           gib(hdr_.arena_bytes) + " (" + num(hdr_.arena_bytes) + " B), pack hash " + hex16(hdr_.pack_hash) +
           ", geometry hash " + hex16(hdr_.geom_hash);
}

}  // namespace strata::core
