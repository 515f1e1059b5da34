// tests/cpp/arena_fuzz_cpu_test.cpp - a hand-off arena reader against damaged arena files, under AddressSanitizer
// and UndefinedBehaviorSanitizer (host only).
//
// A decode instance maps an arena file that another process writes, so its reader must refuse a damaged file
// without touching memory outside what it mapped.  The program writes a real arena (two tiers, one READY slot),
// copies it to a second file, and in each round damages that copy - random bytes of the arena header or of a slot
// header flipped, one 64-bit field set to an extreme value, the file cut short (also inside a slot with the header's
// size agreeing) or lengthened - then opens it as a reader and reads every slot index (and two outside the
// table), hashing each payload it is given, then re-opens it as a writer would after a restart and claims, publishes
// and releases a slot of each tier.  Every step may refuse; none may fault (a payload mapped past the end of the
// file would raise SIGBUS and stop the run).
// Two checks pin the harness: the undamaged copy opens and its slot reads back with the writer's hash.
//
// Usage: arena_fuzz_cpu_test <directory> <rounds>   (exit 0 = pass)
#include "strata_kv/handoff.hpp"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

using namespace strata::core;

namespace {

int checks = 0, failures = 0;

void check(bool ok, const std::string& what) {
    ++checks;
    if (!ok) {
        ++failures;
        std::fprintf(stderr, "FAIL: %s\n", what.c_str());
    }
}

std::vector<uint8_t> read_range(const std::string& path, uint64_t off, uint64_t n) {
    std::vector<uint8_t> b(n);
    const int fd = ::open(path.c_str(), O_RDONLY);
    const ssize_t got = ::pread(fd, b.data(), n, (off_t) off);
    ::close(fd);
    b.resize(got > 0 ? (size_t) got : 0);
    return b;
}

void write_range(const std::string& path, uint64_t off, const std::vector<uint8_t>& b) {
    const int fd = ::open(path.c_str(), O_WRONLY);
    if (::pwrite(fd, b.data(), b.size(), (off_t) off) != (ssize_t) b.size()) std::abort();
    ::close(fd);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    const std::string dir = argv[1];
    const int rounds = std::atoi(argv[2]);
    constexpr uint64_t kPack = 0x1234, kGeom = 0x5678, kClient = 9;
    std::string err;

    // a real arena: two tiers, one slot published for kClient
    HandoffSizing sizing;
    check(handoff_size_arena({{1024, 2}, {4096, 1}}, std::vector<uint64_t>{8192, 16384}, sizing, err), "sized: " + err);
    HandoffArena writer;
    const std::string path = dir + "/arena", copy = dir + "/damaged";
    check(writer.open_writer(path, sizing, kPack, kGeom, err), "writer opens: " + err);
    HandoffClaim claim;
    check(writer.claim(1, kClient, 1, claim, err), "claimed: " + err);
    std::vector<uint8_t> payload(12000);
    for (size_t i = 0; i < payload.size(); ++i) payload[i] = (uint8_t) (i * 131 + 7);
    check(writer.write_payload(claim, 0, payload.data(), payload.size(), err), "payload written: " + err);
    const uint64_t hash = fnv1a64(payload.data(), payload.size());
    check(writer.publish(claim, 3000, payload.size(), hash, err), "published: " + err);
    if (failures) return 1;

    // the regions a reader parses: the arena header and every slot header
    struct stat st{};
    ::stat(path.c_str(), &st);
    const uint64_t file_bytes = (uint64_t) st.st_size;
    std::vector<uint64_t> headers = {0};
    for (size_t t = 0; t < sizing.tiers.size(); ++t)
        for (uint64_t k = 0; k < sizing.tiers[t].slot_count; ++k)
            headers.push_back(sizing.slot_off[t] + k * (kHandoffHeaderBytes + sizing.slot_bytes[t]));
    std::vector<std::vector<uint8_t>> pristine;
    for (uint64_t h : headers) pristine.push_back(read_range(path, h, kHandoffHeaderBytes));
    {
        const std::vector<uint8_t> all = read_range(path, 0, file_bytes);
        const int fd = ::open(copy.c_str(), O_CREAT | O_TRUNC | O_WRONLY, 0600);
        if (::write(fd, all.data(), all.size()) != (ssize_t) all.size()) std::abort();
        ::close(fd);
    }
    auto restore = [&]() {
        if (::truncate(copy.c_str(), (off_t) file_bytes) != 0) std::abort();
        for (size_t i = 0; i < headers.size(); ++i) write_range(copy, headers[i], pristine[i]);
    };
    auto read_all = [&](int& served) {
        HandoffArena reader;
        std::string e;
        if (!reader.open_reader(copy, kPack, kGeom, e)) return false;
        const int n = (int) sizing.tiers.size() + 2;
        for (int idx = -1; idx <= n + 1; ++idx) {
            HandoffSlotInfo info;
            (void) reader.slot_info(idx, info);
            HandoffPayload p;
            if (reader.read_slot(idx, claim.nonce, kClient, p, e)) {
                (void) HandoffArena::payload_hash_of(p);   // touches every byte it was given
                ++served;
            }
        }
        return true;
    };

    int served = 0;
    check(read_all(served) && served == 1, "the undamaged copy opens and serves its one READY slot");
    {
        HandoffArena reader;
        HandoffPayload p;
        check(reader.open_reader(copy, kPack, kGeom, err) && reader.read_slot(claim.index, claim.nonce, kClient, p, err) &&
                  HandoffArena::payload_hash_of(p) == hash,
              "and the payload reads back with the writer's hash");
    }

    std::mt19937_64 rng(0xa7e4a5eedull);
    static const uint64_t extremes[] = {0, 1, 4096, 4095, 0xffffffffull, 0x7fffffffffffffffull, ~0ull,
                                        ~0ull - 4095, 1ull << 40, 1ull << 62};
    int opened = 0, refused = 0, rewritten = 0;
    for (int r = 0; r < rounds; ++r) {
        restore();
        const size_t which = rng() % headers.size();
        switch (rng() % 5) {
            case 0: {   // flip bytes of one header
                std::vector<uint8_t> h = pristine[which];
                const int n = 1 + (int) (rng() % 6);
                for (int i = 0; i < n; ++i) h[rng() % 512] ^= (uint8_t) (1u + rng() % 255u);
                write_range(copy, headers[which], h);
                break;
            }
            case 1: {   // one 64-bit field of one header set to an extreme value (or near the file size)
                std::vector<uint8_t> h = pristine[which];
                uint64_t v = extremes[rng() % (sizeof extremes / sizeof extremes[0])];
                if (rng() % 3 == 0) v = file_bytes + (rng() % 8192) - 4096;
                std::memcpy(h.data() + (rng() % 64) * 8, &v, 8);
                write_range(copy, headers[which], h);
                break;
            }
            case 2:     // cut short
                if (::truncate(copy.c_str(), (off_t) (rng() % file_bytes)) != 0) std::abort();
                break;
            case 3: {   // cut short inside or just past a slot, with the header's arena_bytes agreeing (so the size
                        // check alone passes)
                const uint64_t slot = headers[1 + rng() % (headers.size() - 1)];
                const uint64_t to = std::min<uint64_t>(file_bytes - 1, slot + rng() % (2 * kHandoffHeaderBytes + 16384));
                if (::truncate(copy.c_str(), (off_t) to) != 0) std::abort();
                std::vector<uint8_t> h = pristine[0];
                std::memcpy(h.data() + offsetof(HandoffArenaHeader, arena_bytes), &to, 8);
                write_range(copy, 0, h);
                break;
            }
            default:    // lengthened
                if (::truncate(copy.c_str(), (off_t) (file_bytes + 1 + rng() % (1u << 20))) != 0) std::abort();
        }
        int s = 0;
        (read_all(s) ? opened : refused) += 1;
        // a writer re-opening the damaged file (an instance restarting on it): refused, or it reclaims and serves
        {
            HandoffArena w2;
            std::string e;
            if (w2.open_writer(copy, sizing, kPack, kGeom, e, /*allow_existing_writer=*/true)) {
                (void) w2.reclaim(&e);
                (void) w2.free_slots(&e);
                for (uint32_t tier = 0; tier < (uint32_t) sizing.tiers.size(); ++tier) {
                    HandoffClaim c;
                    if (w2.claim(tier, kClient, 77, c, e)) {
                        (void) w2.write_payload(c, 0, payload.data(), 100, e);
                        (void) w2.publish(c, 1, 100, fnv1a64(payload.data(), 100), e);
                        (void) w2.release(c.index, c.nonce, e);
                    }
                }
                ++rewritten;
            }
        }
    }
    check(refused > 0, "damaged arenas are refused");
    std::printf("arena_fuzz_cpu_test: %d damaged arenas refused at open, %d opened (their slots read or refused one by "
                "one), %d re-opened by a writer, %d checks, %s\n",
                refused, opened, rewritten, checks, failures ? "FAILED" : "OK");
    return failures ? 1 : 0;
}
