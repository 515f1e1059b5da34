// tests/cpp/wire_fuzz_cpu_test.cpp - the SR4H decoders against damaged payloads, under AddressSanitizer and
// UndefinedBehaviorSanitizer (host only).
//
// A payload can arrive from another process or another machine, so every decoder must refuse a damaged one
// without reading or writing out of bounds.  Starting from payloads the reference itself wrote (tests/golden), each
// round damages one copy - random bytes flipped, a 64-bit field of the header or the record stream replaced by an
// extreme value, the payload cut short or padded - and runs the full decoder (conversation_wire_decode) and the
// shape decoder the device mount uses (wire_detail::decode_shape).  Either may accept or refuse; neither may
// fault, and the sanitizers stop the program at the first bad access.  Two checks pin the harness: the undamaged
// payloads decode, and a payload one byte short is refused.
//
// Usage: wire_fuzz_cpu_test <rounds per payload> <payload.bin>...   (exit 0 = pass)
#include "strata_kv/conversation_wire.hpp"
#include "wire_detail.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>
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

std::vector<uint8_t> load(const char* path) {
    std::ifstream f(path, std::ios::binary);
    return std::vector<uint8_t>(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
}

/// Both decoders on one candidate payload; returns how many accepted it.
int decode_both(const std::vector<uint8_t>& p) {
    int accepted = 0;
    std::string error;
    {
        SavedConversation image;
        WireDecoded info;
        if (conversation_wire_decode(p.data(), p.size(), image, info, WireExpect{}, error)) ++accepted;
    }
    {
        SpanWireSource source(p.data(), p.size());
        SavedConversation image;
        WireDecoded info;
        wire_detail::BlobTable blobs;
        if (wire_detail::decode_shape(source, image, info, WireExpect{}, blobs, error)) {
            ++accepted;
            // every blob the shape decoder hands to the device mount lies inside the payload
            for (const auto& [key, at] : blobs)
                check(at.off <= p.size() && at.bytes <= p.size() - at.off, "a shape blob lies inside the payload");
        }
    }
    return accepted;
}

/// The end of the header and record stream (where the blob pool starts), clamped to the payload.
uint64_t records_end(const std::vector<uint8_t>& p) {
    WireHeaderRecord h;
    std::string error;
    if (!conversation_wire_peek(p.data(), p.size(), h, error)) return std::min<uint64_t>(p.size(), 256);
    return std::min<uint64_t>(p.size(), std::max<uint64_t>(h.blob_pool_off, 256));
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    const int rounds = std::atoi(argv[1]);
    std::mt19937_64 rng(0x5eed5eedull);
    int accepted_damaged = 0, refused_damaged = 0;
    for (int a = 2; a < argc; ++a) {
        const std::vector<uint8_t> clean = load(argv[a]);
        check(clean.size() >= 256, std::string("payload read: ") + argv[a]);
        if (clean.size() < 256) continue;
        check(decode_both(clean) == 2, std::string("the undamaged payload decodes both ways: ") + argv[a]);
        std::vector<uint8_t> short_one(clean.begin(), clean.end() - 1);
        check(decode_both(short_one) == 0, "a payload one byte short is refused both ways");
        const uint64_t rec_end = records_end(clean);
        static const uint64_t extremes[] = {0, 1, 2, 3, 0xffffffffull, 0x80000000ull, 0x7fffffffffffffffull,
                                            0x8000000000000000ull, ~0ull, ~0ull - 255, 1ull << 40, 4096, 65536};
        for (int r = 0; r < rounds; ++r) {
            std::vector<uint8_t> p = clean;
            switch (rng() % 4) {
                case 0: {   // flip a few bytes, mostly in the header and records
                    const int n = 1 + (int) (rng() % 8);
                    for (int i = 0; i < n; ++i) {
                        const uint64_t span = rng() % 5 ? rec_end : p.size();
                        p[rng() % span] ^= (uint8_t) (1u + rng() % 255u);
                    }
                    break;
                }
                case 1: {   // one 8-byte field of the header or the records set to an extreme value
                    const uint64_t at = (rng() % (rec_end / 8)) * 8;
                    uint64_t v = extremes[rng() % (sizeof extremes / sizeof extremes[0])];
                    if (rng() % 3 == 0) v = p.size() + (rng() % 512) - 256;
                    std::memcpy(p.data() + at, &v, std::min<uint64_t>(8, p.size() - at));
                    break;
                }
                case 2:     // cut short anywhere
                    p.resize(rng() % p.size());
                    break;
                default: {  // padded with junk, or a 32-bit field set to an extreme value
                    if (rng() % 2) {
                        const size_t extra = 1 + rng() % 4096;
                        for (size_t i = 0; i < extra; ++i) p.push_back((uint8_t) rng());
                    } else {
                        const uint64_t at = (rng() % (rec_end / 4)) * 4;
                        const uint32_t v = (uint32_t) extremes[rng() % (sizeof extremes / sizeof extremes[0])];
                        std::memcpy(p.data() + at, &v, 4);
                    }
                }
            }
            if (p == clean) continue;
            (decode_both(p) ? accepted_damaged : refused_damaged) += 1;
        }
    }
    check(refused_damaged > 0, "damaged payloads are refused");
    std::printf("wire_fuzz_cpu_test: %d damaged payloads refused, %d accepted (the damage left a well-formed payload: "
                "blob bytes, token ids, trailing bytes), %d checks, %s\n",
                refused_damaged, accepted_damaged, checks, failures ? "FAILED" : "OK");
    return failures ? 1 : 0;
}
