// tests/cpp/arena_threads_cpu_test.cpp - one hand-off arena shared by threads, under ThreadSanitizer (host only).
//
// An engine may run its hand-off work on several threads against one HandoffArena handle, for example the
// request loop claiming and publishing while a copy-out thread releases acknowledged slots.  Every decision
// takes the handle's process mutex and the file's flock.  Here four threads share one writer handle and one
// reader handle.  Each thread loops: note its client pid, claim a slot, write a payload, publish it, read it
// back through the reader and check its hash, look at the slot, release it.  At the end every slot must be free
// and no read may have failed.  ThreadSanitizer stops the program at the first data race.
//
// Usage: arena_threads_cpu_test <directory>   (exit 0 = pass)
#include "strata_kv/handoff.hpp"

#include <atomic>
#include <cstdio>
#include <string>
#include <thread>
#include <vector>

using namespace strata::core;

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string dir = argv[1];
    std::string err;
    HandoffSizing sizing;
    if (!handoff_size_arena({{1024, 6}, {4096, 2}}, std::vector<uint64_t>{8192, 16384}, sizing, err)) {
        std::fprintf(stderr, "FAIL: sizing: %s\n", err.c_str());
        return 1;
    }
    HandoffArena writer, reader;
    if (!writer.open_writer(dir + "/arena", sizing, 1, 2, err) || !reader.open_reader(dir + "/arena", 1, 2, err)) {
        std::fprintf(stderr, "FAIL: open: %s\n", err.c_str());
        return 1;
    }
    constexpr int kThreads = 4, kRounds = 300;
    std::atomic<int> cycles{0}, failures{0};
    std::vector<std::thread> threads;
    for (int t = 0; t < kThreads; ++t)
        threads.emplace_back([&, t] {
            const uint64_t client = 100 + (uint64_t) t;
            std::vector<uint8_t> payload(5000 + 100 * (size_t) t, (uint8_t) (t + 1));
            const uint64_t hash = fnv1a64(payload.data(), payload.size());
            for (int i = 0; i < kRounds; ++i) {
                std::string e;
                HandoffClaim c;
                writer.note_client_pid(client, 1);
                if (!writer.claim((uint32_t) (i % 2), client, (uint64_t) i, c, e)) continue;   // the tier is full
                bool ok = writer.write_payload(c, 0, payload.data(), payload.size(), e) &&
                          writer.publish(c, 10, payload.size(), hash, e);
                HandoffPayload p;
                ok = ok && reader.read_slot(c.index, c.nonce, client, p, e) && HandoffArena::payload_hash_of(p) == hash;
                p.unbind();
                HandoffSlotInfo info;
                ok = ok && writer.slot_info(c.index, info) && info.state == kHandoffReady;
                ok = writer.release(c.index, c.nonce, e) && ok;
                if (!ok) {
                    ++failures;
                    std::fprintf(stderr, "FAIL: thread %d round %d: %s\n", t, i, e.c_str());
                }
                ++cycles;
            }
        });
    for (auto& th : threads) th.join();
    const std::string free_slots = writer.free_slots();
    const bool all_free = free_slots == "8/8";
    if (!all_free) std::fprintf(stderr, "FAIL: free slots at the end: %s\n", free_slots.c_str());
    std::printf("arena_threads_cpu_test: %d claim-publish-read-release cycles on %d threads, free %s, %s\n",
                cycles.load(), kThreads, free_slots.c_str(), failures || !all_free || cycles == 0 ? "FAILED" : "OK");
    return failures || !all_free || cycles == 0 ? 1 : 0;
}
