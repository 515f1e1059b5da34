// tests/cpp/serve_swap_gpu_test.cpp - the reference's serve-slot hand-over driven through this build on a GPU.
//
// The reference's engine swaps conversations in and out of its ONE live session with
// strata::program::serve_swap::run(Plan, Hooks) (include/strata/program/serve_swap.hpp:486-577): drain, validate
// the incoming image, unmount (park) the outgoing branch, mount (restore) the incoming one.  Its hooks are
// generate.cpp's: `unmount` is park_current (src/program/generate.cpp:4185-4266: price the snapshot, take the
// retained K/V for an incremental capture, make room in the ConversationCache, save, put with the owner's claim);
// `validate` is conversation_snapshot_validate; `mount` restores, then hands the mounted K/V to the cache for the
// next incremental park (:5913-5940).  This program writes those hooks against this build's snapshot layer and
// ConversationCache and runs the reference's own serve_swap::run (its header, compiled unchanged) over three
// serve slots in one device session:
//
//   * A, B, C are prefilled in turn (each parked when the next one takes the session);
//   * C -> A, A -> B, B -> A hand-overs: every mount equals its slot's content byte for byte (K/V through the
//     session's page tables, GDN rows, ids, PLE window), the last one from an image captured incrementally (the
//     retained K/V of A's mount reused by A's second park); the steps that ran are the plan's, in order;
//   * a refused mount (an image from another geometry) stops at `validate`: the session is untouched bit for bit,
//     the outgoing branch was not parked, the report says intact and not poisoned;
//   * a mount whose copy launch fails (the library's fault seam; nothing faults on the GPU) is a `restore` fault:
//     the report says the session is poisoned, exactly the reference's rule.
//
// Built by oracle/Makefile (it needs the reference's include tree); run by tests/test_cpp_gpu.py.
#include "session_fixture.hpp"
#include "transfer.hpp"

#include "strata/program/serve_swap.hpp"

#include <memory>
#include <optional>
#include <string>

using namespace strata::core;
using namespace fixture;
namespace sw = strata::program::serve_swap;

namespace {

ModelGeometry small_geometry() {
    ModelGeometry g;
    g.n_layers = 8;
    g.ssm_state_size = 16;
    g.ssm_v_heads = 4;
    g.ssm_conv_channels = 64;
    return g;
}

uint64_t fnv(uint64_t h, const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

/// The one live session of the engine, the slot whose branch it holds, and the park store.
struct Engine {
    DeviceSession& s;
    ConversationCache cache{size_t(1) << 32, ConversationCache::default_slots};
    std::vector<int32_t> live;                 // the mounted branch's ids (empty: nothing mounted)
    int64_t mounted = -1;                      // the slot the session describes
    std::vector<ConversationImageKey> images;  // no image chunks in this workload
    std::vector<ConversationCheckpoint> checks;
    size_t reused_bytes = 0;

    explicit Engine(DeviceSession& session) : s(session) {}

    /// generate.cpp park_current: price, fit, save (reusing the retained K/V when it fits), put with the claim.
    bool park_current(size_t held, int64_t owner, std::string& err) {
        const ConversationView view{live, images, checks, true};
        ConversationKvReuse reuse = cache.take_reuse();
        size_t estimate = 0;
        if (!conversation_snapshot_bytes(view, s.ss, s.g, s.draft, estimate, err)) return false;
        const size_t fresh = estimate;
        if (!reuse.kv.empty() && !conversation_snapshot_capture_bytes(reuse, view, s.ss, s.g, s.draft, estimate, err)) {
            reuse = {};
            estimate = fresh;
            err.clear();
        }
        if (!reuse.kv.empty() && !cache.can_fit(estimate, held)) {
            reuse = {};
            estimate = fresh;
        }
        if (!cache.make_room(estimate, held)) return false;
        SavedConversation image;
        size_t reused = 0;
        if (!conversation_snapshot_save(image, view, s.ss, s.g, s.draft, err, std::move(reuse), &reused)) return false;
        check(image.bytes() <= estimate, "the parked image fits its admitted estimate");
        reused_bytes = reused;
        return cache.put(std::move(image), owner, held);
    }
};

/// Everything a mount writes, read back: K/V of every layer through its slots, the GDN rows, the PLE window.
uint64_t session_fingerprint(const DeviceSession& s) {
    cuda(cudaDeviceSynchronize(), "settle");
    uint64_t h = 1469598103934665603ull;
    for (size_t j = 0; j <= s.qsa.size(); ++j)
        for (int kv = 0; kv < 2; ++kv) {
            const auto b = s.get(j, kv);
            h = fnv(h, b.data(), b.size());
        }
    const size_t row = (size_t) (s.g.ssm_state_size * s.g.ssm_v_heads * s.g.ssm_state_size +
                                 s.g.ssm_conv_channels * (s.g.ssm_d_conv - 1));
    const auto gdn = from_device(s.gdn, (size_t) s.g.n_gdn_layers() * row);
    h = fnv(h, gdn.data(), gdn.size() * 4);
    return fnv(h, s.ss.ple_prev, sizeof s.ss.ple_prev);
}

void check_slot(const Engine& e, const Content& c, const char* what) {
    for (size_t j = 0; j <= e.s.qsa.size(); ++j) {
        check(e.s.get(j, 0) == c.k[j], what);
        check(e.s.get(j, 1) == c.v[j], what);
    }
    check(from_device(e.s.gdn, c.gdn.size()) == c.gdn, what);
    check(e.live == c.ids, what);
    const size_t n = c.ids.size();
    check(e.s.ss.ple_prev[0] == c.ids[n - 2] && e.s.ss.ple_prev[1] == c.ids[n - 1], what);
}

bool ran_in_order(const sw::Report& r, std::initializer_list<sw::Step> want) {
    return std::vector<sw::Step>(want) == r.ran;
}

strata::kv::TransferStep fail_kind = strata::kv::TransferStep::launch;
bool fail_next = false;
bool seam(strata::kv::TransferStep step) {
    if (!fail_next || step != fail_kind) return false;
    fail_next = false;
    return true;
}

}  // namespace

int main() {
    cuda(cudaSetDevice(0), "cudaSetDevice(0)");
    const ModelGeometry g = small_geometry();
    DeviceSession session(g, 900, 96, 21);
    Engine e(session);
    const Content slot_content[3] = {make_content(session, 101), make_content(session, 202), make_content(session, 303)};
    const char* name = "ABC";
    strata::kv::set_transfer_fault_hook(seam);

    // ---- prefill A, B and C in turn; each takes the session from the one before (save only, nothing to mount)
    for (int k = 0; k < 3; ++k) {
        std::string err;
        if (e.mounted >= 0) {
            sw::Plan plan;
            plan.save = true;
            sw::Hooks h;
            h.unmount = [&](std::string& er) { return e.park_current(0, e.mounted, er); };
            const sw::Report r = sw::run(plan, h, err);
            check(r.ok && r.session_intact && ran_in_order(r, {sw::Step::drain_residency, sw::Step::return_loan,
                                                                  sw::Step::unmount}),
                  "the outgoing slot is parked before the next prefill");
        }
        upload(session, slot_content[k]);   // the prefill of slot k writes the session
        cuda(cudaDeviceSynchronize(), "prefill");
        e.live = slot_content[k].ids;
        e.mounted = k;
        session.ss.ple_prev[0] = e.live[e.live.size() - 2];
        session.ss.ple_prev[1] = e.live.back();
    }
    check(e.cache.size() == 2, "A and B are parked, C is live");

    // ---- C -> A, A -> B, B -> A: full hand-overs through serve_swap::run
    auto hand_over = [&](int to, bool expect_reuse) {
        std::string err;
        const auto m = e.cache.best_exact(slot_content[to].ids, e.images, true);
        check(m.tokens == (int64_t) slot_content[to].ids.size() && m.live, "the incoming slot's branch is parked");
        std::optional<SavedConversation> incoming = e.cache.take(m.index);
        const size_t held = incoming->bytes();
        sw::Plan plan;
        plan.save = plan.mount = true;
        sw::Hooks h;
        h.validate = [&](std::string& er) { return conversation_snapshot_validate(*incoming, session.ss, g, session.draft, er); };
        h.unmount = [&](std::string& er) { return e.park_current(held, e.mounted, er); };
        h.mount = [&](std::string& er) {
            if (conversation_snapshot_restore(*incoming, session.ss, g, session.draft, er) != ConversationRestore::restored)
                return false;
            e.live = std::move(incoming->live.ids);
            e.cache.retain(std::move(incoming->kv), (int64_t) e.live.size());
            incoming.reset();
            e.mounted = to;
            return true;
        };
        const sw::Report r = sw::run(plan, h, err);
        check(r.ok && !r.session_intact && !r.session_poisoned, (std::string("hand-over to ") + name[to] + ": " + err).c_str());
        check(ran_in_order(r, {sw::Step::drain_residency, sw::Step::return_loan, sw::Step::validate, sw::Step::unmount,
                               sw::Step::mount}),
              "the steps ran in the reference's order");
        check_slot(e, slot_content[to], "the mounted slot equals its content byte for byte");
        check(!expect_reuse || e.reused_bytes > 0, "the outgoing park reused the retained K/V of its mount");
        check(e.cache.retained_bytes() > 0, "the mounted K/V is retained for the next incremental park");
    };
    hand_over(0, false);   // C -> A (C's park is a fresh capture: C was prefilled, not mounted)
    hand_over(1, true);    // A -> B (A's park reuses the K/V retained from A's mount)
    hand_over(0, true);    // B -> A (A's image is the incrementally captured one)
    std::printf("A/B/A: three hand-overs through serve_swap::run, every mount exact; incremental park reused %zu bytes\n",
                e.reused_bytes);

    // ---- a refused mount: an image from another geometry stops at `validate`, the session untouched
    {
        std::string err;
        const auto m = e.cache.best_exact(slot_content[1].ids, e.images, true);
        check(m.tokens > 0, "B is parked");
        SavedConversation bad = e.cache.take(m.index);
        bad.geometry[0] += 1;
        const uint64_t before = session_fingerprint(session);
        const size_t parked_before = e.cache.size();
        sw::Plan plan;
        plan.save = plan.mount = true;
        sw::Hooks h;
        bool unmounted = false, mounted = false;
        h.validate = [&](std::string& er) { return conversation_snapshot_validate(bad, session.ss, g, session.draft, er); };
        h.unmount = [&](std::string& er) { unmounted = true; return e.park_current(bad.bytes(), e.mounted, er); };
        h.mount = [&](std::string&) { mounted = true; return false; };
        const sw::Report r = sw::run(plan, h, err);
        check(!r.ok && r.fault == sw::Fault::validation && r.failed_at == sw::Step::validate, "the refusal is a validation fault");
        check(r.session_intact && !r.session_poisoned && sw::fault_is_recoverable(r.fault), "the session is intact");
        check(!unmounted && !mounted && e.cache.size() == parked_before, "nothing was parked or mounted");
        check(session_fingerprint(session) == before, "the live session is untouched, bit for bit");
        check_slot(e, slot_content[0], "and still holds slot A");
    }

    // ---- a mount whose copy launch fails after validation: a restore fault poisons the session
    {
        std::string err;
        const auto m = e.cache.best_exact(slot_content[2].ids, e.images, true);
        check(m.tokens > 0, "C is parked");
        SavedConversation incoming = e.cache.take(m.index);
        sw::Plan plan;
        plan.mount = true;
        sw::Hooks h;
        h.validate = [&](std::string& er) { return conversation_snapshot_validate(incoming, session.ss, g, session.draft, er); };
        h.mount = [&](std::string& er) {
            fail_next = true;
            const ConversationRestore res = conversation_snapshot_restore(incoming, session.ss, g, session.draft, er);
            fail_next = false;
            return res == ConversationRestore::restored;
        };
        const sw::Report r = sw::run(plan, h, err);
        check(!r.ok && r.fault == sw::Fault::restore && r.failed_at == sw::Step::mount, "a failed restore is a restore fault");
        check(r.session_poisoned && !r.session_intact, "and the session may not be decoded from");
    }
    strata::kv::set_transfer_fault_hook(nullptr);
    std::printf("serve_swap_gpu_test: %d checks passed\n", checks);
    return 0;
}
