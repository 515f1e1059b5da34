// tests/cpp/transfer_faults_gpu_test.cpp - host-side transfer failures injected into the drop-in's park and mount.
//
// The reference runs its real restore under a link-wrapped cudaMemcpy / cudaDeviceSynchronize that fail on the Nth
// call (src/core/conversation_validation_test.cpp:15-33) and checks what each failure leaves behind: a failure
// before the first write refuses with nothing changed, one after it is transfer_failed with partial state, never a
// fall-back to "invalid image" (:171-195 for one session, :475-500 for a layer split).  This build moves the bytes
// in batches (host copies into a staging image, one copy-kernel launch, one stream synchronisation per device), so
// the same questions are asked of ITS host-side steps through the library's fault seam
// (strata::kv::set_transfer_fault_hook): every device synchronisation, host copy, copy-kernel launch and stream
// synchronisation of a park or a mount is failed, one at a time, in the order the call issues them.  Nothing faults
// on the GPU: a failed copy or launch is one the host never issues; a failed synchronisation completed and then
// reports an error.
//
//   mount, one session: for every step k of a clean mount, failing step k gives transfer_failed; when step k comes
//     at or before the first copy-kernel launch the session is unchanged bit for bit (the earlier steps only filled
//     the staging image), after it the session has been written.  An unhooked mount then restores every byte.
//   park: failing any step of a clean park refuses it and leaves the caller's image exactly as it was; a clean park
//     afterwards equals the first byte for byte (no copy of a failed park still lands in recycled pinned memory).
//   mount, a two-carve layer split on one device: failing the first device synchronisation writes nothing to either
//     carve; failing the later stage's launch, its stream synchronisation or the last device synchronisation is
//     transfer_failed after writes; an unhooked mount restores both carves.
//
// Usage: transfer_faults_gpu_test   (exit 0 = pass)
#include "session_fixture.hpp"
#include "transfer.hpp"

#include <string>

using namespace strata::core;
using namespace fixture;
using strata::kv::TransferStep;

namespace {

struct Injector {
    int fail_at = 0;                 // 1-based step to fail (0: none)
    std::vector<TransferStep> seen;  // every step asked since arm()
} inj;

bool hook(TransferStep step) {
    inj.seen.push_back(step);
    return (int) inj.seen.size() == inj.fail_at;
}
void arm(int fail_at) {
    inj.fail_at = fail_at;
    inj.seen.clear();
}
int first_of(const std::vector<TransferStep>& steps, TransferStep kind) {
    for (size_t i = 0; i < steps.size(); ++i)
        if (steps[i] == kind) return (int) i + 1;
    return 0;
}
int last_of(const std::vector<TransferStep>& steps, TransferStep kind) {
    for (size_t i = steps.size(); i-- > 0;)
        if (steps[i] == kind) return (int) i + 1;
    return 0;
}

uint64_t fnv(uint64_t h, const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

ModelGeometry small_geometry() {
    ModelGeometry g;
    g.n_layers = 8;   // QSA layers 3 and 7, GDN layers 0-2 and 4-6
    g.ssm_state_size = 16;
    g.ssm_v_heads = 4;
    g.ssm_conv_channels = 64;
    return g;
}
size_t gdn_row_floats(const ModelGeometry& g) {
    return (size_t) (g.ssm_state_size * g.ssm_v_heads * g.ssm_state_size + g.ssm_conv_channels * (g.ssm_d_conv - 1));
}

/// Every byte a mount writes: each layer's K and V through its slots, each QSA layer's indexer buffers, the GDN rows
/// and the PLE window.
uint64_t fingerprint(const DeviceSession& s) {
    cuda(cudaDeviceSynchronize(), "settle");
    uint64_t h = 1469598103934665603ull;
    for (size_t j = 0; j <= s.qsa.size(); ++j)
        for (int kv = 0; kv < 2; ++kv) {
            const auto bytes = s.get(j, kv);
            h = fnv(h, bytes.data(), bytes.size());
        }
    for (const QsaState& st : s.qsa) {
        const auto pooled = from_device(st.idx_pooled, (size_t) st.idx_pooled_rows * (size_t) s.g.idx_key_dim);
        const auto tail = from_device(st.idx_tail, 3 * (size_t) s.g.idx_key_dim);
        const auto dead = from_device(st.idx_dead, (size_t) s.g.idx_key_dim);
        const auto pos = from_device(st.idx_block_pos, 1);
        h = fnv(fnv(fnv(fnv(h, pooled.data(), pooled.size() * 4), tail.data(), tail.size() * 4), dead.data(), dead.size() * 4),
                pos.data(), 4);
    }
    const auto gdn = from_device(s.gdn, (size_t) s.g.n_gdn_layers() * gdn_row_floats(s.g));
    h = fnv(h, gdn.data(), gdn.size() * 4);
    return fnv(h, s.ss.ple_prev, sizeof s.ss.ple_prev);
}

/// Overwrite everything a mount writes with a pattern the image never holds.
void scribble(DeviceSession& s) {
    cuda(cudaMemset(s.base, 0x31, (size_t) s.pool_blocks * kSlotPages * (size_t) s.page_bytes), "pool scribbled");
    for (const QsaState& st : s.qsa) {
        cuda(cudaMemset(st.idx_pooled, 0x31, (size_t) st.idx_pooled_rows * (size_t) s.g.idx_key_dim * 4), "pooled");
        cuda(cudaMemset(st.idx_tail, 0x31, 3 * (size_t) s.g.idx_key_dim * 4), "tail");
        cuda(cudaMemset(st.idx_dead, 0x31, (size_t) s.g.idx_key_dim * 4), "dead");
        cuda(cudaMemset(st.idx_block_pos, 0x31, 4), "block_pos");
    }
    cuda(cudaMemset(s.gdn, 0x31, (size_t) s.g.n_gdn_layers() * gdn_row_floats(s.g) * 4), "gdn");
    s.ss.ple_prev[0] = s.ss.ple_prev[1] = -7;
    cuda(cudaDeviceSynchronize(), "scribbled");
}

/// Every host byte of an image (K/V of every layer, the live running state, the ids, stage parts).
uint64_t digest(const SavedConversation& im) {
    uint64_t h = 1469598103934665603ull;
    auto feed_cp = [&](const ConversationCheckpoint& c) {
        h = fnv(h, c.ids.data(), c.ids.size() * 4);
        for (const auto* v : {&c.gdn, &c.ple, &c.tails, &c.dead, &c.block_pos}) h = fnv(h, v->data(), v->size());
    };
    auto feed_kv = [&](const std::vector<ConversationKv>& kv) {
        for (const ConversationKv& l : kv)
            for (const ConversationBuffer* b : {&l.k, &l.v, &l.k_scale, &l.v_scale, &l.pooled}) {
                const auto bytes = read_buffer(*b);
                h = fnv(h, bytes.data(), bytes.size());
            }
    };
    feed_cp(im.live);
    feed_kv(im.kv);
    for (const auto& part : im.stage_parts) {
        feed_cp(part.state);
        feed_kv(part.kv);
    }
    return h;
}

void check_content(const DeviceSession& s, const Content& c, const char* what) {
    for (size_t j = 0; j <= s.qsa.size(); ++j) {
        check(s.get(j, 0) == c.k[j], what);
        check(s.get(j, 1) == c.v[j], what);
    }
    check(from_device(s.gdn, c.gdn.size()) == c.gdn, what);
    const size_t n = c.ids.size();
    check(s.ss.ple_prev[0] == c.ids[n - 2] && s.ss.ple_prev[1] == c.ids[n - 1], what);
}

}  // namespace

int main() {
    cuda(cudaSetDevice(0), "cudaSetDevice(0)");
    const ModelGeometry g = small_geometry();
    const int64_t T = 700;   // 3 blocks of 256 tokens, the last one partial
    DeviceSession a(g, T, 64, 5);
    const Content content = make_content(a, 9);
    upload(a, content);
    cuda(cudaDeviceSynchronize(), "upload");
    const std::vector<ConversationImageKey> images;
    const std::vector<ConversationCheckpoint> checkpoints;
    const ConversationView view{content.ids, images, checkpoints, true};
    std::string err;
    strata::kv::set_transfer_fault_hook(hook);

    // ---- park: a clean one, its steps, then each step failed on its own
    arm(0);
    SavedConversation image;
    check_ok(conversation_snapshot_save(image, view, a.ss, g, a.draft, err), err, "clean park");
    const std::vector<TransferStep> park_steps = inj.seen;
    check(first_of(park_steps, TransferStep::launch) && first_of(park_steps, TransferStep::copy) &&
              first_of(park_steps, TransferStep::stream_sync),
          "a park launches, copies and synchronises through the seam");
    const uint64_t image_digest = digest(image);
    SavedConversation kept;
    check_ok(conversation_snapshot_save(kept, view, a.ss, g, a.draft, err), err, "second clean park");
    const uint64_t kept_digest = digest(kept);
    check(kept_digest == image_digest, "two clean parks agree");
    for (int k = 1; k <= (int) park_steps.size(); ++k) {
        arm(k);
        err.clear();
        check(!conversation_snapshot_save(kept, view, a.ss, g, a.draft, err), "a park whose step failed is refused");
        check(!err.empty(), "and says why");
        arm(0);
        check(digest(kept) == kept_digest, "a refused park leaves the caller's image as it was");
    }
    arm(0);
    SavedConversation again;
    check_ok(conversation_snapshot_save(again, view, a.ss, g, a.draft, err), err, "clean park after the failed ones");
    check(digest(again) == image_digest, "a clean park after failed ones equals the first, byte for byte");
    std::printf("park: %zu steps, each failed once: refused, the caller's image untouched\n", park_steps.size());

    // ---- mount: a clean one, its steps, then each step failed on its own
    scribble(a);
    arm(0);
    check(conversation_snapshot_restore(image, a.ss, g, a.draft, err) == ConversationRestore::restored, "clean mount");
    const std::vector<TransferStep> mount_steps = inj.seen;
    check_content(a, content, "a clean mount restores every byte and the PLE window");
    const int first_launch = first_of(mount_steps, TransferStep::launch);
    check(mount_steps.front() == TransferStep::device_sync && first_launch > 1,
          "a mount synchronises the device first and launches after its host copies");
    int unchanged = 0, partial = 0;
    for (int k = 1; k <= (int) mount_steps.size(); ++k) {
        scribble(a);
        const uint64_t before = fingerprint(a);
        arm(k);
        err.clear();
        const ConversationRestore r = conversation_snapshot_restore(image, a.ss, g, a.draft, err);
        const size_t asked = inj.seen.size();
        arm(0);
        check(r == ConversationRestore::transfer_failed, "a failed mount step is fatal, never an invalid-image refusal");
        check(!err.empty(), "and the error says why");
        const bool same = fingerprint(a) == before;
        if (k <= first_launch) {
            check(same, "a failure at or before the first launch changed nothing");
            ++unchanged;
        } else {
            check(!same, "a failure after the first launch left partial state");
            ++partial;
        }
        if (k == 1) check(asked == 1, "nothing is issued after a failed first synchronisation");
    }
    scribble(a);
    check(conversation_snapshot_restore(image, a.ss, g, a.draft, err) == ConversationRestore::restored,
          "an unhooked mount after the failed ones");
    check_content(a, content, "and it restores every byte");
    std::printf("mount: %zu steps, each failed once: transfer_failed; %d with nothing changed, %d after writes\n",
                mount_steps.size(), unchanged, partial);

    // ---- a two-carve layer split of the same session on one device
    const size_t row = gdn_row_floats(g);
    SessionState head = a.ss, tail = a.ss;
    head.layer_lo = 0;
    head.layer_hi = 4;
    head.qsa_ord0 = 0;
    head.qsa_alloc = 1;
    head.gdn_alloc = 3;
    tail.layer_lo = 4;
    tail.layer_hi = 8;
    tail.qsa_ord0 = 1;
    tail.qsa_alloc = 1;
    tail.gdn_alloc = 3;
    tail.gdn_state = a.gdn + 3 * row;
    const ConversationStage later{&tail, 0};
    const ConversationStageSet stages{&later, 1, 0, 0};
    SavedConversation split;
    check_ok(conversation_snapshot_save(split, view, head, stages, g, a.draft, err), err, "split park");
    check(split.stage_parts.size() == 1, "one part for the later stage");
    auto sync_both = [&] { a.ss.ple_prev[0] = head.ple_prev[0], a.ss.ple_prev[1] = head.ple_prev[1]; };
    scribble(a);
    head.ple_prev[0] = head.ple_prev[1] = -7;
    arm(0);
    check(conversation_snapshot_restore(split, head, stages, g, a.draft, err) == ConversationRestore::restored,
          "clean split mount");
    const std::vector<TransferStep> split_steps = inj.seen;
    sync_both();
    check_content(a, content, "a clean split mount restores both carves");
    struct Case {
        int step;
        bool writes;
        const char* what;
    };
    const Case cases[] = {{1, false, "split: a failed first synchronisation wrote nothing to either carve"},
                          {last_of(split_steps, TransferStep::launch), true, "split: the later stage's launch failed"},
                          {last_of(split_steps, TransferStep::stream_sync), true, "split: the later stage's stream sync failed"},
                          {last_of(split_steps, TransferStep::device_sync), true, "split: the last device sync failed"}};
    for (const Case& c : cases) {
        scribble(a);
        head.ple_prev[0] = head.ple_prev[1] = -7;
        sync_both();
        const uint64_t before = fingerprint(a);
        arm(c.step);
        const ConversationRestore r = conversation_snapshot_restore(split, head, stages, g, a.draft, err);
        arm(0);
        check(c.step > 0 && r == ConversationRestore::transfer_failed, c.what);
        sync_both();
        check((fingerprint(a) == before) == !c.writes, c.what);
    }
    scribble(a);
    check(conversation_snapshot_restore(split, head, stages, g, a.draft, err) == ConversationRestore::restored,
          "an unhooked split mount after the failed ones");
    sync_both();
    check_content(a, content, "and it restores both carves");
    strata::kv::set_transfer_fault_hook(nullptr);
    std::printf("split mount: %zu steps; failures before and after the writes behave as for one session\n",
                split_steps.size());
    std::printf("transfer_faults_gpu_test: %d checks passed\n", checks);
    return 0;
}
