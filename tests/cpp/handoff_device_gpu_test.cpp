// tests/cpp/handoff_device_gpu_test.cpp - the split-role hand-off across two processes and two GPUs, with only a
// device descriptor in the hand-off slot.
//
// The process forks BEFORE any CUDA call.  The parent is the prefill instance on GPU 0: it places config 1 into a
// pool at seed-random slots, creates the hand-off arena, claims a slot, packs the session into a device buffer
// it exported through CUDA IPC (handoff_device_publish), and sends DONE <slot> <nonce> down a pipe.  The child is
// the decode instance on GPU 1: it opens the arena as a reader, reads the slot (nonce, client, pack and geometry
// checked), imports the handle, mounts straight from GPU 0's HBM into its own differently permuted pool
// (handoff_device_mount), checks every byte against the oracle's content, and sends ACK <nonce>; the parent then
// releases the slot.  Every wait is bounded (poll with a deadline).
//
// Usage: handoff_device_gpu_test <directory for the arena> [tokens]   (exit 0 = pass, 77 = fewer than two GPUs)
#include "session_fixture.hpp"
#include "strata_kv/handoff_device.hpp"

#include <poll.h>
#include <sys/wait.h>
#include <unistd.h>

#include <string>

using namespace strata::core;
using namespace fixture;

namespace {

constexpr uint64_t kGeomHash = 0x1111222233334444ull, kPackHash = 0x5555666677778888ull;
constexpr uint64_t kClient = 7, kRequest = 1;
int64_t T = 4096;   // tokens (argv[2]); config 1's length by default
constexpr int kRounds = 5;   // the first hand-off pays the module loads, the IPC import and peer enablement

ModelGeometry config_geometry() {
    ModelGeometry g;
    g.ssm_v_heads = 32;
    g.ssm_conv_channels = 8192;
    return g;
}

void send_line(int fd, const std::string& line) {
    const std::string l = line + "\n";
    check(write(fd, l.data(), l.size()) == (ssize_t) l.size(), "pipe write");
}
/// One line from `fd`, waiting at most `ms`; empty on timeout or a closed pipe.
std::string recv_line(int fd, int ms) {
    std::string out;
    char c = 0;
    while (true) {
        pollfd p{fd, POLLIN, 0};
        if (poll(&p, 1, ms) <= 0) return {};
        if (read(fd, &c, 1) != 1) return {};
        if (c == '\n') return out;
        out += c;
    }
}

int prefill(const std::string& dir, int to_decode, int from_decode, pid_t decode_pid) {
    cuda(cudaSetDevice(0), "cudaSetDevice(0)");
    const ModelGeometry g = config_geometry();
    DeviceSession a(g, T, std::max<int64_t>(4096, 13 * ((T + 255) / 256) + 64), 11);
    const Content content = make_content(a, 1);
    upload(a, content);
    cuda(cudaDeviceSynchronize(), "upload");
    const std::vector<ConversationImageKey> images;
    const std::vector<ConversationCheckpoint> checkpoints;
    const ConversationView view{content.ids, images, checkpoints, true};
    std::string err;
    HandoffSizing sizing;
    check_ok(handoff_size_arena({{(uint64_t) T, 1}}, std::vector<uint64_t>{kDeviceDescriptorBytes}, sizing, err), err,
             "arena sized for one descriptor slot");
    HandoffArena arena;
    const std::string path = dir + "/arena";
    check_ok(arena.open_writer(path, sizing, kPackHash, kGeomHash, err), err, "prefill opens the arena");
    arena.note_client_pid(kClient, (uint64_t) decode_pid);
    WirePlan plan;
    check_ok(conversation_wire_pack_plan(view, a.ss, g, a.draft, plan, err), err, "payload planned");
    skv_pool* payload_pool = nullptr;
    const uint64_t cap = (plan.total_bytes + 1023) & ~uint64_t(1023);
    check(skv_pool_create(0, 1, cap, &payload_pool) == SKV_OK, "payload buffer");
    uint8_t* buf = static_cast<uint8_t*>(skv_pool_base(payload_pool));
    uint8_t handle[64];
    check(skv_ipc_export(buf, handle) == SKV_OK, "payload exported through CUDA IPC");
    double publish_ms = 0, round_ms = 0;
    WireDevicePhases pack{};
    WireEncoded enc;
    for (int round = 0; round < kRounds; ++round) {
        HandoffClaim claim;
        check_ok(arena.claim(0, kClient, kRequest + (uint64_t) round, claim, err), err, "slot claimed");
        const auto t0 = std::chrono::steady_clock::now();
        check_ok(handoff_device_publish(arena, claim, view, a.ss, {}, g, a.draft, {kGeomHash, kPackHash}, buf, cap,
                                        handle, 0, enc, err),
                 err, "the session packed into HBM and its descriptor published");
        publish_ms = ms_since(t0);
        pack = conversation_wire_device_last_phases();
        check(enc.bytes == plan.total_bytes, "the published payload is the planned one");
        send_line(to_decode, "DONE " + std::to_string(claim.index) + " " + std::to_string(claim.nonce));
        const std::string ack = recv_line(from_decode, 120000);
        check(ack == "ACK " + std::to_string(claim.nonce), ("the decode instance acknowledged (got '" + ack + "')").c_str());
        check_ok(arena.release(claim.index, claim.nonce, err), err, "the slot is released on ACK");
        // the last round's ACK waits for the decode side's byte-by-byte checks: it does not time a hand-off
        if (round + 1 < kRounds) round_ms = round_ms == 0 ? ms_since(t0) : std::min(round_ms, ms_since(t0));
        HandoffSlotInfo info;
        check(arena.slot_info(claim.index, info) && info.state == kHandoffFree, "and is FREE again");
    }
    skv_pool_destroy(payload_pool);
    std::printf("prefill: last of %d rounds: publish (pack into HBM + descriptor) %.3f ms; fastest claim-to-release "
                "(publish, DONE, decode mount, ACK, release) %.3f ms for %llu payload bytes; %d checks passed\n",
                kRounds, publish_ms, round_ms, (unsigned long long) enc.bytes, checks);
    std::printf("prefill: pack phases prepare %.3f issue %.3f complete %.3f total %.3f ms\n", pack.prepare_ms,
                pack.issue_ms, pack.complete_ms, pack.total_ms);
    return 0;
}

int decode(const std::string& dir, int from_prefill, int to_prefill) {
    cuda(cudaSetDevice(1), "cudaSetDevice(1)");
    const ModelGeometry g = config_geometry();
    DeviceSession c(g, T, std::max<int64_t>(4096, 13 * ((T + 255) / 256) + 64), 37);
    const Content content = make_content(c, 1);   // the oracle's content: what the prefill instance holds
    std::string err;
    HandoffArena arena;
    DevicePayloadImports imports(1);
    WireExpect ex;
    ex.check_geometry = true;
    const std::array<int64_t, 18> key = {g.n_embd,    g.n_layers,       g.qsa_interval,  g.ssm_state_size, g.ssm_k_heads,
                                         g.ssm_v_heads, g.ssm_d_conv,   g.ssm_conv_channels, g.ssm_value_dim, g.n_head,
                                         g.n_head_kv, g.head_dim,       g.idx_q_heads,   g.idx_key_dim,    g.hc,
                                         g.hc_lr,     g.n_expert,       g.n_ff};
    ex.geometry = key;
    ex.check_hashes = true;
    ex.geom_hash = kGeomHash;
    ex.pack_hash = kPackHash;
    SavedConversation meta;
    WireDecoded info;
    double mount_ms = 0;
    WireDevicePhases mount{};
    unsigned long long nonce = 0;
    for (int round = 0; round < kRounds; ++round) {
        const std::string done = recv_line(from_prefill, 120000);
        unsigned long long index = 0;
        check(std::sscanf(done.c_str(), "DONE %llu %llu", &index, &nonce) == 2, ("a DONE line (got '" + done + "')").c_str());
        if (round == 0) check_ok(arena.open_reader(dir + "/arena", kPackHash, kGeomHash, err), err, "decode opens the arena");
        HandoffPayload slot;
        check(!arena.read_slot((int) index, nonce ^ 1, kClient, slot, err), "a wrong nonce cannot read the slot");
        check(!arena.read_slot((int) index, nonce, kClient + 1, slot, err), "nor another client");
        const auto t0 = std::chrono::steady_clock::now();
        check_ok(arena.read_slot((int) index, nonce, kClient, slot, err), err, "the slot is READY for this client");
        check(handoff_device_is_descriptor(slot.data, slot.payload_bytes), "the slot holds a device descriptor");
        check(handoff_device_mount(slot, imports, c.ss, {}, g, c.draft, ex, meta, info, err) ==
                  ConversationRestore::restored,
              ("mounted from GPU 0's HBM: " + err).c_str());
        mount_ms = ms_since(t0);
        mount = conversation_wire_device_last_phases();
        if (round + 1 < kRounds) send_line(to_prefill, "ACK " + std::to_string(nonce));
    }
    for (size_t j = 0; j < c.qsa.size() + 1; ++j) {
        check(c.get(j, 0) == content.k[j], "K arrived through the decode GPU's table");
        check(c.get(j, 1) == content.v[j], "V arrived through the decode GPU's table");
    }
    check(from_device(c.gdn, content.gdn.size()) == content.gdn, "GDN rows arrived");
    for (size_t j = 0; j < c.qsa.size(); ++j) {
        const QsaState& st = c.qsa[j];
        check(from_device(st.idx_tail, content.tail[j].size()) == content.tail[j], "indexer tail arrived");
        check(from_device(st.idx_dead, content.dead[j].size()) == content.dead[j], "indexer dead key arrived");
        check(from_device(st.idx_block_pos, 1)[0] == content.block_pos[j], "indexer block position arrived");
        const size_t rows = (size_t) (T / 4), dim = (size_t) g.idx_key_dim;
        const auto pooled = from_device(st.idx_pooled, (rows + 1) * dim);
        check(std::equal(pooled.begin(), pooled.begin() + rows * dim, content.pooled[j].begin()), "pooled rows arrived");
    }
    check(meta.live.ids == content.ids, "the token ids");
    send_line(to_prefill, "ACK " + std::to_string(nonce));
    std::printf("decode: last of %d rounds: read the slot + mount from the peer's HBM %.3f ms (%llu payload bytes "
                "over NVLink); %d checks passed\n",
                kRounds, mount_ms, (unsigned long long) info.bytes, checks);
    std::printf("decode: mount phases prepare %.3f issue %.3f complete %.3f total %.3f ms\n", mount.prepare_ms,
                mount.issue_ms, mount.complete_ms, mount.total_ms);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    const std::string dir = argc > 1 ? argv[1] : "/tmp";
    if (argc > 2) T = std::strtoll(argv[2], nullptr, 10);
    if (T < 1 || T > 131072) return 2;
    int p2d[2], d2p[2];
    if (pipe(p2d) != 0 || pipe(d2p) != 0) return 2;
    const pid_t child = fork();   // before any CUDA call in either process
    if (child < 0) return 2;
    if (child == 0) {
        close(p2d[1]);
        close(d2p[0]);
        int devices = 0;
        if (cudaGetDeviceCount(&devices) != cudaSuccess || devices < 2) return 77;
        return decode(dir, p2d[0], d2p[1]);
    }
    close(p2d[0]);
    close(d2p[1]);
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices < 2) {
        kill(child, SIGTERM);
        waitpid(child, nullptr, 0);
        return 77;
    }
    const int rc = prefill(dir, p2d[1], d2p[0], child);
    int status = 0;
    waitpid(child, &status, 0);
    const int child_rc = WIFEXITED(status) ? WEXITSTATUS(status) : 1;
    if (rc != 0 || child_rc != 0) {
        std::fprintf(stderr, "FAIL: prefill %d, decode %d\n", rc, child_rc);
        return 1;
    }
    std::printf("handoff_device_gpu_test: both instances passed\n");
    return 0;
}
