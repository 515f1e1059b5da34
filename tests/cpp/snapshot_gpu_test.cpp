// tests/cpp/snapshot_gpu_test.cpp - the C++ drop-in park/mount path on a real device, against the reference.
//
// Config 1 of the benchmark (full geometry, 4,096 tokens, seed 1) is placed into a 4,096-block pool at
// seed-random slots - a NON-identity page table - and parked with conversation_snapshot_save.  The parked image,
// encoded with the SR4H codec, must hash to exactly the FNV-1a the reference's own save + encode produced from
// its identity-layout pool (tests/golden/golden.json, passed on the command line).  The image is then mounted into
// a second pool with different random slots and every byte is read back through that pool's table.  The
// device-side pack must write the same payload straight from the permuted pool, into pinned host memory and into
// device memory, and that payload must decode back to the parked image.
//
// Usage: snapshot_gpu_test <golden payload bytes> <golden payload fnv>      (exit 0 = pass)
// The synthetic content comes from the test oracle's seeded generators (oracle/kv_oracle.c), the same calls
// tests/golden/make_golden.py made.
#include "session_fixture.hpp"
#include "strata_kv/conversation_wire.hpp"
#include "strata_kv/conversation_wire_device.hpp"

using namespace strata::core;
using namespace fixture;


int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: snapshot_gpu_test <golden bytes> <golden fnv>\n");
        return 2;
    }
    const uint64_t golden_bytes = std::strtoull(argv[1], nullptr, 10);
    const uint64_t golden_hash = std::strtoull(argv[2], nullptr, 10);
    const uint64_t geom_hash = 0x1111222233334444ull, pack_hash = 0x5555666677778888ull;   // make_golden.py's
    cuda(cudaSetDevice(0), "cudaSetDevice");

    ModelGeometry g;
    g.ssm_v_heads = 32;
    g.ssm_conv_channels = 8192;   // the configs' GDN state: 32 x 128 x 128 fp32 + 3 x 8192 fp32 conv tail
    const int64_t T = 4096;
    std::string err;

    DeviceSession a(g, T, 4096, 11);
    const Content content = make_content(a, 1);
    upload(a, content);
    cuda(cudaDeviceSynchronize(), "upload done");
    const std::vector<ConversationImageKey> images;
    const std::vector<ConversationCheckpoint> checkpoints;
    const ConversationView view{content.ids, images, checkpoints, true};

    // ---- park a permuted pool; the image is the reference's, byte for byte
    size_t estimate = 0;
    check_ok(conversation_snapshot_bytes(view, a.ss, g, a.draft, estimate, err), err, "snapshot priced");
    SavedConversation img;
    auto t0 = std::chrono::steady_clock::now();
    check_ok(conversation_snapshot_save(img, view, a.ss, g, a.draft, err), err, "snapshot saved from a permuted pool");
    const double park_ms = ms_since(t0);
    check(img.bytes() == estimate, "the estimate is exactly what the image holds");
    check(img.kv.size() == (size_t) g.n_qsa_layers() + 1, "main layers and the draft");
    for (size_t j = 0; j < img.kv.size(); ++j) {
        check(read_buffer(img.kv[j].k) == content.k[j], "parked K equals the logical K of the layer");
        check(read_buffer(img.kv[j].v) == content.v[j], "parked V equals the logical V of the layer");
    }
    check(img.live.gdn == as_bytes(content.gdn), "parked GDN rows");
    VectorWireSink sink;
    WireEncoded enc;
    check_ok(conversation_wire_encode(img, sink, {geom_hash, pack_hash}, enc, err), err, "encoded");
    check(enc.bytes == golden_bytes, "the payload has the reference's length");
    check(enc.payload_hash == golden_hash, "the payload's FNV-1a is the reference's (every byte identical)");
    t0 = std::chrono::steady_clock::now();
    {
        VectorWireSink again_sink(golden_bytes);
        WireEncoded again_enc;
        check_ok(conversation_wire_encode(img, again_sink, {geom_hash, pack_hash}, again_enc, err), err, "encoded again");
    }
    const double encode_ms = ms_since(t0);

    // ---- the device-side pack: the same payload straight from the permuted pool, no host image in between
    double pack_ms = 0, pack_hash_ms = 0, pack_dev_ms = 0, mount_dev_ms = 0;
    {
        WirePlan plan;
        check_ok(conversation_wire_pack_plan(view, a.ss, g, a.draft, plan, err), err, "device pack planned");
        check(plan.total_bytes == golden_bytes, "the planned payload has the reference's length");
        uint8_t* pinned = nullptr;
        cuda(cudaHostAlloc(reinterpret_cast<void**>(&pinned), plan.total_bytes, cudaHostAllocDefault), "pinned payload");
        std::memset(pinned, 0xA5, plan.total_bytes);   // every byte has to be written by the pack
        WirePlan used;
        WireEncoded denc;
        t0 = std::chrono::steady_clock::now();
        check_ok(conversation_wire_pack_device(view, a.ss, g, a.draft, {geom_hash, pack_hash}, pinned, plan.total_bytes,
                                               used, denc, err),
                 err, "device pack into pinned host memory");
        pack_hash_ms = ms_since(t0);
        check(denc.bytes == golden_bytes, "the device-packed payload has the reference's length");
        check(denc.payload_hash == golden_hash, "the device-packed payload's FNV-1a is the reference's");
        check(std::memcmp(pinned, sink.data().data(), golden_bytes) == 0, "and it equals the host encoder's bytes");
        check(used.total_bytes == plan.total_bytes && denc.blobs == plan.blobs, "the pack follows its plan");

        std::memset(pinned, 0x5A, plan.total_bytes);
        WireDeviceOptions no_hash;
        no_hash.hash = false;
        t0 = std::chrono::steady_clock::now();
        check_ok(conversation_wire_pack_device(view, a.ss, g, a.draft, {geom_hash, pack_hash}, pinned, plan.total_bytes,
                                               used, denc, err, no_hash),
                 err, "device pack without the host hash pass");
        pack_ms = ms_since(t0);
        check(denc.payload_hash == 0, "no hash when none is asked for");
        check(fnv1a64(pinned, golden_bytes) == golden_hash, "a second pack over other garbage writes the same bytes");

        SavedConversation decoded;
        WireDecoded info;
        WireExpect expect;
        expect.check_payload_hash = true;
        expect.payload_hash = golden_hash;
        check_ok(conversation_wire_decode(pinned, golden_bytes, decoded, info, expect, err), err,
                 "the device-packed payload decodes");
        check(decoded.kv.size() == img.kv.size(), "every layer decoded");
        for (size_t j = 0; j < img.kv.size(); ++j)
            check(decoded.kv[j].k == img.kv[j].k && decoded.kv[j].v == img.kv[j].v &&
                      decoded.kv[j].pooled == img.kv[j].pooled,
                  "decoded K/V and indexer rows equal the parked image");
        check(decoded.live.gdn == img.live.gdn && decoded.live.tails == img.live.tails &&
                  decoded.live.dead == img.live.dead && decoded.live.block_pos == img.live.block_pos,
              "decoded running state equals the parked image");

        uint8_t* on_device = nullptr;
        cuda(cudaMalloc(&on_device, plan.total_bytes), "device payload");
        cuda(cudaMemset(on_device, 0xA5, plan.total_bytes), "device payload garbage");
        t0 = std::chrono::steady_clock::now();
        check_ok(conversation_wire_pack_device(view, a.ss, g, a.draft, {geom_hash, pack_hash}, on_device,
                                               plan.total_bytes, used, denc, err),
                 err, "device pack into device memory");
        pack_dev_ms = ms_since(t0);
        std::vector<uint8_t> back(golden_bytes);
        cuda(cudaMemcpy(back.data(), on_device, golden_bytes, cudaMemcpyDeviceToHost), "device payload read back");
        check(back == sink.data(), "the device-resident payload equals the host encoder's bytes");

        check(!conversation_wire_pack_device(view, a.ss, g, a.draft, {geom_hash, pack_hash}, pinned,
                                             plan.total_bytes - 1, used, denc, err),
              "a destination one byte short is refused");
        check(err.find("needs") != std::string::npos, "and the refusal names the size");

        // ---- the device mount: that device-resident payload straight into a differently permuted pool
        {
            DeviceSession c(g, T, 4096, 37);
            check(c.slots[0] != a.slots[0], "the mount target's placement differs from the source's");
            WireExpect ex;
            ex.check_geometry = true;
            ex.geometry = img.geometry;
            ex.check_hashes = true;
            ex.geom_hash = geom_hash;
            ex.pack_hash = pack_hash;
            SavedConversation meta;
            WireDecoded dinfo;
            // refusals first: nothing may be written
            const auto before = c.get(0, 0);
            {
                WireExpect wrong = ex;
                wrong.pack_hash ^= 1;
                check(conversation_wire_mount_device(on_device, plan.total_bytes, c.ss, g, c.draft, wrong, meta, dinfo,
                                                     err) == ConversationRestore::invalid,
                      "a payload for another pack is refused");
                SessionState fewer = c.ss;
                fewer.qsa_alloc -= 1;   // a session that owns one QSA layer less than the image carries
                check(conversation_wire_mount_device(on_device, plan.total_bytes, fewer, g, c.draft, ex, meta, dinfo,
                                                     err) == ConversationRestore::invalid,
                      "an image for another layer carve is refused");
                uint8_t* bad = nullptr;
                cuda(cudaMalloc(&bad, plan.total_bytes), "corrupt copy");
                cuda(cudaMemcpy(bad, on_device, plan.total_bytes, cudaMemcpyDeviceToDevice), "corrupt copy");
                const uint8_t flip = 0x10;
                cuda(cudaMemcpy(bad + 6, &flip, 1, cudaMemcpyHostToDevice), "flip a header flag bit");
                check(conversation_wire_mount_device(bad, plan.total_bytes, c.ss, g, c.draft, ex, meta, dinfo, err) ==
                          ConversationRestore::invalid,
                      "a corrupted header is refused");
                cudaFree(bad);
                check(c.get(0, 0) == before, "and none of the refusals wrote anything");
            }
            t0 = std::chrono::steady_clock::now();
            check(conversation_wire_mount_device(on_device, plan.total_bytes, c.ss, g, c.draft, ex, meta, dinfo, err) ==
                      ConversationRestore::restored,
                  ("device mount of the device payload: " + err).c_str());
            mount_dev_ms = ms_since(t0);
            check(meta.live.ids == content.ids && meta.live.gdn.empty() && meta.kv.size() == img.kv.size(),
                  "the mount's metadata: the ids on the host, the bytes on the device");
            for (size_t j = 0; j < img.kv.size(); ++j) {
                check(c.get(j, 0) == content.k[j], "device-mounted K reads back through the destination table");
                check(c.get(j, 1) == content.v[j], "device-mounted V reads back through the destination table");
            }
            check(from_device(c.gdn, content.gdn.size()) == content.gdn, "device-mounted GDN rows");
            for (size_t j = 0; j < c.qsa.size(); ++j) {
                const QsaState& st = c.qsa[j];
                check(from_device(st.idx_tail, content.tail[j].size()) == content.tail[j], "device-mounted indexer tail");
                check(from_device(st.idx_dead, content.dead[j].size()) == content.dead[j], "device-mounted dead key");
                check(from_device(st.idx_block_pos, 1)[0] == content.block_pos[j], "device-mounted block position");
                const size_t rows = (size_t) (T / 4), dim = (size_t) g.idx_key_dim;
                const auto pooled = from_device(st.idx_pooled, (rows + 1) * dim);
                check(std::equal(pooled.begin(), pooled.begin() + rows * dim, content.pooled[j].begin()),
                      "device-mounted pooled rows");
                check(std::equal(pooled.begin() + rows * dim, pooled.end(), content.dead[j].begin()),
                      "the spare pooled row is the dead key again");
            }
            check(c.ss.ple_prev[0] == content.ids[T - 2] && c.ss.ple_prev[1] == content.ids[T - 1],
                  "the PLE window after a device mount");
            uint64_t fp = 0;
            check_ok(conversation_kv_verify(img.kv.back(), c.draft, g, T, false, fp, err), err,
                     "read-back verify of the device-mounted draft");
        }
        cudaFree(on_device);
        cudaFreeHost(pinned);
    }

    // ---- mount into a pool with different random slots
    DeviceSession b(g, T, 4096, 23);
    check(b.slots[0] != a.slots[0], "the destination placement differs from the source's");
    t0 = std::chrono::steady_clock::now();
    check(conversation_snapshot_restore(img, b.ss, g, b.draft, err) == ConversationRestore::restored,
          "mounted into a differently permuted pool");
    const double mount_ms = ms_since(t0);
    for (size_t j = 0; j < img.kv.size(); ++j) {
        check(b.get(j, 0) == content.k[j], "mounted K reads back through the destination table");
        check(b.get(j, 1) == content.v[j], "mounted V reads back through the destination table");
    }
    check(from_device(b.gdn, content.gdn.size()) == content.gdn, "mounted GDN rows");
    for (size_t j = 0; j < b.qsa.size(); ++j) {
        const QsaState& st = b.qsa[j];
        check(from_device(st.idx_tail, content.tail[j].size()) == content.tail[j], "mounted indexer tail");
        check(from_device(st.idx_dead, content.dead[j].size()) == content.dead[j], "mounted indexer dead key");
        const size_t rows = (size_t) (T / 4), dim = (size_t) g.idx_key_dim;
        const auto pooled = from_device(st.idx_pooled, (rows + 1) * dim);
        check(std::equal(pooled.begin(), pooled.begin() + rows * dim, content.pooled[j].begin()), "mounted pooled rows");
        check(std::equal(pooled.begin() + rows * dim, pooled.end(), content.dead[j].begin()),
              "the spare pooled row is the dead key again");
    }
    check(b.ss.ple_prev[0] == content.ids[T - 2] && b.ss.ple_prev[1] == content.ids[T - 1], "the PLE window");
    // read-back verify: the draft after the whole mount (what the engine verifies), and an index layer right
    // after a per-layer restore (a whole mount rewrites its moving spare pooled row with the dead key)
    uint64_t fp = 0;
    check_ok(conversation_kv_verify(img.kv.back(), b.draft, g, T, false, fp, err), err, "read-back verify of the draft");
    check(fp != 0, "a fingerprint");
    check_ok(conversation_kv_restore(img.kv[0], b.qsa[0], g, T, true, err), err, "per-layer restore");
    check_ok(conversation_kv_verify(img.kv[0], b.qsa[0], g, T, true, fp, err), err, "read-back verify of an index layer");
    check(conversation_checkpoint_restore(img.live, b.ss, g, err), "the running state again");
    {
        const int32_t flipped = 0x5a5a5a5a;
        int32_t* k_first = reinterpret_cast<int32_t*>(b.base + (int64_t) b.slots[0][0] * kSlotPages * b.page_bytes);
        int32_t saved_word = 0;
        cuda(cudaMemcpy(&saved_word, k_first, 4, cudaMemcpyDeviceToHost), "read a K word");
        cuda(cudaMemcpy(k_first, &flipped, 4, cudaMemcpyHostToDevice), "corrupt a K word");
        check(!conversation_kv_verify(img.kv[0], b.qsa[0], g, T, true, fp, err), "read-back detects a corrupted byte");
        cuda(cudaMemcpy(k_first, &saved_word, 4, cudaMemcpyHostToDevice), "repair the K word");
    }

    // ---- incremental re-park: the retained K/V is reused, the result is the same image
    ConversationKvReuse reuse{img.kv, T, T};
    SavedConversation again;
    size_t reused = 0;
    check_ok(conversation_snapshot_save(again, view, a.ss, g, a.draft, err, std::move(reuse), &reused), err,
             "incremental re-park");
    check(reused > 0, "the unchanged prefix was not copied again");
    for (size_t j = 0; j < img.kv.size(); ++j)
        check(again.kv[j].k == img.kv[j].k && again.kv[j].v == img.kv[j].v && again.kv[j].pooled == img.kv[j].pooled,
              "incremental capture equals the full capture");

    // ---- refusals before any write; a device-side refusal after it
    {
        SavedConversation bad = img;
        bad.kv[3].v.pop_back();
        const auto before = b.get(0, 0);
        check(conversation_snapshot_restore(bad, b.ss, g, b.draft, err) == ConversationRestore::invalid,
              "a corrupted image is refused");
        check(b.get(0, 0) == before, "and nothing was written");
    }
    {
        const int32_t bad_page = (int32_t) (b.pool_blocks * kSlotPages + 1000);
        cuda(cudaMemcpy(b.dev_tables[2] + 5, &bad_page, 4, cudaMemcpyHostToDevice), "poison one table entry");
        check(conversation_snapshot_restore(img, b.ss, g, b.draft, err) == ConversationRestore::transfer_failed,
              "a table entry outside the pool fails the mount (the kernel refused it, nothing out of bounds)");
        check(err.find("outside its pool") != std::string::npos, "and says why");
        const int32_t good = b.tables[2][5];
        cuda(cudaMemcpy(b.dev_tables[2] + 5, &good, 4, cudaMemcpyHostToDevice), "restore the entry");
        check(conversation_snapshot_restore(img, b.ss, g, b.draft, err) == ConversationRestore::restored,
              "the same mount succeeds once the table is sound");
    }
    std::printf("park %.2f ms, mount %.2f ms for %.1f MB of K/V + state (%llu payload bytes)\n", park_ms, mount_ms,
                (double) img.bytes() / 1e6, (unsigned long long) enc.bytes);
    std::printf("host encode %.2f ms; device pack %.2f ms to pinned host (%.2f ms with the FNV pass), %.2f ms to "
                "device memory; device mount %.2f ms\n",
                encode_ms, pack_ms, pack_hash_ms, pack_dev_ms, mount_dev_ms);
    std::printf("snapshot_gpu_test: %d checks passed\n", checks);
    return 0;
}
