// tests/cpp/handoff_device_cpu_test.cpp - the device descriptor and its trip through a hand-off slot, host only.
//
// Encode -> decode round trip; every refusal (size, magic, version, header bytes, reserved bytes, bus id, a
// payload shorter than a header, a misaligned offset); an SR4H payload is not mistaken for a descriptor; and a
// descriptor claimed, written, published and read back through a real HandoffArena (tmpfs or any directory).
//
// Usage: handoff_device_cpu_test <directory for the arena>      (exit 0 = pass)
#include "strata_kv/handoff_device.hpp"

#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

using namespace strata::core;

namespace {
int checks = 0;
void check(bool ok, const std::string& label) {
    ++checks;
    if (!ok) {
        std::fprintf(stderr, "FAIL: %s\n", label.c_str());
        std::exit(1);
    }
}
HandoffDeviceDescriptor sample() {
    HandoffDeviceDescriptor d;
    for (int i = 0; i < 64; ++i) d.ipc_handle[i] = (uint8_t) (i * 7 + 3);
    d.alloc_offset = 4096;
    d.payload_bytes = 194429376;
    d.device = 3;
    std::strcpy(d.pci_bus_id, "0000:1b:00.0");
    d.geom_hash = 0x1111222233334444ull;
    d.pack_hash = 0x5555666677778888ull;
    d.tokens = 4096;
    d.payload_fnv = 0xABCDEF0123456789ull;
    return d;
}
bool same(const HandoffDeviceDescriptor& a, const HandoffDeviceDescriptor& b) {
    return std::memcmp(a.ipc_handle, b.ipc_handle, 64) == 0 && a.alloc_offset == b.alloc_offset &&
           a.payload_bytes == b.payload_bytes && a.device == b.device && std::strcmp(a.pci_bus_id, b.pci_bus_id) == 0 &&
           a.geom_hash == b.geom_hash && a.pack_hash == b.pack_hash && a.tokens == b.tokens &&
           a.payload_fnv == b.payload_fnv;
}
}  // namespace

int main(int argc, char** argv) {
    const std::string dir = argc > 1 ? argv[1] : "/tmp";
    std::string err;
    uint8_t rec[kDeviceDescriptorBytes];
    const HandoffDeviceDescriptor d = sample();
    handoff_device_encode(d, rec);
    HandoffDeviceDescriptor back;
    check(handoff_device_decode(rec, sizeof rec, back, err) && same(d, back), "round trip: " + err);
    check(handoff_device_is_descriptor(rec, sizeof rec), "recognised by its magic");
    check(!handoff_device_is_descriptor(rec, sizeof rec - 1), "but not at another size");
    uint8_t sr4h[kDeviceDescriptorBytes] = {'S', 'R', '4', 'H'};
    check(!handoff_device_is_descriptor(sr4h, sizeof sr4h), "an SR4H payload is not a descriptor");
    auto refused = [&](void (*mutate)(uint8_t*), const char* what, const char* needle) {
        uint8_t bad[kDeviceDescriptorBytes];
        std::memcpy(bad, rec, sizeof bad);
        mutate(bad);
        HandoffDeviceDescriptor out;
        check(!handoff_device_decode(bad, sizeof bad, out, err), std::string(what) + " is refused");
        check(err.find(needle) != std::string::npos, std::string(what) + ": the refusal says why (" + err + ")");
    };
    refused([](uint8_t* p) { p[0] = 'X'; }, "a bad magic", "magic");
    refused([](uint8_t* p) { p[8] = 2; }, "another version", "version");
    refused([](uint8_t* p) { p[13] = 0; }, "another header size", "header_bytes");
    refused([](uint8_t* p) { p[200] = 1; }, "a non-zero reserved byte", "reserved");
    refused([](uint8_t* p) { p[131] = 'x'; }, "an unterminated bus id", "bus id");
    refused([](uint8_t* p) { std::memset(p + 88, 0, 8); }, "a payload shorter than a header", "shorter");
    refused([](uint8_t* p) { p[80] = 17; }, "a misaligned payload offset", "boundary");
    HandoffDeviceDescriptor out;
    check(!handoff_device_decode(rec, sizeof rec - 1, out, err) && err.find("256") != std::string::npos,
          "a short record is refused");

    // through a hand-off slot
    HandoffSizing sizing;
    check(handoff_size_arena({{4096, 2}}, std::vector<uint64_t>{kDeviceDescriptorBytes}, sizing, err), "sized: " + err);
    const std::string path = dir + "/skv-device-descriptor-" + std::to_string(getpid()) + "/arena";
    HandoffArena writer;
    check(writer.open_writer(path, sizing, d.pack_hash, d.geom_hash, err), "writer: " + err);
    HandoffClaim claim;
    check(writer.claim(0, 9, 1, claim, err), "claim: " + err);
    check(writer.write_payload(claim, 0, rec, sizeof rec, err) &&
              writer.publish(claim, d.tokens, sizeof rec, fnv1a64(rec, sizeof rec), err),
          "published: " + err);
    HandoffArena reader;
    check(reader.open_reader(path, d.pack_hash, d.geom_hash, err), "reader: " + err);
    HandoffPayload slot;
    check(reader.read_slot(claim.index, claim.nonce, 9, slot, err), "read: " + err);
    check(handoff_device_is_descriptor(slot.data, slot.payload_bytes), "the slot holds the descriptor");
    check(HandoffArena::payload_hash_of(slot) == slot.payload_hash, "its hash matches the slot header");
    check(handoff_device_decode(slot.data, slot.payload_bytes, out, err) && same(d, out), "and decodes: " + err);
    check(writer.release(claim.index, claim.nonce, err), "released: " + err);
    std::remove(path.c_str());
    std::remove((dir + "/skv-device-descriptor-" + std::to_string(getpid())).c_str());
    std::printf("handoff_device_cpu_test: %d checks passed\n", checks);
    return 0;
}
