#pragma once

// Records exchanged over the shared-memory rings. Every record starts with a
// shm::WireHdr; the producing rank is implicit (ring index).
//
// Host (CPU tensor) messages:
//   EAGER  first fragment of a message <= eager limit: key, total, msg id
//   FRAG   continuation bytes of an EAGER message or of a rendezvous DATA
//          stream (msg id in the sender's id space for EAGER, recv id with
//          kDataBit for DATA)
//   RTS    request-to-send for a large host message (no payload)
//   CTS    clear-to-send: receiver matched an RTS, names its recv id
// Device (CUDA tensor) messages:
//   DRTS   device request-to-send: sender's IPC descriptors and flag slot;
//          the receiver pulls the bytes with a kernel
//   FIN    receiver -> sender: the transfer of send id is complete
// Control:
//   ABORT  the producer aborts the group (code, reason)

#include <cstdint>

#include "shm.hpp"

namespace commux {
namespace proto {

enum : std::uint16_t {
  kEager = 1,
  kFrag = 2,
  kRts = 3,
  kCts = 4,
  kDrts = 5,
  kFin = 6,
  kAbort = 7,
  kIndirect = 8,  // sender-local, TCP peers only: never crosses the wire
};

constexpr std::uint64_t kDataBit = 1ull << 63;

struct EagerRec {
  shm::WireHdr h;
  std::uint64_t key;     // match key (tag without the rank field)
  std::uint64_t total;   // message bytes
  std::uint64_t msg_id;  // sender id of this message
  std::uint64_t nbytes;  // payload bytes in this record
  // payload follows
};

struct FragRec {
  shm::WireHdr h;
  std::uint64_t msg_id;
  std::uint64_t offset;
  std::uint64_t nbytes;
  // payload follows
};

// Written into the out-ring of a TCP peer instead of an EAGER or FRAG record
// with a large payload: it names the payload in this process's memory, and
// the TCP pump sends the record header it carries followed by the payload
// straight from there (zero padding up to wire_len), so the payload is not
// copied into the ring first. With h.flags == kIndirectComplete, the request
// `done_id` completes once the pump has sent the record: the payload memory
// must stay valid until then.
constexpr std::uint16_t kIndirectComplete = 1;
struct IndirectRec {
  shm::WireHdr h;
  std::uint32_t wire_len;    // bytes of the record on the wire (header + payload + pad)
  std::uint32_t head_bytes;  // bytes of the header below (EagerRec or FragRec)
  std::uint64_t payload;     // address of the payload in this process
  std::uint64_t payload_bytes;
  std::uint64_t done_id;
  std::uint64_t head[5];     // the on-wire record header
};
static_assert(sizeof(EagerRec) <= sizeof(IndirectRec::head) && sizeof(FragRec) <= sizeof(IndirectRec::head),
              "an indirect record carries the whole record header");

// Host rendezvous. When the sender's bytes are in at most kCmaSegs host
// segments, the record also lists them (address, length) with the sender's
// pid: a receiver on the same host may then copy them straight out of the
// sender's memory (process_vm_readv) and answer with a FIN instead of a CTS.
constexpr std::uint32_t kCmaSegs = 16;

struct CmaSeg {
  std::uint64_t addr;
  std::uint64_t bytes;
};

struct RtsRec {
  shm::WireHdr h;
  std::uint64_t key;
  std::uint64_t total;
  std::uint64_t send_id;
  std::int32_t pid;     // sender's pid (single-copy read)
  std::uint32_t nseg;   // CmaSeg entries that follow (0: CTS path only)
  // CmaSeg seg[nseg] follow
};

struct CtsRec {
  shm::WireHdr h;
  std::uint64_t send_id;
  std::uint64_t recv_id;
};

struct DrtsRec {
  shm::WireHdr h;
  std::uint64_t key;
  std::uint64_t total;
  std::uint64_t send_id;
  std::uint32_t blob_bytes;  // device descriptor blob (opaque to the engine)
  std::uint32_t pad;
  // blob follows
};

struct FinRec {
  shm::WireHdr h;
  std::uint64_t send_id;
  std::int64_t status;  // 0 ok, kFinLaunched, else error code (negative)
};
// FIN status of a device message whose sender waits on its GPU: the receiver
// has enqueued the copy (a second FIN with status 0 follows its completion)
constexpr std::int64_t kFinLaunched = 1;

struct AbortRec {
  shm::WireHdr h;
  std::int64_t code;
  char reason[112];
};

}  // namespace proto
}  // namespace commux
