// Out-of-process sidecar for the resident epoch engine: one client on a Unix
// stream socket under /dev/shm, fixed-size little-endian messages (136-byte
// requests, 352-byte responses, the 4,088-byte device-IPC metadata after a
// request of operation 5), one engine created through the reference-compatible
// C ABI.  Wire format, operations, startup handshake and exit codes follow the
// reference sidecar (native/resident_epoch_server.cpp:1-216,
// src/vllm_ascend_resident_epoch/sidecar_backend.py:23-36) so its Python client
// can drive this server unchanged.
//
//   usage: cruise_epoch_server SOCKET MODEL GRAPH_CONFIG FUNC_CONFIG WEIGHTS TILING
//
// MODEL is a preset name ("qwen2.5-7b", "tiny"), WEIGHTS a directory of raw bf16
// tensors or "synthetic:<seed>", TILING an optional 72-byte file ("" for none);
// GRAPH_CONFIG and FUNC_CONFIG are accepted and ignored, as by the bridge.
//
// Exit codes: 64 usage, 65 socket, 66 accept, 100 + create status when the
// engine cannot be created (also sent as the startup response's status), 67
// startup send, 68 client gone, 70 shutdown reply, 72 reply, 73 short metadata;
// 0 after a shutdown request.

#include <cerrno>
#include <csignal>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include "../../include/cruise_epoch.h"
#include "../../include/cruise_protocol.h"

namespace {

constexpr uint32_t kRequestMagic = 0x71317131u;
constexpr uint32_t kResponseMagic = 0x71327132u;

enum Operation : uint16_t { kExecute = 1, kWarmUp = 2, kShutdown = 3, kImportExecute = 4, kDeviceIpcExecute = 5 };

// Wire layouts (packed, little-endian as on the host).
#pragma pack(push, 1)
struct alignas(8) WireRequest {
  uint32_t magic;
  uint16_t version;
  uint16_t operation;
  int32_t request_count;
  int32_t max_steps;
  uint64_t transfer_id;
  int64_t token[CRUISE_BATCH];
  int64_t position[CRUISE_BATCH];
  int32_t seq_len[CRUISE_BATCH];
  int32_t eos[CRUISE_BATCH];
  int32_t generation[CRUISE_BATCH];
};

struct alignas(8) WireResponse {
  uint32_t magic;
  int32_t transport_status;
  int32_t device_status;
  int32_t model_calls;
  int32_t feed_calls;
  int32_t fetch_calls;
  int32_t commit_state;
  int32_t import_checksum;
  int64_t wall_us;
  int64_t native_cpu_us;
  int64_t declared_input_bytes;
  int64_t declared_output_bytes;
  int32_t executed[CRUISE_BATCH];
  int32_t generation[CRUISE_BATCH];
  int64_t tokens[CRUISE_BATCH * CRUISE_MAX_STEPS];   // [row][step], -1 filled
};
#pragma pack(pop)

static_assert(sizeof(WireRequest) == CRUISE_SIDECAR_REQUEST_BYTES, "sidecar request size");
static_assert(sizeof(WireResponse) == CRUISE_SIDECAR_RESPONSE_BYTES, "sidecar response size");
static_assert(sizeof(ResidentEpochIpcMetadata) == CRUISE_RESIDENT_IPC_METADATA_BYTES, "IPC metadata size");

// A connected stream socket with whole-message reads and writes.
class Channel {
 public:
  explicit Channel(int fd) : fd_(fd) {}
  ~Channel() {
    if (fd_ >= 0) close(fd_);
  }
  Channel(const Channel &) = delete;
  Channel &operator=(const Channel &) = delete;

  bool receive(void *dst, size_t bytes) {
    auto *p = static_cast<uint8_t *>(dst);
    while (bytes != 0) {
      const ssize_t n = read(fd_, p, bytes);
      if (n == 0) return false;   // peer closed
      if (n < 0) {
        if (errno == EINTR) continue;
        return false;
      }
      p += n;
      bytes -= static_cast<size_t>(n);
    }
    return true;
  }

  bool send(const void *src, size_t bytes) {
    const auto *p = static_cast<const uint8_t *>(src);
    while (bytes != 0) {
      const ssize_t n = write(fd_, p, bytes);
      if (n < 0) {
        if (errno == EINTR) continue;
        return false;
      }
      p += n;
      bytes -= static_cast<size_t>(n);
    }
    return true;
  }

 private:
  int fd_;
};

// The listening socket; the path is removed again when the server ends.
class Listener {
 public:
  explicit Listener(const char *path) : path_(path == nullptr ? "" : path) {
    if (path_.rfind("/dev/shm/", 0) != 0) return;   // the deployment keeps the control socket in shm
    sockaddr_un addr{};
    if (path_.size() >= sizeof(addr.sun_path)) return;
    addr.sun_family = AF_UNIX;
    std::memcpy(addr.sun_path, path_.c_str(), path_.size() + 1);
    const int fd = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) return;
    unlink(path_.c_str());
    if (bind(fd, reinterpret_cast<const sockaddr *>(&addr), sizeof(addr)) != 0 || listen(fd, 1) != 0) {
      close(fd);
      unlink(path_.c_str());
      return;
    }
    fd_ = fd;
  }
  ~Listener() {
    if (fd_ >= 0) {
      close(fd_);
      unlink(path_.c_str());
    }
  }
  Listener(const Listener &) = delete;
  Listener &operator=(const Listener &) = delete;

  bool ok() const { return fd_ >= 0; }
  int accept_one() const {
    for (;;) {
      const int fd = accept4(fd_, nullptr, nullptr, SOCK_CLOEXEC);
      if (fd >= 0 || errno != EINTR) return fd;
    }
  }

 private:
  std::string path_;
  int fd_ = -1;
};

WireResponse blank_response(int32_t transport_status) {
  WireResponse r{};
  r.magic = kResponseMagic;
  r.transport_status = transport_status;
  r.device_status = -1;
  r.commit_state = CRUISE_EPOCH_PREPARED;
  for (int64_t &t : r.tokens) t = -1;
  return r;
}

// One request through resident_epoch_execute; the snapshot import reads the
// transfer file next to the socket and removes it afterwards.
WireResponse run(void *engine, const WireRequest &q, const std::string &transfer_path,
                 const ResidentEpochIpcMetadata *ipc) {
  WireResponse r = blank_response(0);
  const bool snapshot = q.operation == kImportExecute;
  r.transport_status = resident_epoch_execute(
      engine, q.request_count, q.max_steps, q.token, q.position, q.seq_len, q.eos, q.generation, r.tokens,
      r.executed, r.generation, &r.model_calls, &r.device_status, &r.feed_calls, &r.fetch_calls, &r.commit_state,
      &r.import_checksum, &r.wall_us, &r.native_cpu_us, &r.declared_input_bytes, &r.declared_output_bytes,
      snapshot ? transfer_path.c_str() : nullptr, q.transfer_id, ipc);
  if (snapshot) unlink(transfer_path.c_str());
  return r;
}

int serve(Channel &client, void *engine, const std::string &transfer_path) {
  for (;;) {
    WireRequest q{};
    if (!client.receive(&q, sizeof(q))) return 68;
    WireResponse r = blank_response(0);
    if (q.magic != kRequestMagic || q.version != CRUISE_SIDECAR_PROTOCOL_VERSION) {
      r.transport_status = 69;
    } else if (q.operation == kShutdown) {
      return client.send(&r, sizeof(r)) ? 0 : 70;
    } else if (q.operation == kDeviceIpcExecute) {
      ResidentEpochIpcMetadata md{};
      if (!client.receive(&md, sizeof(md))) return 73;
      r = run(engine, q, transfer_path, &md);
    } else if (q.operation == kExecute || q.operation == kWarmUp || q.operation == kImportExecute) {
      r = run(engine, q, transfer_path, nullptr);
    } else {
      r.transport_status = 71;
    }
    if (!client.send(&r, sizeof(r))) return 72;
  }
}

}  // namespace

int main(int argc, char **argv) {
  if (argc != 7) {
    std::fprintf(stderr, "usage: %s SOCKET MODEL GRAPH_CONFIG FUNC_CONFIG WEIGHTS TILING\n", argv[0]);
    return 64;
  }
  std::signal(SIGPIPE, SIG_IGN);   // a vanished client is an error return, not a signal
  const std::string transfer_path = std::string(argv[1]) + ".kv-transfer";
  int code = 0;
  {
    Listener listener(argv[1]);
    if (!listener.ok()) return 65;
    const int fd = listener.accept_one();
    if (fd < 0) return 66;
    Channel client(fd);
    int32_t status = -1;
    void *engine = resident_epoch_create(argv[2], argv[3], argv[4], argv[5], argv[6], &status);
    const int32_t startup_status = engine == nullptr ? 100 + status : 0;
    const WireResponse startup = blank_response(startup_status);
    if (!client.send(&startup, sizeof(startup))) {
      code = engine == nullptr ? startup_status : 67;
    } else if (engine == nullptr) {
      code = startup_status;
    } else {
      code = serve(client, engine, transfer_path);
    }
    if (engine != nullptr) resident_epoch_destroy(engine);
  }
  unlink(transfer_path.c_str());
  return code;
}
