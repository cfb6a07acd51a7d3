// dual_supplier: a KV-supplier process in native code.
//
// Replaces the Python/ctypes donor side of the reference's supplier lifecycle
// (final/cooperative_4gpu/code/peer/host4.py:47-96, V/nvlink_cooperation/.../cuda_ipc.py:18-88,
// coop/run.py:22-47): it owns one bank of `layers x 2 x slots x 8 x 128` bf16 on its GPU, exports
// it, runs the two-way probe handshake with the compute process, and frees the memory once the
// compute side has unmapped it.  The messages are the ones dual_b200/ipc.py exchanges
// (allocation -> probe_written -> verified -> closed -> freed, or failure), one JSON object per
// line over a Unix-domain stream socket; the 64-byte handle travels as hex.
//
//   dual_supplier --socket PATH --role R --device D --layers L --slots S
//                 [--backend cuda|file] [--dir DIR] [--timeout SEC] [--close-timeout SEC]
//
// backend cuda: cudaMalloc + cudaIpcGetMemHandle on device D (the product path);
// backend file: the bank is the file DIR/bank_<pid>_<role>.bin, mapped with mmap, the handle is
// its name (NUL-padded) -- the same convention as the file-backed memory the CPU tests use.
// Every wait is bounded: no connection, no message or a wrong probe within the timeout ends the
// process with a failure message (if a peer is connected) and exit status 1.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <poll.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/un.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

namespace {

constexpr size_t kSlotBytesPerLayer = 2 * 8 * 128 * 2;  // K + V, 8 kv heads x 128 dims x bf16

uint16_t bf16_bits(float x) {  // exact for the probe values (role + 1.5, role + 2.25)
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return static_cast<uint16_t>(u >> 16);
}

std::string hex(const unsigned char* p, size_t n) {
  static const char* d = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < n; ++i) {
    s += d[p[i] >> 4];
    s += d[p[i] & 15];
  }
  return s;
}

// ------------------------------------------------------------------ memory backends
struct Bank {
  virtual ~Bank() = default;
  virtual void write_u16(uint16_t v) = 0;  // element 0 of the bank
  virtual uint16_t read_u16() = 0;
  virtual std::string handle_hex() = 0;
  virtual void release() = 0;
};

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

struct CudaBank : Bank {
  int device;
  void* ptr = nullptr;
  CudaBank(int dev, size_t bytes) : device(dev) {
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    cuda_check(cudaMalloc(&ptr, bytes), "cudaMalloc");
    cuda_check(cudaMemset(ptr, 0, bytes), "cudaMemset");
    cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  }
  void write_u16(uint16_t v) override {
    cuda_check(cudaMemcpy(ptr, &v, 2, cudaMemcpyHostToDevice), "probe write");
  }
  uint16_t read_u16() override {
    uint16_t v = 0;
    cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    cuda_check(cudaMemcpy(&v, ptr, 2, cudaMemcpyDeviceToHost), "probe read");
    return v;
  }
  std::string handle_hex() override {
    cudaIpcMemHandle_t h;
    cuda_check(cudaIpcGetMemHandle(&h, ptr), "cudaIpcGetMemHandle");
    return hex(reinterpret_cast<const unsigned char*>(&h), sizeof(h));
  }
  void release() override {
    if (ptr) cuda_check(cudaFree(ptr), "cudaFree");
    ptr = nullptr;
  }
  ~CudaBank() override {
    if (ptr) cudaFree(ptr);
  }
};

struct FileBank : Bank {
  std::string dir, name;
  size_t bytes;
  unsigned char* map = nullptr;
  FileBank(const std::string& d, int role, size_t n) : dir(d), bytes(n) {
    name = "bank_" + std::to_string(getpid()) + "_" + std::to_string(role) + ".bin";
    const std::string path = dir + "/" + name;
    const int fd = open(path.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0600);
    if (fd < 0) throw std::runtime_error("open " + path + ": " + std::strerror(errno));
    if (ftruncate(fd, static_cast<off_t>(bytes)) != 0) {
      close(fd);
      throw std::runtime_error("ftruncate: " + std::string(std::strerror(errno)));
    }
    void* m = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) throw std::runtime_error("mmap: " + std::string(std::strerror(errno)));
    map = static_cast<unsigned char*>(m);
  }
  void write_u16(uint16_t v) override {
    std::memcpy(map, &v, 2);
    msync(map, 4096 < bytes ? 4096 : bytes, MS_SYNC);
  }
  uint16_t read_u16() override {
    uint16_t v;
    std::memcpy(&v, const_cast<const unsigned char*>(map), 2);
    return v;
  }
  std::string handle_hex() override {
    unsigned char h[64] = {0};
    std::memcpy(h, name.data(), name.size() < 64 ? name.size() : 64);
    return hex(h, 64);
  }
  void release() override {
    if (map) munmap(map, bytes);
    map = nullptr;
    unlink((dir + "/" + name).c_str());
  }
  ~FileBank() override {
    if (map) release();
  }
};

// ------------------------------------------------------------------ framing: one JSON object per line
struct Conn {
  int fd = -1;
  std::string buf;

  void send_line(const std::string& s) {
    std::string line = s + "\n";
    size_t off = 0;
    while (off < line.size()) {
      const ssize_t n = ::send(fd, line.data() + off, line.size() - off, MSG_NOSIGNAL);
      if (n <= 0) throw std::runtime_error("send failed: peer gone");
      off += size_t(n);
    }
  }

  // next line within `timeout_s` (negative: no limit), or throw
  std::string recv_line(double timeout_s) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      const size_t nl = buf.find('\n');
      if (nl != std::string::npos) {
        std::string line = buf.substr(0, nl);
        buf.erase(0, nl + 1);
        return line;
      }
      int wait_ms = 200;
      if (timeout_s >= 0) {
        const double left = timeout_s - std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (left <= 0) throw std::runtime_error("no message from the compute process within the timeout");
        wait_ms = int(left * 1000) < 200 ? int(left * 1000) + 1 : 200;
      }
      pollfd p{fd, POLLIN, 0};
      const int r = poll(&p, 1, wait_ms);
      if (r < 0 && errno != EINTR) throw std::runtime_error("poll failed");
      if (r > 0) {
        char tmp[4096];
        const ssize_t n = ::recv(fd, tmp, sizeof(tmp), 0);
        if (n <= 0) throw std::runtime_error("compute process closed the connection");
        buf.append(tmp, size_t(n));
      }
    }
  }
};

// value of a string field "key": "..." in a flat JSON object (the messages this service reads)
std::string json_string(const std::string& obj, const std::string& key) {
  const std::string pat = "\"" + key + "\"";
  size_t k = obj.find(pat);
  if (k == std::string::npos) return "";
  k = obj.find(':', k + pat.size());
  if (k == std::string::npos) return "";
  k = obj.find('"', k + 1);
  if (k == std::string::npos) return "";
  const size_t e = obj.find('"', k + 1);
  return e == std::string::npos ? "" : obj.substr(k + 1, e - k - 1);
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += c;
    } else if (c == '\n') {
      o += "\\n";
    } else if (static_cast<unsigned char>(c) >= 0x20) {
      o += c;
    }
  }
  return o;
}

struct Options {
  std::string socket_path, backend = "cuda", dir = ".";
  int role = -1, device = 0;
  long layers = 0, slots = 0;
  double timeout = 120.0, close_timeout = -1.0;  // close_timeout < 0: wait for the compute side's close
};

Options parse(int argc, char** argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (i + 1 >= argc) throw std::runtime_error("missing value for " + a);
    const std::string v = argv[++i];
    if (a == "--socket") o.socket_path = v;
    else if (a == "--role") o.role = std::stoi(v);
    else if (a == "--device") o.device = std::stoi(v);
    else if (a == "--layers") o.layers = std::stol(v);
    else if (a == "--slots") o.slots = std::stol(v);
    else if (a == "--backend") o.backend = v;
    else if (a == "--dir") o.dir = v;
    else if (a == "--timeout") o.timeout = std::stod(v);
    else if (a == "--close-timeout") o.close_timeout = std::stod(v);
    else throw std::runtime_error("unknown option " + a);
  }
  if (o.socket_path.empty() || o.role < 0 || o.layers <= 0 || o.slots <= 0)
    throw std::runtime_error("need --socket, --role >= 0, --layers > 0, --slots > 0");
  if (o.backend != "cuda" && o.backend != "file") throw std::runtime_error("--backend must be cuda or file");
  if (o.socket_path.size() >= sizeof(sockaddr_un::sun_path)) throw std::runtime_error("socket path too long");
  return o;
}

// listen on the socket path and accept the compute process, within `timeout_s`
int accept_one(const std::string& path, double timeout_s) {
  const int ls = socket(AF_UNIX, SOCK_STREAM, 0);
  if (ls < 0) throw std::runtime_error("socket failed");
  sockaddr_un addr{};
  addr.sun_family = AF_UNIX;
  std::strncpy(addr.sun_path, path.c_str(), sizeof(addr.sun_path) - 1);
  unlink(path.c_str());
  if (bind(ls, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0 || listen(ls, 1) != 0) {
    close(ls);
    throw std::runtime_error("cannot listen on " + path + ": " + std::strerror(errno));
  }
  pollfd p{ls, POLLIN, 0};
  const int r = poll(&p, 1, int(timeout_s * 1000));
  if (r <= 0) {
    close(ls);
    unlink(path.c_str());
    throw std::runtime_error("no compute process connected within the timeout");
  }
  const int fd = accept(ls, nullptr, nullptr);
  close(ls);
  unlink(path.c_str());
  if (fd < 0) throw std::runtime_error("accept failed");
  return fd;
}

void expect(const std::string& msg, const char* type) {
  const std::string t = json_string(msg, "type");
  if (t == "failure") throw std::runtime_error("compute process failed: " + json_string(msg, "error"));
  if (t != type) throw std::runtime_error(std::string("expected ") + type + ", got '" + t + "'");
}

}  // namespace

int main(int argc, char** argv) {
  Conn conn;
  Bank* bank = nullptr;
  int role = -1;
  try {
    const Options o = parse(argc, argv);
    role = o.role;
    const size_t bytes = size_t(o.layers) * size_t(o.slots) * kSlotBytesPerLayer;
    if (o.backend == "cuda") bank = new CudaBank(o.device, bytes);
    else bank = new FileBank(o.dir, o.role, bytes);
    bank->write_u16(bf16_bits(float(o.role) + 1.5f));
    const std::string handle = bank->handle_hex();
    conn.fd = accept_one(o.socket_path, o.timeout);
    conn.send_line("{\"type\": \"allocation\", \"role\": " + std::to_string(o.role) +
                   ", \"owner_device\": " + std::to_string(o.device) + ", \"layers\": " + std::to_string(o.layers) +
                   ", \"slots\": " + std::to_string(o.slots) + ", \"bytes\": " + std::to_string(bytes) +
                   ", \"handle\": \"" + handle + "\", \"backend\": \"" + o.backend + "\"}");
    expect(conn.recv_line(o.timeout), "probe_written");
    const uint16_t seen = bank->read_u16();
    if (seen != bf16_bits(float(o.role) + 2.25f))
      throw std::runtime_error("probe write not visible on the supplier (bits " + std::to_string(seen) + ")");
    conn.send_line("{\"type\": \"verified\"}");
    expect(conn.recv_line(o.close_timeout), "closed");
    bank->release();
    delete bank;
    bank = nullptr;
    conn.send_line("{\"type\": \"freed\"}");
    close(conn.fd);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "dual_supplier (role %d): %s\n", role, e.what());
    if (conn.fd >= 0) {
      try {
        conn.send_line("{\"type\": \"failure\", \"role\": " + std::to_string(role) + ", \"error\": \"" +
                       json_escape(e.what()) + "\"}");
      } catch (...) {
      }
      close(conn.fd);
    }
    if (bank) {
      try {
        bank->release();
      } catch (...) {
      }
      delete bank;
    }
    return 1;
  }
}
