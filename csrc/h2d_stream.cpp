// Host -> device layer streaming engine (the low-VRAM path).
//
// The weights of a model's repeated blocks live on the host (pinned RAM copies, or byte ranges of files
// on disk) and reach the GPU through K rotating device slots.  The engine owns one copy stream, one
// worker thread and the events that order everything:
//
//   * the blocks run in a fixed cyclic schedule (block 0..n-1, then again for the next sampling step);
//     the engine keeps the next K entries of that schedule in flight: when compute releases schedule
//     position p, the copy for position p + K is queued into the slot p just vacated;
//   * copy of position q into slot s = q % K:  cudaStreamWaitEvent(copy, compute_done[s]) so the slot's
//     previous occupant has been consumed, then cudaMemcpyAsync from pinned memory (RAM groups) or, for
//     file groups, pread() of the group's extents into a pinned staging buffer (reused once the copy that
//     last read it has completed) followed by cudaMemcpyAsync; then copy_done[s] is recorded;
//   * acquire(position) (compute thread) waits, bounded, until the worker has issued that copy and makes
//     the compute stream wait on copy_done[s]; release() records compute_done[s] on the compute stream and
//     queues position + K.
//
// No thread blocks the GPU: the compute stream only waits on events, and the copy engine moves the
// bytes while the SMs compute the previous block.  With device < 0 the same bookkeeping runs with plain
// memcpy into host "slots" (no CUDA calls), which is how the schedule is tested without a GPU.
//
// Parity: the low-VRAM streaming of dmad_h3/lowmem.py:176-331 (what it does: weights one block ahead of
// compute with two device buffers); the engine, its scheduling and its file reader are this library's.
#include <torch/extension.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace py = pybind11;

namespace dmad {
namespace {

#define H2D_CHECK(call)                                                                          \
  do {                                                                                           \
    cudaError_t err__ = (call);                                                                  \
    if (err__ != cudaSuccess)                                                                    \
      throw std::runtime_error(std::string("h2d stream: ") + #call + ": " + cudaGetErrorString(err__)); \
  } while (0)

struct Extent {
  int file;          // index into files_
  int64_t file_off;  // byte offset in the file
  int64_t nbytes;
  int64_t dst_off;   // byte offset in the group's layout
};

struct Group {
  const uint8_t* ram = nullptr;  // pinned (or, for host mode, plain) copy of the whole layout
  int64_t nbytes = 0;
  std::vector<Extent> extents;   // file group: pieces of the layout read from files
};

struct Pending {
  int64_t position;  // schedule position
  int slot;
  bool issued = false;
};

class H2DStreamer {
 public:
  H2DStreamer(std::vector<int64_t> slot_ptrs, int64_t slot_bytes, int device, std::vector<int64_t> staging_ptrs,
              int64_t staging_bytes, double timeout_s)
      : slot_bytes_(slot_bytes), device_(device), staging_bytes_(staging_bytes), timeout_s_(timeout_s) {
    if (slot_ptrs.size() < 2) throw std::invalid_argument("h2d stream: need at least two slots");
    for (int64_t p : slot_ptrs) slots_.push_back(reinterpret_cast<uint8_t*>(p));
    for (int64_t p : staging_ptrs) staging_.push_back(reinterpret_cast<uint8_t*>(p));
    if (device_ >= 0) {
      H2D_CHECK(cudaSetDevice(device_));
      H2D_CHECK(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
      compute_done_.resize(slots_.size());
      copy_done_.resize(slots_.size());
      for (auto& e : compute_done_) H2D_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      for (auto& e : copy_done_) H2D_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      staged_.resize(staging_.size());
      staged_used_.assign(staging_.size(), false);
      for (auto& e : staged_) H2D_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
  }

  ~H2DStreamer() {
    try {
      close();
    } catch (...) {
    }
    for (int fd : fds_) ::close(fd);
    if (device_ >= 0) {
      cudaSetDevice(device_);
      for (auto e : compute_done_) cudaEventDestroy(e);
      for (auto e : copy_done_) cudaEventDestroy(e);
      for (auto e : staged_) cudaEventDestroy(e);
      if (copy_stream_) cudaStreamDestroy(copy_stream_);
    }
  }

  int add_file(const std::string& path) {
    int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw std::runtime_error("h2d stream: cannot open " + path + ": " + std::strerror(errno));
    fds_.push_back(fd);
    return (int)fds_.size() - 1;
  }

  int add_ram_group(int64_t host_ptr, int64_t nbytes) {
    check_size(nbytes);
    Group g;
    g.ram = reinterpret_cast<const uint8_t*>(host_ptr);
    g.nbytes = nbytes;
    groups_.push_back(std::move(g));
    return (int)groups_.size() - 1;
  }

  int add_file_group(const std::vector<std::vector<int64_t>>& extents, int64_t nbytes) {
    check_size(nbytes);
    if (staging_.empty() || staging_bytes_ < nbytes)
      throw std::invalid_argument("h2d stream: file groups need staging buffers of at least the group size");
    Group g;
    g.nbytes = nbytes;
    for (const auto& e : extents) {
      if (e.size() != 4) throw std::invalid_argument("h2d stream: extent = (file, file_offset, nbytes, dst_offset)");
      if (e[0] < 0 || e[0] >= (int64_t)fds_.size()) throw std::invalid_argument("h2d stream: unknown file index");
      if (e[3] < 0 || e[2] < 0 || e[3] + e[2] > nbytes) throw std::invalid_argument("h2d stream: extent outside group");
      g.extents.push_back({(int)e[0], e[1], e[2], e[3]});
    }
    groups_.push_back(std::move(g));
    return (int)groups_.size() - 1;
  }

  // Starts the cyclic schedule `order` (group indices) and queues its first K positions.
  void start(const std::vector<int64_t>& order) {
    if (worker_.joinable()) throw std::logic_error("h2d stream: already started");
    if (order.size() < 1) throw std::invalid_argument("h2d stream: empty schedule");
    for (int64_t g : order)
      if (g < 0 || g >= (int64_t)groups_.size()) throw std::invalid_argument("h2d stream: schedule names no group");
    order_ = order;
    stop_ = false;
    worker_ = std::thread([this] { run(); });
    std::lock_guard<std::mutex> lk(mu_);
    for (size_t k = 0; k < slots_.size(); ++k) enqueue_locked((int64_t)k);
    cv_work_.notify_all();
  }

  // Blocks (bounded) until the copy of the next schedule position is issued; makes `stream` wait for it.
  // Returns (slot, group) of that position.
  std::pair<int, int64_t> acquire(int64_t stream) {
    std::unique_lock<std::mutex> lk(mu_);
    if (pending_.empty()) throw std::logic_error("h2d stream: acquire without a queued copy (not started?)");
    const auto t0 = std::chrono::steady_clock::now();
    const auto limit = t0 + std::chrono::duration<double>(timeout_s_);
    {
      py::gil_scoped_release nogil;
      while (!pending_.front().issued && error_.empty()) {
        if (cv_done_.wait_until(lk, limit) == std::cv_status::timeout && !pending_.front().issued && error_.empty()) {
          error_ = "timed out after " + std::to_string(timeout_s_) + " s waiting for the copy of schedule position " +
                   std::to_string(pending_.front().position);
          break;
        }
      }
    }
    wait_s_ += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (!error_.empty()) throw std::runtime_error("h2d stream: " + error_);
    Pending& p = pending_.front();
    if (device_ >= 0) H2D_CHECK(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), copy_done_[p.slot], 0));
    acquired_ = true;
    return {p.slot, order_[p.position % order_.size()]};
  }

  // The position acquired last is consumed once `stream` reaches this point; its slot takes position + K.
  void release(int64_t stream) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!acquired_ || pending_.empty()) throw std::logic_error("h2d stream: release without acquire");
    Pending p = pending_.front();
    pending_.pop_front();
    acquired_ = false;
    if (device_ >= 0) H2D_CHECK(cudaEventRecord(compute_done_[p.slot], reinterpret_cast<cudaStream_t>(stream)));
    enqueue_locked(p.position + (int64_t)slots_.size());
    cv_work_.notify_all();
  }

  void close() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      cv_work_.notify_all();
    }
    if (worker_.joinable()) {
      py::gil_scoped_release nogil;
      worker_.join();
    }
    if (device_ >= 0 && copy_stream_) {
      cudaSetDevice(device_);
      cudaStreamSynchronize(copy_stream_);
    }
  }

  py::dict stats() {
    std::lock_guard<std::mutex> lk(mu_);
    py::dict d;
    d["bytes_copied"] = bytes_copied_;
    d["copies"] = copies_;
    d["bytes_read_from_files"] = bytes_read_;
    d["host_wait_s"] = wait_s_;
    d["slots"] = (int64_t)slots_.size();
    d["slot_bytes"] = slot_bytes_;
    return d;
  }

 private:
  void check_size(int64_t nbytes) {
    if (nbytes <= 0 || nbytes > slot_bytes_) throw std::invalid_argument("h2d stream: group larger than a slot");
  }

  void enqueue_locked(int64_t position) {
    Pending p;
    p.position = position;
    p.slot = (int)(position % (int64_t)slots_.size());
    pending_.push_back(p);
    work_.push_back(position);
  }

  void read_extents(const Group& g, uint8_t* dst) {
    for (const Extent& e : g.extents) {
      int64_t done = 0;
      while (done < e.nbytes) {
        ssize_t r = ::pread(fds_[e.file], dst + e.dst_off + done, (size_t)(e.nbytes - done), e.file_off + done);
        if (r <= 0) throw std::runtime_error(std::string("h2d stream: short read: ") + (r < 0 ? std::strerror(errno) : "end of file"));
        done += r;
      }
      bytes_read_ += e.nbytes;
    }
  }

  void run() {
    try {
      if (device_ >= 0) H2D_CHECK(cudaSetDevice(device_));
      int64_t staging_seq = 0;
      for (;;) {
        int64_t position;
        {
          std::unique_lock<std::mutex> lk(mu_);
          cv_work_.wait(lk, [this] { return stop_ || !work_.empty(); });
          if (stop_) return;
          position = work_.front();
          work_.pop_front();
        }
        const int slot = (int)(position % (int64_t)slots_.size());
        const Group& g = groups_[order_[position % order_.size()]];
        uint8_t* dst = slots_[slot];
        if (device_ < 0) {  // host mode: synchronous copies, same schedule
          if (g.ram) {
            std::memcpy(dst, g.ram, (size_t)g.nbytes);
          } else {
            read_extents(g, dst);
          }
        } else {
          H2D_CHECK(cudaStreamWaitEvent(copy_stream_, compute_done_[slot], 0));
          if (g.ram) {
            H2D_CHECK(cudaMemcpyAsync(dst, g.ram, (size_t)g.nbytes, cudaMemcpyHostToDevice, copy_stream_));
          } else {
            const size_t b = (size_t)(staging_seq++ % (int64_t)staging_.size());
            if (staged_used_[b]) H2D_CHECK(cudaEventSynchronize(staged_[b]));  // its last copy has read it
            read_extents(g, staging_[b]);
            H2D_CHECK(cudaMemcpyAsync(dst, staging_[b], (size_t)g.nbytes, cudaMemcpyHostToDevice, copy_stream_));
            H2D_CHECK(cudaEventRecord(staged_[b], copy_stream_));
            staged_used_[b] = true;
          }
          H2D_CHECK(cudaEventRecord(copy_done_[slot], copy_stream_));
        }
        std::lock_guard<std::mutex> lk(mu_);
        for (auto& p : pending_)
          if (p.position == position) p.issued = true;
        bytes_copied_ += g.nbytes;
        copies_ += 1;
        cv_done_.notify_all();
      }
    } catch (const std::exception& e) {  // reported to the compute thread by its next acquire
      std::lock_guard<std::mutex> lk(mu_);
      error_ = e.what();
      cv_done_.notify_all();
    }
  }

  std::vector<uint8_t*> slots_;
  int64_t slot_bytes_;
  int device_;
  std::vector<uint8_t*> staging_;
  int64_t staging_bytes_;
  double timeout_s_;
  std::vector<int> fds_;
  std::vector<Group> groups_;
  std::vector<int64_t> order_;

  cudaStream_t copy_stream_ = nullptr;
  std::vector<cudaEvent_t> compute_done_, copy_done_, staged_;
  std::vector<bool> staged_used_;

  std::mutex mu_;
  std::condition_variable cv_work_, cv_done_;
  std::deque<Pending> pending_;
  std::deque<int64_t> work_;
  bool stop_ = false;
  bool acquired_ = false;
  std::string error_;
  std::thread worker_;

  int64_t bytes_copied_ = 0, copies_ = 0, bytes_read_ = 0;
  double wait_s_ = 0.0;
};

}  // namespace

void register_h2d_stream(py::module& m) {
  py::class_<H2DStreamer>(m, "H2DStreamer")
      .def(py::init<std::vector<int64_t>, int64_t, int, std::vector<int64_t>, int64_t, double>(), py::arg("slot_ptrs"),
           py::arg("slot_bytes"), py::arg("device"), py::arg("staging_ptrs"), py::arg("staging_bytes"),
           py::arg("timeout_s"))
      .def("add_file", &H2DStreamer::add_file)
      .def("add_ram_group", &H2DStreamer::add_ram_group)
      .def("add_file_group", &H2DStreamer::add_file_group)
      .def("start", &H2DStreamer::start)
      .def("acquire", &H2DStreamer::acquire)
      .def("release", &H2DStreamer::release)
      .def("close", &H2DStreamer::close)
      .def("stats", &H2DStreamer::stats);
}

}  // namespace dmad
