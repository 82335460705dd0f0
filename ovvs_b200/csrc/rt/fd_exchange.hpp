// File-descriptor exchange between the ranks of one communicator on one host, over Unix-domain
// sockets in the abstract namespace (no file system entry). Each rank serves one descriptor to
// every peer and receives every peer's descriptor (SCM_RIGHTS); the kernel duplicates a
// descriptor into the receiving process, so the receiver holds its own reference to the object
// behind it (here: a CUDA physical allocation exported as a POSIX file descriptor).
//
// Every step is bounded by a deadline: a peer that never appears gives an error, not a hang.
// Connections are accepted only from processes of the same user (SO_PEERCRED).
#pragma once

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

namespace ovvs {
namespace rt {

inline int64_t fdx_now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

// Abstract socket address of `rank` for exchange `tag`.
inline socklen_t fdx_address(uint64_t tag, int rank, sockaddr_un* a) {
  std::memset(a, 0, sizeof(*a));
  a->sun_family = AF_UNIX;
  const int len = std::snprintf(a->sun_path + 1, sizeof(a->sun_path) - 1, "ovvs-fdx-%016llx-%d",
                                static_cast<unsigned long long>(tag), rank);
  return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + len);
}

// Sends `fd` over the connected socket `s` (one payload byte carries the descriptor).
inline bool fdx_send_fd(int s, int fd) {
  char byte = 'f';
  iovec iov{&byte, 1};
  alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))];
  std::memset(ctrl, 0, sizeof(ctrl));
  msghdr m{};
  m.msg_iov = &iov;
  m.msg_iovlen = 1;
  m.msg_control = ctrl;
  m.msg_controllen = sizeof(ctrl);
  cmsghdr* c = CMSG_FIRSTHDR(&m);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int));
  std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
  return sendmsg(s, &m, MSG_NOSIGNAL) == 1;
}

// Receives one descriptor from `s`, waiting at most until `deadline_ms`; -1 on failure.
inline int fdx_recv_fd(int s, int64_t deadline_ms) {
  pollfd p{s, POLLIN, 0};
  const int64_t left = deadline_ms - fdx_now_ms();
  if (left <= 0 || poll(&p, 1, static_cast<int>(left)) != 1) return -1;
  char byte = 0;
  iovec iov{&byte, 1};
  alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))];
  msghdr m{};
  m.msg_iov = &iov;
  m.msg_iovlen = 1;
  m.msg_control = ctrl;
  m.msg_controllen = sizeof(ctrl);
  if (recvmsg(s, &m, MSG_CMSG_CLOEXEC) != 1) return -1;
  for (cmsghdr* c = CMSG_FIRSTHDR(&m); c; c = CMSG_NXTHDR(&m, c)) {
    if (c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS &&
        c->cmsg_len == CMSG_LEN(sizeof(int))) {
      int fd = -1;
      std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
      return fd;
    }
  }
  return -1;
}

// Exchanges descriptors among `world` ranks: rank `rank` offers `my_fd` and, on success, gets
// peer_fd[p] (a descriptor of its own, to be closed by the caller) for every p != rank, and
// peer_fd[rank] = -1. All ranks must call this with the same tag; `tag` must differ between
// concurrent exchanges on the host. Returns false (and closes whatever it received) when a peer
// does not show up before `timeout_ms`.
inline bool exchange_fds(uint64_t tag, int rank, int world, int my_fd, std::vector<int>& peer_fd,
                         int64_t timeout_ms) {
  peer_fd.assign(static_cast<size_t>(world), -1);
  if (world <= 1) return true;
  const int64_t deadline = fdx_now_ms() + timeout_ms;
  const int srv = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (srv < 0) return false;
  sockaddr_un addr;
  const socklen_t alen = fdx_address(tag, rank, &addr);
  if (bind(srv, reinterpret_cast<sockaddr*>(&addr), alen) != 0 || listen(srv, world) != 0) {
    close(srv);
    return false;
  }
  // Serve the descriptor to world - 1 peers while fetching theirs.
  std::atomic<bool> served_ok{true}, stop{false};
  std::thread server([&] {
    for (int served = 0; served < world - 1;) {
      pollfd p{srv, POLLIN, 0};
      const int64_t left = deadline - fdx_now_ms();
      if (left <= 0 || stop.load()) {
        served_ok = false;
        return;
      }
      // short slices, so that a failed fetch below ends the serving early
      if (poll(&p, 1, static_cast<int>(left < 20 ? left : 20)) != 1) continue;
      const int c = accept4(srv, nullptr, nullptr, SOCK_CLOEXEC);
      if (c < 0) continue;
      ucred cred{};
      socklen_t cl = sizeof(cred);
      const bool same_user = getsockopt(c, SOL_SOCKET, SO_PEERCRED, &cred, &cl) == 0 &&
                             cred.uid == getuid();
      if (same_user && fdx_send_fd(c, my_fd)) ++served;
      close(c);
    }
  });
  bool ok = true;
  for (int p = 0; p < world && ok; ++p) {
    if (p == rank) continue;
    sockaddr_un pa;
    const socklen_t pl = fdx_address(tag, p, &pa);
    int fd = -1;
    while (fd < 0) {
      const int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
      if (s < 0) break;
      if (connect(s, reinterpret_cast<sockaddr*>(&pa), pl) == 0) fd = fdx_recv_fd(s, deadline);
      close(s);
      if (fd >= 0 || fdx_now_ms() >= deadline) break;
      std::this_thread::sleep_for(std::chrono::milliseconds(1));  // peer not listening yet
    }
    if (fd < 0) ok = false;
    peer_fd[static_cast<size_t>(p)] = fd;
  }
  if (!ok) stop = true;
  server.join();
  close(srv);
  ok = ok && served_ok.load();
  if (!ok) {
    for (int& fd : peer_fd) {
      if (fd >= 0) close(fd);
      fd = -1;
    }
  }
  return ok;
}

}  // namespace rt
}  // namespace ovvs
