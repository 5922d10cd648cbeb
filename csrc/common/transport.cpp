#include "ofld/transport.h"

#include <arpa/inet.h>
#include <errno.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

#include "ofld/log.h"

namespace ofld {

namespace {
[[noreturn]] void sys_fail(const char* what) {
    throw std::runtime_error(std::string(what) + ": " + std::strerror(errno));
}

void send_all_or_throw(int s, const uint8_t* p, size_t n) {
    while (n > 0) {
        ssize_t w = ::send(s, p, n, MSG_NOSIGNAL);
        if (w < 0) {
            if (errno == EINTR) continue;
            sys_fail("send");
        }
        if (w == 0) throw std::runtime_error("send: peer closed");
        p += w;
        n -= static_cast<size_t>(w);
    }
}
}  // namespace

bool write_all(int fd, const void* p, size_t n) {
    const uint8_t* c = static_cast<const uint8_t*>(p);
    while (n > 0) {
        ssize_t w = ::write(fd, c, n);
        if (w < 0) {
            if (errno == EINTR) continue;
            return false;
        }
        if (w == 0) return false;
        c += w;
        n -= static_cast<size_t>(w);
    }
    return true;
}

bool read_all(int fd, void* p, size_t n) {
    uint8_t* c = static_cast<uint8_t*>(p);
    while (n > 0) {
        ssize_t r = ::read(fd, c, n);
        if (r < 0) {
            if (errno == EINTR) continue;
            return false;
        }
        if (r == 0) return false;
        c += r;
        n -= static_cast<size_t>(r);
    }
    return true;
}

void send_frame(int sock, const std::vector<uint8_t>& frame, const std::vector<int>& fds) {
    if (frame.size() < kFrameHeaderSize) throw std::runtime_error("send_frame: short frame");
    if (fds.empty()) {
        send_all_or_throw(sock, frame.data(), frame.size());
        return;
    }
    if (fds.size() > static_cast<size_t>(kMaxFdsPerFrame))
        throw std::runtime_error("send_frame: too many fds");
    // Header bytes carry the ancillary fds; continue with plain sends.
    alignas(cmsghdr) char cbuf[CMSG_SPACE(sizeof(int) * kMaxFdsPerFrame)];
    std::memset(cbuf, 0, sizeof(cbuf));
    msghdr msg{};
    iovec iov{const_cast<uint8_t*>(frame.data()), kFrameHeaderSize};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    msg.msg_control = cbuf;
    msg.msg_controllen = CMSG_SPACE(sizeof(int) * fds.size());
    cmsghdr* c = CMSG_FIRSTHDR(&msg);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int) * fds.size());
    std::memcpy(CMSG_DATA(c), fds.data(), sizeof(int) * fds.size());
    size_t sent = 0;
    while (sent < kFrameHeaderSize) {
        iov.iov_base = const_cast<uint8_t*>(frame.data()) + sent;
        iov.iov_len = kFrameHeaderSize - sent;
        ssize_t w = ::sendmsg(sock, &msg, MSG_NOSIGNAL);
        if (w < 0) {
            if (errno == EINTR) continue;
            sys_fail("sendmsg");
        }
        sent += static_cast<size_t>(w);
        msg.msg_control = nullptr;  // fds went with the first successful send
        msg.msg_controllen = 0;
    }
    if (frame.size() > kFrameHeaderSize)
        send_all_or_throw(sock, frame.data() + kFrameHeaderSize, frame.size() - kFrameHeaderSize);
}

bool recv_frame(int sock, Op* op, std::vector<uint8_t>* payload, std::vector<int>* fds) {
    if (fds) fds->clear();
    uint8_t hdr[kFrameHeaderSize];
    alignas(cmsghdr) char cbuf[CMSG_SPACE(sizeof(int) * kMaxFdsPerFrame)];
    size_t got = 0;
    bool first = true;
    while (got < kFrameHeaderSize) {
        msghdr msg{};
        iovec iov{hdr + got, kFrameHeaderSize - got};
        msg.msg_iov = &iov;
        msg.msg_iovlen = 1;
        if (first) {
            msg.msg_control = cbuf;
            msg.msg_controllen = sizeof(cbuf);
        }
        ssize_t r = ::recvmsg(sock, &msg, MSG_CMSG_CLOEXEC);
        if (r < 0) {
            if (errno == EINTR) continue;
            sys_fail("recvmsg");
        }
        if (r == 0) {
            if (got == 0) return false;
            throw std::runtime_error("recvmsg: EOF inside frame header");
        }
        if (first) {
            for (cmsghdr* c = CMSG_FIRSTHDR(&msg); c; c = CMSG_NXTHDR(&msg, c)) {
                if (c->cmsg_level != SOL_SOCKET || c->cmsg_type != SCM_RIGHTS) continue;
                size_t cnt = (c->cmsg_len - CMSG_LEN(0)) / sizeof(int);
                const int* fp = reinterpret_cast<const int*>(CMSG_DATA(c));
                for (size_t i = 0; i < cnt; ++i) {
                    if (fds)
                        fds->push_back(fp[i]);
                    else
                        ::close(fp[i]);
                }
            }
        }
        first = false;
        got += static_cast<size_t>(r);
    }
    FrameHeader h = parse_frame_header(hdr, kFrameHeaderSize);
    if (h.payload_len > kMaxFramePayload) throw std::runtime_error("frame payload too large");
    if (op) *op = static_cast<Op>(h.opcode);
    std::vector<uint8_t> scratch;
    std::vector<uint8_t>* dst = payload ? payload : &scratch;
    dst->resize(h.payload_len);
    size_t off = 0;
    while (off < h.payload_len) {
        ssize_t r = ::recv(sock, dst->data() + off, h.payload_len - off, 0);
        if (r < 0) {
            if (errno == EINTR) continue;
            sys_fail("recv");
        }
        if (r == 0) throw std::runtime_error("recv: EOF inside frame payload");
        off += static_cast<size_t>(r);
    }
    return true;
}

int uds_listen(const std::string& path, int backlog) {
    sockaddr_un addr{};
    if (path.size() >= sizeof(addr.sun_path)) throw std::runtime_error("socket path too long");
    int fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) sys_fail("socket(AF_UNIX)");
    ::unlink(path.c_str());
    addr.sun_family = AF_UNIX;
    std::memcpy(addr.sun_path, path.c_str(), path.size());
    if (::bind(fd, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) < 0 ||
        ::listen(fd, backlog) < 0) {
        int e = errno;
        ::close(fd);
        errno = e;
        sys_fail(("bind/listen " + path).c_str());
    }
    return fd;
}

int tcp_listen(uint16_t port, int backlog, const char* bind_addr) {
    int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) sys_fail("socket(AF_INET)");
    int one = 1;
    ::setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons(port);
    a.sin_addr.s_addr = bind_addr ? inet_addr(bind_addr) : htonl(INADDR_ANY);
    if (::bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) < 0 || ::listen(fd, backlog) < 0) {
        int e = errno;
        ::close(fd);
        errno = e;
        sys_fail("tcp bind/listen");
    }
    return fd;
}

int accept_conn(int listen_fd) {
    int fd = ::accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
    if (fd < 0) {
        if (errno == EINTR || errno == EAGAIN || errno == ECONNABORTED) return -1;
        sys_fail("accept");
    }
    int one = 1;
    ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));  // no-op on AF_UNIX
    return fd;
}

int uds_connect(const std::string& path, int timeout_ms) {
    sockaddr_un addr{};
    if (path.size() >= sizeof(addr.sun_path)) throw std::runtime_error("socket path too long");
    addr.sun_family = AF_UNIX;
    std::memcpy(addr.sun_path, path.c_str(), path.size());
    uint64_t deadline = mono_ns() + uint64_t(timeout_ms) * 1000000ull;
    for (;;) {
        int fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (fd < 0) sys_fail("socket(AF_UNIX)");
        if (::connect(fd, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) == 0) return fd;
        int e = errno;
        ::close(fd);
        if ((e == ENOENT || e == ECONNREFUSED || e == EAGAIN) && mono_ns() < deadline) {
            sleep_us(20000);
            continue;
        }
        errno = e;
        sys_fail(("connect " + path).c_str());
    }
}

int tcp_connect(const std::string& host, uint16_t port, int timeout_ms) {
    addrinfo hints{};
    hints.ai_family = AF_UNSPEC;
    hints.ai_socktype = SOCK_STREAM;
    addrinfo* res = nullptr;
    std::string ps = std::to_string(port);
    uint64_t deadline = mono_ns() + uint64_t(timeout_ms) * 1000000ull;
    for (;;) {
        if (::getaddrinfo(host.c_str(), ps.c_str(), &hints, &res) != 0 || !res)
            throw std::runtime_error("getaddrinfo failed for " + host);
        int fd = -1;
        for (addrinfo* ai = res; ai; ai = ai->ai_next) {
            fd = ::socket(ai->ai_family, ai->ai_socktype | SOCK_CLOEXEC, ai->ai_protocol);
            if (fd < 0) continue;
            if (::connect(fd, ai->ai_addr, ai->ai_addrlen) == 0) break;
            ::close(fd);
            fd = -1;
        }
        ::freeaddrinfo(res);
        if (fd >= 0) {
            int one = 1;
            ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
            return fd;
        }
        if (mono_ns() >= deadline) throw std::runtime_error("tcp connect failed: " + host);
        sleep_us(20000);
    }
}

void close_fd(int fd) {
    if (fd >= 0) ::close(fd);
}

bool split_host_port(const std::string& s, std::string* host, uint16_t* port) {
    size_t c = s.rfind(':');
    if (c == std::string::npos || c == 0 || c + 1 >= s.size()) return false;
    char* end = nullptr;
    unsigned long p = std::strtoul(s.c_str() + c + 1, &end, 10);
    if (*end != '\0' || p == 0 || p > 65535) return false;
    *host = s.substr(0, c);
    *port = static_cast<uint16_t>(p);
    return true;
}

void RpcClient::roundtrip(Op op, const std::vector<uint8_t>& body, const std::vector<int>& fds_in,
                          std::vector<uint8_t>* reply, std::vector<int>* fds_out) {
    std::lock_guard<std::mutex> g(mu_);
    send_frame(sock_, make_frame(op, body), fds_in);
    Op rop = Op::kInvalid;
    std::vector<int> fds;
    if (!recv_frame(sock_, &rop, reply, &fds)) throw std::runtime_error("rpc: daemon closed connection");
    if (rop != op) {
        for (int f : fds) ::close(f);
        throw std::runtime_error(std::string("rpc: reply opcode mismatch for ") + op_name(op));
    }
    if (fds_out)
        *fds_out = std::move(fds);
    else
        for (int f : fds) ::close(f);
}

}  // namespace ofld
