// Stream-socket transport for framed RPC: AF_UNIX (with SCM_RIGHTS fd passing)
// and TCP. Semantics follow StateSpectre's uds.cpp (reference:
// src/common/uds.cpp:57-274): fds ride the first sendmsg that carries the
// 12-byte header, at most 32 per frame; payloads over 256 MiB are rejected;
// connect retries while the listener is not up yet.
#pragma once

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "ofld/codec.h"

namespace ofld {

constexpr int kMaxFdsPerFrame = 32;

// Send one frame; `fds` (may be empty) are attached to the header bytes.
void send_frame(int sock, const std::vector<uint8_t>& frame, const std::vector<int>& fds = {});
// Receive one frame. Returns false on clean EOF at a frame boundary.
bool recv_frame(int sock, Op* op, std::vector<uint8_t>* payload, std::vector<int>* fds);

int uds_listen(const std::string& path, int backlog = 128);
int tcp_listen(uint16_t port, int backlog = 128, const char* bind_addr = nullptr);
int accept_conn(int listen_fd);  // -1 on EINTR/EAGAIN
int uds_connect(const std::string& path, int timeout_ms = 10000);
int tcp_connect(const std::string& host, uint16_t port, int timeout_ms = 10000);
void close_fd(int fd);
// Split "host:port"; false if malformed.
bool split_host_port(const std::string& s, std::string* host, uint16_t* port);
bool write_all(int fd, const void* p, size_t n);
bool read_all(int fd, void* p, size_t n);

// Synchronous request/response client over one connected socket. A mutex
// serialises whole round trips so any thread may call. The reply opcode must
// match the request's.
class RpcClient {
 public:
    explicit RpcClient(int sock) : sock_(sock) {}
    ~RpcClient() { close_fd(sock_); }
    RpcClient(const RpcClient&) = delete;
    RpcClient& operator=(const RpcClient&) = delete;

    template <Op O>
    typename OpTypes<O>::Response call(const typename OpTypes<O>::Request& req,
                                       std::vector<int>* fds_out = nullptr,
                                       const std::vector<int>& fds_in = {}) {
        std::vector<uint8_t> reply;
        roundtrip(O, encode(req), fds_in, &reply, fds_out);
        return decode<typename OpTypes<O>::Response>(reply);
    }
    int fd() const { return sock_; }

 private:
    void roundtrip(Op op, const std::vector<uint8_t>& body, const std::vector<int>& fds_in,
                   std::vector<uint8_t>* reply, std::vector<int>* fds_out);
    int sock_;
    std::mutex mu_;
};

}  // namespace ofld
