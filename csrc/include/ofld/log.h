// Clocks and leveled stderr logging.
//
// OFLD_LOG_LEVEL selects 0=error, 1=warn, 2=info (default), 3=debug, the same
// variable and scale StateSpectre uses (reference: src/common/util.h:26-38).
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <ctime>
#include <mutex>

namespace ofld {

inline uint64_t mono_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return uint64_t(ts.tv_sec) * 1000000000ull + uint64_t(ts.tv_nsec);
}
inline uint64_t real_ns() {
    timespec ts;
    clock_gettime(CLOCK_REALTIME, &ts);
    return uint64_t(ts.tv_sec) * 1000000000ull + uint64_t(ts.tv_nsec);
}
inline void sleep_us(uint64_t us) {
    timespec ts{static_cast<time_t>(us / 1000000ull), static_cast<long>((us % 1000000ull) * 1000)};
    nanosleep(&ts, nullptr);
}

enum class Level : int { kError = 0, kWarn = 1, kInfo = 2, kDebug = 3 };

inline int log_level() {
    static const int lvl = [] {
        const char* e = std::getenv("OFLD_LOG_LEVEL");
        int v = e ? std::atoi(e) : 2;
        return v < 0 ? 0 : (v > 3 ? 3 : v);
    }();
    return lvl;
}

void log_write(Level lvl, const char* tag, const char* fmt, ...)
    __attribute__((format(printf, 3, 4)));

}  // namespace ofld

#define OFLD_LOG(lvl, tag, ...)                                                  \
    do {                                                                         \
        if (static_cast<int>(lvl) <= ::ofld::log_level())                        \
            ::ofld::log_write(lvl, tag, __VA_ARGS__);                            \
    } while (0)
#define LOG_ERR(tag, ...) OFLD_LOG(::ofld::Level::kError, tag, __VA_ARGS__)
#define LOG_WARN(tag, ...) OFLD_LOG(::ofld::Level::kWarn, tag, __VA_ARGS__)
#define LOG_INFO(tag, ...) OFLD_LOG(::ofld::Level::kInfo, tag, __VA_ARGS__)
#define LOG_DEBUG(tag, ...) OFLD_LOG(::ofld::Level::kDebug, tag, __VA_ARGS__)
