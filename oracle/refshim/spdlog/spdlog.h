// Logging stand-in used only to compile the reference's own search sources
// into the test oracle (oracle/_ref). The reference logs through spdlog, whose
// submodule is empty here; its log macros expand to nothing.
#pragma once
#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <pthread.h>
#include <sched.h>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#define SPDLOG_LEVEL_TRACE 0
#define SPDLOG_INFO(...) ((void)0)
#define SPDLOG_DEBUG(...) ((void)0)
#define SPDLOG_WARN(...) ((void)0)
#define SPDLOG_ERROR(...) ((void)0)
