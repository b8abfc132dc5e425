// See ../spdlog.h: part of the logging stand-in for the reference build.
#pragma once
