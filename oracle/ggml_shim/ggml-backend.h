// Part of the test-only ggml stand-in: every declaration lives in ggml.h.
#pragma once
#include "ggml.h"
