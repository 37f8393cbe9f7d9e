// CPU-only stand-in header for the ncnn API subset the reference DiT sources use.
#pragma once
#include "shim_all.h"
