// Address-space and function qualifiers of MSL, erased for host C++
// (test infrastructure; included only through include/metal_stdlib).
#pragma once
#define kernel
#define device
#define constant const
#define thread
#define threadgroup static
