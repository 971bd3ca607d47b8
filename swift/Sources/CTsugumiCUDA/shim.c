/* SwiftPM builds a C target from at least one source file; the symbols come
 * from libtsugumi_cuda.so, which the module map links.  This file only pins
 * the ABI version the Swift side was written against. */
#include "tsugumi_cuda.h"

#if TSG_ABI_VERSION != 1
#error "TsugumiCUDA.swift targets TSG_ABI_VERSION 1"
#endif
