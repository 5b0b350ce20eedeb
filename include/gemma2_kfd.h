/* Drop-in for the reference's src/gemma2_kfd.h: the reference's engine
 * (vendor/embeddinggemma.c/src/engine.c, compiled with -DEI_ENABLE_KFD=1)
 * includes "gemma2_kfd.h"; with this directory first on its include path it
 * gets the same three executor entry points (ei_gemma2_kfd_create / _free /
 * _batch, declared in eg2_executor.h) and links them from libeg2_b200.so. */
#ifndef EG2_GEMMA2_KFD_H
#define EG2_GEMMA2_KFD_H
#include "eg2_executor.h"
#endif
