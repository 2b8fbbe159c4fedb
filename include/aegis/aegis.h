/* Drop-in include path of the reference (include/aegis/aegis.h): callers and
 * the Rust aegis-sys bindings include "aegis/aegis.h". The declarations live
 * in include/aegis.h. */
#ifndef AEGIS_AEGIS_H
#define AEGIS_AEGIS_H
#include "../aegis.h"
#endif
