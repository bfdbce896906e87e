/* ORACLE build shim: stand-in for the sysdef.h of CrossCache's absent
 * infrastructure submodule (only sys_assert is used by mem.cpp). */
#ifndef ORACLE_REFSHIM_SYSDEF_H
#define ORACLE_REFSHIM_SYSDEF_H
#include <stdlib.h>
#define sys_assert(x) do { if (!(x)) abort(); } while (0)
#endif
