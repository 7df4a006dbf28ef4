/* Linux stand-in for the Windows <direct.h> that the reference includes.
 * Test infrastructure only: it lets the reference's single C file compile here
 * so its own CPU functions can serve as the parity oracle. */
#ifndef TLREF_SHIM_DIRECT_H
#define TLREF_SHIM_DIRECT_H
#include <sys/stat.h>
#include <sys/types.h>
#include <stdio.h>
#define _mkdir(p) mkdir((p), 0755)
#define _fseeki64(f, o, w) fseeko((f), (off_t)(o), (w))
#define _ftelli64(f) ((long long)ftello(f))
#endif
