/* Stubs for the three Win32 imports the reference declares (executable
 * directory lookup and peak-RAM query).  Test infrastructure only: with these
 * the reference links on Linux; neither value feeds any arithmetic. */
unsigned long GetModuleFileNameA(void *m, char *buf, unsigned long n)
{ (void)m; (void)buf; (void)n; return 0; }
void *GetCurrentProcess(void) { return 0; }
int K32GetProcessMemoryInfo(void *p, void *c, unsigned long n)
{ (void)p; (void)c; (void)n; return 0; }
