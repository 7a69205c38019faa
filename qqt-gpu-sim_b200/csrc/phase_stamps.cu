// Host side of the phase stamps (qqt_common.cuh): copy out / clear the
// device ring of the phase-stamp build; the regular build has no ring.

extern "C" int qqt_phase_read(uint64_t* host, uint32_t cap, uint32_t* n_out) {
  if (!n_out) return QQT_E_ARG;
  *n_out = 0;
#ifdef QQT_PHASE_STAMPS
  unsigned int n = 0;
  if (cudaMemcpyFromSymbol(&n, qqt::g_ph_n, sizeof(n)) != cudaSuccess) return QQT_E_LAUNCH;
  if (n > QQT_PH_CAP) n = QQT_PH_CAP;
  if (n > cap) n = cap;
  if (n && (!host || cudaMemcpyFromSymbol(host, qqt::g_ph, (size_t)n * 16) != cudaSuccess))
    return host ? QQT_E_LAUNCH : QQT_E_ARG;
  *n_out = n;
  return QQT_OK;
#else
  (void)host;
  (void)cap;
  return QQT_E_ARG;
#endif
}

extern "C" int qqt_phase_reset(void) {
#ifdef QQT_PHASE_STAMPS
  const unsigned int z = 0;
  return cudaMemcpyToSymbol(qqt::g_ph_n, &z, sizeof(z)) == cudaSuccess ? QQT_OK : QQT_E_LAUNCH;
#else
  return QQT_E_ARG;
#endif
}
